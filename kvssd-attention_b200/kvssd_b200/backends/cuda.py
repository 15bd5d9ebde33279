"""The B200 attention backend, registered under kvssd's name ``cuda``.

Drop-in for CudaExtensionBackend (src/kvssd/backends/cuda.py:17-48): same name, probe
semantics (available only on a CUDA device with the native library present; always
``accelerated``) and run contract, but ``run`` calls libkvssd_b200's split-KV tensor-core
kernel through the C ABI instead of the kvssd._C extension. It duck-types its ``batch``
argument, so kvssd's own PackedBatch works too.
"""

from __future__ import annotations

import torch

from .. import _native, ops
from .base import BackendAvailability, PackedBatch

SM100 = (10, 0)


class B200AttentionBackend:
    name = "cuda"

    def probe(self, device: torch.device) -> BackendAvailability:
        device = torch.device(device)
        if device.type != "cuda":
            reason = f"CUDA extension requires a CUDA device, got {device.type}"
            return BackendAvailability(self.name, False, True, False, reason, device.type)
        if not _native.available():
            reason = "libkvssd_b200 not built; run `python -m kvssd_b200._build`"
            return BackendAvailability(self.name, False, True, False, reason, device.type)
        if not torch.cuda.is_available():
            return BackendAvailability(self.name, False, True, False, "CUDA is unavailable",
                                       device.type)
        index = device.index if device.index is not None else torch.cuda.current_device()
        cap = torch.cuda.get_device_capability(index)
        if cap != SM100:
            reason = f"kernels are built for sm_100a (B200); device has sm_{cap[0]}{cap[1]}"
            return BackendAvailability(self.name, False, True, False, reason, device.type)
        return BackendAvailability(self.name, True, True, False,
                                   "B200 sm_100a split-KV decode kernels are available",
                                   device.type)

    def run(
        self, query: torch.Tensor, batch: PackedBatch, sm_scale: float
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """(out fp32 [QH, D], lse fp32 [QH]) on the current stream, without synchronising.

        Kernel failures surface the way the reference's TORCH_CHECK does, as an exception,
        but without a host synchronisation per call: the call's device status word is copied
        into pinned memory after its kernels, and a later ``run`` on the same stream raises
        ops.DeviceFailure (a RuntimeError) if that word flagged a failure -- the first one
        after the copy has landed, and at the latest the fourth, which waits for it -- as does
        ``check``, which waits. The failed call's own out/lse are NaN, and so are those of every
        call after it until the word is cleared, so nothing plausible is returned meanwhile.
        """
        PackedBatch.validate(batch, query)
        if query.device.type != "cuda":
            raise RuntimeError(f"CUDA extension requires a CUDA device, got {query.device.type}")
        if not _native.available():
            raise RuntimeError("CUDA extension unavailable; run `python -m kvssd_b200._build`")
        watch = ops.status_watch(query.device)
        watch.poll("B200AttentionBackend.run (an earlier call)")
        result = ops.decode(
            query,
            batch.packed_k.contiguous(),
            batch.packed_v.contiguous(),
            batch.scales_k.contiguous(),
            batch.scales_v.contiguous(),
            batch.valid_tokens.to(torch.int32).contiguous(),
            batch.bits,
            batch.group_size,
            sm_scale,
        )
        watch.arm("B200AttentionBackend.run")
        return result

    def check(self, device: torch.device | str | None = None) -> None:
        """Waits for this stream's outstanding status reads and raises ops.DeviceFailure if
        any call on it flagged a failure."""
        device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        ops.status_watch(device).check("B200AttentionBackend.run")
