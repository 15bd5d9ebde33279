"""KVSSDPipeline: selection -> record reads -> on-GPU record decode -> fused decode -> exact merge.

API of src/kvssd/pipeline.py:19-196 (constructor arguments, ``decode(query, layer,
selector)``, context manager). Execution is CUDA-only. The selected records are read chunk by
chunk (``stage_blocks`` records) by the native reader (``io_depth`` threads, O_DIRECT where
the file system allows it) into two reusable pinned buffers; each chunk is copied to the device
on a transfer stream as one transfer, and on a compute stream, as soon as its copy lands, the
records are decoded into PackedBatch tensors with their headers and payload CRC-32 checked on
the GPU (ops.decode_records) and attended by the fused decode kernel. Reading chunk i + 1 on
the host overlaps the GPU work of chunk i. The per-chunk (out, lse) pairs are merged exactly
by one N-way merge kernel (the reference chains one pairwise merge per chunk). A store opened
with the ``gds`` storage backend skips the pinned buffers and the copy: cuFile reads each chunk
straight into one of two aligned device buffers, and one opened with ``mapped`` copies the
records into them by DMA from the page-locked file mapping on the transfer stream. The records'
integrity statuses are read back once at the end: a bad record raises as kvssd's decode_record
does (ValueError for a bad header or layout, IOError for a CRC mismatch). For a layer that stays
resident in HBM use DeviceBlockPool, which decodes with a single launch.
"""

from __future__ import annotations

import math

import torch

from . import ops
from .attention import select_backend
from .backends import AttentionBackend, PackedBatch
from .backends.cuda import B200AttentionBackend
from .selectors import AllBlocks, BlockSelector


class _PinnedChunk:
    """Pinned raw records of one chunk plus the event of its last host-to-device copy."""

    def __init__(self, spec, blocks: int):
        self.raw = torch.empty((blocks, spec.record_bytes), dtype=torch.uint8,
                               pin_memory=torch.cuda.is_available())
        self.copied: torch.cuda.Event | None = None


class KVSSDPipeline:
    """End-to-end selection, native record reads, on-GPU record decode and fused attention."""

    def __init__(
        self,
        store,
        device: str | torch.device = "cuda",
        io_depth: int = 2,
        stage_blocks: int = 4,
        require_cuda_kernel: bool = False,
        attention_backend: str | AttentionBackend | None = None,
    ):
        self.store = store
        self.device = torch.device(device)
        if self.device.type == "cuda" and not torch.cuda.is_available():
            raise RuntimeError("CUDA device requested but CUDA is unavailable")
        if io_depth < 1:
            raise ValueError("io_depth must be positive")
        if stage_blocks < 1:
            raise ValueError("stage_blocks must be positive")
        self.attention_backend = select_backend(self.device, require_cuda_kernel,
                                                attention_backend)
        self.io_depth = io_depth
        self.stage_blocks = stage_blocks
        self.require_cuda_kernel = require_cuda_kernel
        self.transfer_stream = torch.cuda.Stream(device=self.device)
        self.compute_stream = torch.cuda.Stream(device=self.device)
        self._ring = [_PinnedChunk(store.spec, stage_blocks) for _ in range(2)]
        # gds / mapped storage: records land in device memory by cuFile or by DMA from the
        # page-locked file mapping, with no pinned staging buffer
        self._device_ring = None
        if store.reads_to_device:
            from .storage import _aligned

            rb = store.spec.record_bytes
            self._device_ring = [_aligned(stage_blocks * rb, self.device) for _ in range(2)]
            self._device_free = [None, None]  # event: the compute stream is done with a buffer

    def decode(self, query: torch.Tensor, layer: int,
               selector: BlockSelector | None = None) -> torch.Tensor:
        selector = selector or AllBlocks()
        selected = selector.select(self.store.blocks_for_layer(layer))
        if not selected:
            raise ValueError("selector returned no blocks")
        query = query.to(self.device)
        spec = self.store.spec
        scale = 1.0 / math.sqrt(query.shape[-1])
        n_chunks = -(-len(selected) // self.stage_blocks)
        qh, d = query.shape
        caller = torch.cuda.current_stream(self.device)
        self.compute_stream.wait_stream(caller)
        with torch.cuda.stream(self.compute_stream):
            outs = torch.empty((n_chunks, qh, d), dtype=torch.float32, device=self.device)
            lses = torch.empty((n_chunks, qh), dtype=torch.float32, device=self.device)
            statuses = torch.empty((len(selected),), dtype=torch.int32, device=self.device)
            ids = torch.tensor(selected, dtype=torch.int32).to(self.device, non_blocking=True)
        query.record_stream(self.compute_stream)

        for ci in range(n_chunks):
            lo, hi = ci * self.stage_blocks, min(len(selected), (ci + 1) * self.stage_blocks)
            if self._device_ring is not None:
                slot = ci % 2
                if getattr(self.store.storage_backend, "device_reads_async", False):
                    # mapped: DMA copies on the transfer stream, after the slot's last decode
                    with torch.cuda.stream(self.transfer_stream):
                        if self._device_free[slot] is not None:
                            self.transfer_stream.wait_event(self._device_free[slot])
                        dev = self.store.read_records(layer, selected[lo:hi],
                                                      destination=self._device_ring[slot])
                        ready = torch.cuda.Event()
                        ready.record(self.transfer_stream)
                else:
                    # gds: cuFile writes device memory from the host thread, synchronously
                    if self._device_free[slot] is not None:
                        self._device_free[slot].synchronize()  # its previous chunk is decoded
                    dev = self.store.read_records(layer, selected[lo:hi],
                                                  destination=self._device_ring[slot],
                                                  threads=self.io_depth)
                    ready = None
            else:
                chunk = self._ring[ci % len(self._ring)]
                if chunk.copied is not None:
                    chunk.copied.synchronize()  # the pinned buffer's previous copy has landed
                raw = self.store.read_records(layer, selected[lo:hi], destination=chunk.raw,
                                              threads=self.io_depth)
                with torch.cuda.stream(self.transfer_stream):
                    dev = raw.to(self.device, non_blocking=True)
                    chunk.copied = torch.cuda.Event()
                    chunk.copied.record(self.transfer_stream)
                ready = chunk.copied
            with torch.cuda.stream(self.compute_stream):
                if ready is not None:
                    self.compute_stream.wait_event(ready)
                kp, vp, ks, vs, valid, status = ops.decode_records(dev, spec, layer, ids[lo:hi])
                if self._device_ring is not None:
                    self._device_free[ci % 2] = torch.cuda.Event()
                    self._device_free[ci % 2].record(self.compute_stream)
                self._attend(query, PackedBatch(kp, vp, ks, vs, valid, spec.bits,
                                                spec.group_size), scale, outs[ci], lses[ci])
                statuses[lo:hi].copy_(status)
                dev.record_stream(self.compute_stream)
        with torch.cuda.stream(self.compute_stream):
            if n_chunks == 1:
                out = outs[0]
            else:
                out, _ = ops.merge_chunks(outs, lses)
        done = torch.cuda.Event()
        done.record(self.compute_stream)
        caller.wait_event(done)
        out.record_stream(caller)
        self._raise_on_bad_records(statuses, selected, layer)
        if self._native:
            watch = ops.status_watch(self.device, self.compute_stream)
            with torch.cuda.stream(self.compute_stream):
                watch.arm("KVSSDPipeline.decode")
            watch.check("KVSSDPipeline.decode")  # the record statuses above already waited
        return out.to(query.dtype)

    @property
    def _native(self) -> bool:
        return type(self.attention_backend) is B200AttentionBackend

    def _attend(self, query: torch.Tensor, batch: PackedBatch, scale: float, out: torch.Tensor,
                lse: torch.Tensor) -> None:
        """One chunk's attention into (out, lse) through the resolved backend, as kvssd's
        streamed pipeline calls backend.run per chunk (src/kvssd/pipeline.py:138-145). The
        built-in ``cuda`` backend writes straight into the chunk's rows; another backend's
        result is copied there."""
        if self._native:
            ops.decode(query, batch.packed_k, batch.packed_v, batch.scales_k, batch.scales_v,
                       batch.valid_tokens, batch.bits, batch.group_size, scale, out=out, lse=lse)
            return
        o, l = self.attention_backend.run(query, batch, scale)
        out.copy_(o)
        lse.copy_(l)

    @staticmethod
    def _raise_on_bad_records(statuses: torch.Tensor, selected: list[int], layer: int) -> None:
        bad = statuses.cpu()  # waits for the chunks' record decodes
        if not torch.any(bad):
            return
        for i, st in enumerate(bad.tolist()):
            if st & (ops.RECORD_BAD_HEADER | ops.RECORD_BAD_ID):
                raise ValueError(f"invalid KVSSD record header (layer={layer}, "
                                 f"block={selected[i]})")
            if st & (ops.RECORD_BAD_GEOMETRY | ops.RECORD_BAD_LENGTH):
                raise ValueError("record layout does not match manifest")
            if st & ops.RECORD_BAD_CRC:
                raise IOError(f"CRC mismatch for layer={layer}, block={selected[i]}")

    def close(self) -> None:
        torch.cuda.synchronize(self.device)

    def __enter__(self) -> "KVSSDPipeline":
        return self

    def __exit__(self, *_: object) -> None:
        self.close()
