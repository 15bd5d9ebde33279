"""KVSSDPipeline: selection -> record reads -> staging -> fused decode -> exact merge.

API of src/kvssd/pipeline.py:19-196 (constructor arguments, ``decode(query, layer,
selector)``, context manager). Execution is CUDA-only: records are read by the bounded
loader, copied chunk by chunk (``stage_blocks`` blocks) into reusable pinned buffers, sent to
the device on a transfer stream, and each chunk is decoded on a compute stream as soon as
its copy lands; the per-chunk (out, lse) pairs are merged exactly by one N-way merge kernel
at the end (the reference chains one pairwise merge per chunk). For a layer that stays
resident in HBM use DeviceBlockPool, which decodes with a single launch.
"""

from __future__ import annotations

import math

import torch

from . import ops
from .backends import AttentionBackend, resolve_attention_backend
from .loader import AsyncBlockLoader
from .selectors import AllBlocks, BlockSelector


class _PinnedChunk:
    """Stacked pinned host tensors for one chunk of blocks plus its copy-done event."""

    def __init__(self, spec, blocks: int):
        pin = torch.cuda.is_available()
        p = (blocks, spec.block_tokens, spec.kv_heads, spec.packed_dim)
        s = (blocks, spec.block_tokens, spec.kv_heads, spec.groups)
        self.kp = torch.empty(p, dtype=torch.uint8, pin_memory=pin)
        self.vp = torch.empty(p, dtype=torch.uint8, pin_memory=pin)
        self.ks = torch.empty(s, dtype=torch.float16, pin_memory=pin)
        self.vs = torch.empty(s, dtype=torch.float16, pin_memory=pin)
        self.valid = torch.empty(blocks, dtype=torch.int32, pin_memory=pin)
        self.copied: torch.cuda.Event | None = None


class KVSSDPipeline:
    """End-to-end selection, prefetch, pinned staging and fused packed attention."""

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
        if stage_blocks < 1:
            raise ValueError("stage_blocks must be positive")
        if require_cuda_kernel and attention_backend not in (None, "auto", "cuda"):
            raise ValueError("require_cuda_kernel conflicts with a non-CUDA attention backend")
        requested = "cuda" if require_cuda_kernel else attention_backend
        self.attention_backend = resolve_attention_backend(requested, self.device)
        self.loader = AsyncBlockLoader(store, depth=io_depth, pinned=True)
        self.stage_blocks = stage_blocks
        self.require_cuda_kernel = require_cuda_kernel
        self.transfer_stream = torch.cuda.Stream(device=self.device)
        self.compute_stream = torch.cuda.Stream(device=self.device)
        self._ring = [_PinnedChunk(store.spec, stage_blocks) for _ in range(2)]

    def _stage(self, chunk: _PinnedChunk, count: int) -> tuple[torch.Tensor, ...]:
        """Enqueues the H2D copy of the first ``count`` blocks of a pinned chunk."""
        with torch.cuda.stream(self.transfer_stream):
            dev = tuple(t[:count].to(self.device, non_blocking=True)
                        for t in (chunk.kp, chunk.vp, chunk.ks, chunk.vs, chunk.valid))
            chunk.copied = torch.cuda.Event()
            chunk.copied.record(self.transfer_stream)
        return dev

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
        query.record_stream(self.compute_stream)

        def launch(dev: tuple[torch.Tensor, ...], ready: torch.cuda.Event, index: int) -> None:
            with torch.cuda.stream(self.compute_stream):
                self.compute_stream.wait_event(ready)
                ops.decode(query, dev[0], dev[1], dev[2], dev[3], dev[4], spec.bits,
                           spec.group_size, scale, out=outs[index], lse=lses[index])
                for t in dev:
                    t.record_stream(self.compute_stream)

        filled = 0
        index = 0
        chunk = self._ring[0]
        for block in self.loader.iter_records(layer, selected):
            if filled == 0 and chunk.copied is not None:
                chunk.copied.synchronize()  # the pinned buffer's previous copy has landed
            chunk.kp[filled].copy_(block.key.packed)
            chunk.vp[filled].copy_(block.value.packed)
            chunk.ks[filled].copy_(block.key.scales)
            chunk.vs[filled].copy_(block.value.scales)
            chunk.valid[filled] = block.valid_tokens
            filled += 1
            if filled == self.stage_blocks:
                launch(self._stage(chunk, filled), chunk.copied, index)
                index += 1
                filled = 0
                chunk = self._ring[index % len(self._ring)]
        if filled:
            launch(self._stage(chunk, filled), chunk.copied, index)
            index += 1
        with torch.cuda.stream(self.compute_stream):
            if n_chunks == 1:
                out = outs[0]
            else:
                out, _ = ops.merge_chunks(outs, lses)
        done = torch.cuda.Event()
        done.record(self.compute_stream)
        caller.wait_event(done)
        out.record_stream(caller)
        return out.to(query.dtype)

    def close(self) -> None:
        self.loader.close()

    def __enter__(self) -> "KVSSDPipeline":
        return self

    def __exit__(self, *_: object) -> None:
        self.close()
