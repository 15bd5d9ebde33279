"""Attention entry points with kvssd's API (src/kvssd/attention.py:50-134) on the B200 kernels.

Every function here runs libkvssd_b200's CUDA kernels or raises: the dense
``reference_attention`` / ``packed_attention_reference`` helpers of kvssd are CPU oracles and
live in the test oracle, not in this package. Merges of normalised chunks run as kernels
(kvssd evaluates the same formula with torch ops).
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import torch

from . import ops
from .backends import AttentionBackend, PackedBatch, resolve_attention_backend
from .backends.cuda import B200AttentionBackend
from .format import PackedKVBlock


def stack_blocks(blocks: Sequence[PackedKVBlock], device: torch.device) -> tuple[torch.Tensor, ...]:
    """PackedBatch tensors (packed_k, packed_v, scales_k, scales_v, valid_tokens) of
    ``blocks`` on ``device`` (src/kvssd/attention.py:50-60).

    Host blocks bound for a CUDA device are gathered into one pinned staging tensor per field
    and moved with one asynchronous copy each; blocks already on ``device`` are stacked there.
    """
    if not blocks:
        raise ValueError("at least one block is required")
    device = torch.device(device)
    fields = [lambda b: b.key.packed, lambda b: b.value.packed, lambda b: b.key.scales,
              lambda b: b.value.scales]
    valid = torch.tensor([b.valid_tokens for b in blocks], dtype=torch.int32)
    first = blocks[0]
    if first.key.packed.device == device:
        staged = [torch.stack([field(b) for b in blocks]) for field in fields]
        return (*staged, valid.to(device))
    pinned = device.type == "cuda" and torch.cuda.is_available()
    staged = []
    for field in fields:
        proto = field(first)
        host = torch.empty((len(blocks), *proto.shape), dtype=proto.dtype, pin_memory=pinned)
        for i, block in enumerate(blocks):
            host[i].copy_(field(block))
        staged.append(host.to(device, non_blocking=pinned))
    return (*staged, valid.to(device))


def cuda_extension_available() -> bool:
    """True when the ``cuda`` backend (libkvssd_b200 on a B200) can run on the current device."""
    if not torch.cuda.is_available():
        return False
    return B200AttentionBackend().probe(torch.device("cuda")).available


def select_backend(device: torch.device, require_cuda_kernel: bool,
                   attention_backend: str | AttentionBackend | None) -> AttentionBackend:
    """kvssd's backend choice for packed_attention and KVSSDPipeline (attention.py:116-118,
    pipeline.py:45-48): ``require_cuda_kernel`` forces ``cuda`` and conflicts with any other
    explicit choice."""
    if require_cuda_kernel:
        if attention_backend not in (None, "auto", "cuda"):
            raise ValueError("require_cuda_kernel conflicts with a non-CUDA attention backend")
        attention_backend = "cuda"
    return resolve_attention_backend(attention_backend, device)


def fused_attention_tensors(
    query: torch.Tensor,
    packed_k: torch.Tensor,
    packed_v: torch.Tensor,
    scales_k: torch.Tensor,
    scales_v: torch.Tensor,
    valid_tokens: torch.Tensor,
    bits: int,
    group_size: int,
    sm_scale: float,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Low-level CUDA entry point returning normalised output and log-sum-exp."""
    batch = PackedBatch(packed_k, packed_v, scales_k, scales_v, valid_tokens, bits, group_size)
    return select_backend(query.device, True, None).run(query, batch, sm_scale)


def merge_attention_chunks(
    left_output: torch.Tensor,
    left_lse: torch.Tensor,
    right_output: torch.Tensor,
    right_lse: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact merge of two normalised chunks: L = logaddexp(La, Lb),
    O = Oa*exp(La-L) + Ob*exp(Lb-L), evaluated by a CUDA kernel."""
    return ops.merge_pair(left_output, left_lse, right_output, right_lse)


def merge_attention_chunks_n(outputs: torch.Tensor, lses: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact merge of N normalised chunks ([N, QH, D], [N, QH]) in one kernel."""
    return ops.merge_chunks(outputs, lses)


def packed_attention(
    query: torch.Tensor,
    blocks: Sequence[PackedKVBlock],
    sm_scale: float | None = None,
    require_cuda_kernel: bool = False,
    attention_backend: str | AttentionBackend | None = None,
) -> torch.Tensor:
    """Attention of ``query`` over ``blocks`` in one backend call; output in the query's dtype."""
    if not blocks:
        raise ValueError("at least one block is required")
    backend = select_backend(query.device, require_cuda_kernel, attention_backend)
    batch = PackedBatch(*stack_blocks(blocks, query.device), blocks[0].key.bits,
                        blocks[0].key.group_size)
    scale = 1.0 / math.sqrt(query.shape[-1]) if sm_scale is None else sm_scale
    output, _ = backend.run(query, batch, scale)
    return output.to(query.dtype)
