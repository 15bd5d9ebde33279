"""Attention entry points (API of src/kvssd/attention.py:50-134) on the B200 kernels.

The dense ``reference_attention`` / ``packed_attention_reference`` helpers of the reference
are CPU oracles and live in the test oracle, not here: every function in this module runs the
native CUDA kernels or raises.
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import torch

from . import ops
from .backends import AttentionBackend, PackedBatch, resolve_attention_backend
from .format import PackedKVBlock


def stack_blocks(blocks: Sequence[PackedKVBlock], device: torch.device) -> tuple[torch.Tensor, ...]:
    """Stacks blocks into PackedBatch tensors on ``device`` (src/kvssd/attention.py:50-60)."""
    if not blocks:
        raise ValueError("at least one block is required")
    device = torch.device(device)
    kwargs = {"device": device, "non_blocking": device.type == "cuda"}
    return (
        torch.stack([b.key.packed for b in blocks]).to(**kwargs),
        torch.stack([b.value.packed for b in blocks]).to(**kwargs),
        torch.stack([b.key.scales for b in blocks]).to(**kwargs),
        torch.stack([b.value.scales for b in blocks]).to(**kwargs),
        torch.tensor([b.valid_tokens for b in blocks], dtype=torch.int32, device=device),
    )


def cuda_extension_available() -> bool:
    try:
        resolve_attention_backend("cuda", torch.device("cuda"))
        return True
    except RuntimeError:
        return False


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
    backend = resolve_attention_backend("cuda", query.device)
    return backend.run(
        query,
        PackedBatch(packed_k, packed_v, scales_k, scales_v, valid_tokens, bits, group_size),
        sm_scale,
    )


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
    """Runs packed attention over ``blocks``; returns the output in the query's dtype."""
    if not blocks:
        raise ValueError("at least one block is required")
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(query.shape[-1])
    if require_cuda_kernel and attention_backend not in (None, "auto", "cuda"):
        raise ValueError("require_cuda_kernel conflicts with a non-CUDA attention backend")
    requested = "cuda" if require_cuda_kernel else attention_backend
    backend = resolve_attention_backend(requested, query.device)
    kp, vp, ks, vs, valid = stack_blocks(blocks, query.device)
    output, _ = backend.run(
        query,
        PackedBatch(kp, vp, ks, vs, valid, blocks[0].key.bits, blocks[0].key.group_size),
        scale,
    )
    return output.to(query.dtype)
