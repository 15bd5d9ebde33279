"""Symmetric groupwise INT2/INT4 quantization in kvssd's bit layout.

The layout is a data format shared with kvssd and must stay identical
(src/kvssd/quant.py:28-73): codes are unsigned in [0, 2^bits), packed low-bits-first along
the last dimension; scales are max|x| / (2^(bits-1) - 1) per group in FP32, stored as FP16;
codes are round-half-even(x / scale_fp32) clamped to [-2^(bits-1), 2^(bits-1)-1] plus the
midpoint. These helpers run wherever their tensors live (store creation, test inputs); the
decode hot path never calls them -- it unpacks in registers on the GPU.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class QuantizedTensor:
    packed: torch.Tensor
    scales: torch.Tensor
    original_shape: tuple[int, ...]
    bits: int
    group_size: int


def _check_bits(bits: int) -> None:
    if bits not in (2, 4):
        raise ValueError(f"bits must be 2 or 4, got {bits}")


def _check_quantizable(x: torch.Tensor, bits: int, group_size: int) -> None:
    # Same refusals, in the same order, as src/kvssd/quant.py:17-25.
    _check_bits(bits)
    if x.ndim < 1 or x.shape[-1] % group_size:
        raise ValueError("last dimension must be divisible by group_size")
    if group_size <= 0 or group_size % (8 // bits):
        raise ValueError("group_size must be positive and pack-aligned")
    if not x.is_floating_point():
        raise TypeError("quantization input must be floating point")


def pack_codes(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """Packs unsigned codes along the last dimension, low bits first."""
    if bits not in (2, 4):
        raise ValueError("bits must be 2 or 4")
    per_byte = 8 // bits
    if codes.shape[-1] % per_byte:
        raise ValueError("code dimension is not byte aligned")
    lanes = codes.to(torch.uint8).reshape(*codes.shape[:-1], -1, per_byte)
    out = torch.zeros(lanes.shape[:-1], dtype=torch.uint8, device=codes.device)
    for slot in range(per_byte):
        out |= (lanes[..., slot] & ((1 << bits) - 1)) << (slot * bits)
    return out.contiguous()


def unpack_codes(packed: torch.Tensor, bits: int, elements: int) -> torch.Tensor:
    """Inverse of pack_codes: [..., elements*bits/8] uint8 -> [..., elements] uint8 codes."""
    if bits not in (2, 4):
        raise ValueError("bits must be 2 or 4")
    per_byte = 8 // bits
    mask = (1 << bits) - 1
    lanes = [(packed >> (slot * bits)) & mask for slot in range(per_byte)]
    codes = torch.stack(lanes, dim=-1).reshape(*packed.shape[:-1], -1)
    return codes[..., :elements]


def quantize_tensor(x: torch.Tensor, bits: int, group_size: int = 32) -> QuantizedTensor:
    """Symmetric groupwise quantization (one FP16 scale per group along the last dim)."""
    _check_quantizable(x, bits, group_size)
    shape = tuple(x.shape)
    groups = x.float().reshape(*shape[:-1], shape[-1] // group_size, group_size)
    mid = 1 << (bits - 1)
    top = mid - 1
    scale = groups.abs().amax(dim=-1).clamp_min(1e-8) / top
    centred = torch.round(groups / scale.unsqueeze(-1)).clamp(-mid, top)
    codes = (centred + mid).to(torch.uint8).reshape(shape)
    return QuantizedTensor(
        packed=pack_codes(codes, bits),
        scales=scale.to(torch.float16).contiguous(),
        original_shape=shape,
        bits=bits,
        group_size=group_size,
    )


def dequantize_tensor(q: QuantizedTensor, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """(code - midpoint) * scale in FP32, then cast to ``dtype`` (one rounding for FP16)."""
    mid = 1 << (q.bits - 1)
    codes = unpack_codes(q.packed, q.bits, q.original_shape[-1]).to(torch.float32)
    grouped = codes.reshape(*q.original_shape[:-1], -1, q.group_size)
    values = (grouped - mid) * q.scales.float().unsqueeze(-1)
    return values.reshape(q.original_shape).to(dtype)
