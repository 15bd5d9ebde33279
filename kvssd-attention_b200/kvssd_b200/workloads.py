"""Seeded synthetic decode workloads with the shapes of the benchmark configurations.

The reference publishes no dataset for this path; these generators stand in for it with the
configured shapes and distributions: K, V ~ N(0, 1) cast to FP16, query ~ N(0, 1) FP16,
symmetric groupwise INT2/INT4 codes with FP16 scales, and for the INT2 configuration 1% of the
(kv_head, dim) channels of K and V scaled by 8. Generation on the CPU is bit-reproducible
across machines (torch CPU generator); generation on a CUDA device is faster and
deterministic per device type.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .quant import quantize_tensor


@dataclass(frozen=True)
class Workload:
    name: str
    layers: int
    tokens: int
    kv_heads: int = 8
    head_dim: int = 128
    query_heads: int = 32
    block_tokens: int = 128
    bits: int = 4
    group_size: int = 32
    outlier_fraction: float = 0.0
    outlier_scale: float = 8.0
    sink: int | None = None  # RecentSinkBlocks(sink, recent) when set, else AllBlocks
    recent: int | None = None
    seed: int = 0

    @property
    def blocks_per_layer(self) -> int:
        return -(-self.tokens // self.block_tokens)

    @property
    def packed_dim(self) -> int:
        return self.head_dim * self.bits // 8

    @property
    def bytes_per_block(self) -> int:
        """Packed-KV bytes of one block: K+V codes plus K+V FP16 scales."""
        rows = self.block_tokens * self.kv_heads
        return 2 * rows * self.packed_dim + 2 * rows * (self.head_dim // self.group_size) * 2

    def selected_blocks(self) -> list[int]:
        ids = list(range(self.blocks_per_layer))
        if self.sink is None:
            return ids
        chosen = ids[: self.sink] + (ids[-self.recent :] if self.recent else [])
        return list(dict.fromkeys(chosen))


WORKLOADS: dict[str, Workload] = {
    # CPU-runnable reference configuration.
    "c1": Workload("c1", layers=1, tokens=8192, seed=1),
    # Single-GPU long context: the headline configuration.
    "c2": Workload("c2", layers=1, tokens=131072, seed=2),
    # INT2 with 1% outlier channels x8, RecentSinkBlocks(1, 32) over 1024 blocks.
    "c3": Workload("c3", layers=1, tokens=131072, bits=2, outlier_fraction=0.01, sink=1,
                   recent=32, seed=3),
    # Multi-layer decode step, sharded by KV-head groups across GPUs.
    "c4": Workload("c4", layers=32, tokens=65536, seed=4),
    # Ultra-long split-KV, token-block ranges across GPUs.
    "c5": Workload("c5", layers=1, tokens=1048576, seed=5),
}


@dataclass
class LayerData:
    """One layer's inputs: query and the PackedBatch-layout block pool (all on one device)."""

    query: torch.Tensor        # [QH, D] fp16
    packed_k: torch.Tensor     # [nb, bt, KVH, pd] uint8
    packed_v: torch.Tensor
    scales_k: torch.Tensor     # [nb, bt, KVH, G] fp16
    scales_v: torch.Tensor
    valid_tokens: torch.Tensor  # [nb] int32
    outlier_channels: torch.Tensor | None = None


def raw_layer(w: Workload, layer: int = 0, device: str | torch.device = "cpu"):
    """FP16 K, V [tokens, KVH, D], query [QH, D] and the outlier channel ids of one layer."""
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(w.seed * 1000003 + layer)
    shape = (w.tokens, w.kv_heads, w.head_dim)
    k = torch.randn(shape, generator=gen, device=device)
    v = torch.randn(shape, generator=gen, device=device)
    q = torch.randn((w.query_heads, w.head_dim), generator=gen, device=device)
    channels = None
    if w.outlier_fraction > 0:
        n = math.ceil(w.outlier_fraction * w.kv_heads * w.head_dim)
        channels = torch.randperm(w.kv_heads * w.head_dim, generator=gen, device=device)[:n]
        heads, dims = channels // w.head_dim, channels % w.head_dim
        k[:, heads, dims] *= w.outlier_scale
        v[:, heads, dims] *= w.outlier_scale
    return k.half(), v.half(), q.half(), channels


def blocks_from_raw(w: Workload, k: torch.Tensor, v: torch.Tensor):
    """Pads [tokens, KVH, D] to whole blocks and quantizes: the layout KVCacheStore.create
    writes per block, stacked."""
    nb = w.blocks_per_layer
    pad = nb * w.block_tokens - k.shape[0]
    if pad:
        k = torch.cat([k, k.new_zeros((pad, *k.shape[1:]))])
        v = torch.cat([v, v.new_zeros((pad, *v.shape[1:]))])
    kb = k.reshape(nb, w.block_tokens, w.kv_heads, w.head_dim)
    vb = v.reshape(nb, w.block_tokens, w.kv_heads, w.head_dim)
    kq = quantize_tensor(kb, w.bits, w.group_size)
    vq = quantize_tensor(vb, w.bits, w.group_size)
    valid = torch.full((nb,), w.block_tokens, dtype=torch.int32, device=k.device)
    if pad:
        valid[-1] = w.block_tokens - pad
    return kq.packed, vq.packed, kq.scales, vq.scales, valid


def make_layer(w: Workload, layer: int = 0, device: str | torch.device = "cpu",
               gen_device: str | torch.device | None = None) -> LayerData:
    """Generates one layer on ``gen_device`` (default: ``device``) and moves it to ``device``."""
    gen_device = torch.device(gen_device) if gen_device is not None else torch.device(device)
    k, v, q, channels = raw_layer(w, layer, gen_device)
    kp, vp, ks, vs, valid = blocks_from_raw(w, k, v)
    del k, v
    dev = torch.device(device)
    return LayerData(q.to(dev), kp.to(dev), vp.to(dev), ks.to(dev), vs.to(dev), valid.to(dev),
                     None if channels is None else channels.to(dev))
