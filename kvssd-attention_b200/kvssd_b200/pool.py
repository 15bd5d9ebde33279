"""Device-resident block pool: a layer's packed KV kept in HBM and decoded by block table.

This is the B200 replacement for the reference's per-chunk staging
(src/kvssd/pipeline.py:67-165, which stacks 4 blocks, copies them and launches one kernel plus
one merge per chunk): blocks are uploaded once into pool tensors laid out exactly as a
PackedBatch ([n_blocks, block_tokens, kv_heads, packed_dim] codes, [..., groups] FP16 scales,
[n_blocks] valid counts), and a decode is one kernel launch (plus its combine) over an int32
block table built from the selector's choice.
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import torch

from . import ops
from .format import CacheSpec, PackedKVBlock
from .selectors import AllBlocks, BlockSelector


class DeviceBlockPool:
    """Packed KV of one layer resident on a CUDA device."""

    def __init__(
        self,
        spec: CacheSpec,
        packed_k: torch.Tensor,
        packed_v: torch.Tensor,
        scales_k: torch.Tensor,
        scales_v: torch.Tensor,
        valid_tokens: torch.Tensor,
        block_ids: Sequence[int] | None = None,
    ):
        spec.validate()
        n = packed_k.shape[0]
        expected_p = (n, spec.block_tokens, spec.kv_heads, spec.packed_dim)
        expected_s = (n, spec.block_tokens, spec.kv_heads, spec.groups)
        if tuple(packed_k.shape) != expected_p or tuple(packed_v.shape) != expected_p:
            raise ValueError(f"packed KV must be {expected_p}")
        if tuple(scales_k.shape) != expected_s or tuple(scales_v.shape) != expected_s:
            raise ValueError(f"scales must be {expected_s}")
        if tuple(valid_tokens.shape) != (n,):
            raise ValueError("valid_tokens must contain one count per block")
        self.spec = spec
        self.packed_k = packed_k.contiguous()
        self.packed_v = packed_v.contiguous()
        self.scales_k = scales_k.contiguous()
        self.scales_v = scales_v.contiguous()
        self.valid_tokens = valid_tokens.to(torch.int32).contiguous()
        self.device = self.packed_k.device
        ids = list(range(n)) if block_ids is None else list(block_ids)
        if len(ids) != n:
            raise ValueError("block_ids must name every pool slot")
        self.block_ids = ids
        self._slot_of = {b: i for i, b in enumerate(ids)}

    @classmethod
    def from_blocks(cls, spec: CacheSpec, blocks: Sequence[PackedKVBlock],
                    device: torch.device | str) -> "DeviceBlockPool":
        if not blocks:
            raise ValueError("at least one block is required")
        device = torch.device(device)
        stack = lambda xs: torch.stack(list(xs)).to(device)  # noqa: E731
        return cls(
            spec,
            stack(b.key.packed for b in blocks),
            stack(b.value.packed for b in blocks),
            stack(b.key.scales for b in blocks),
            stack(b.value.scales for b in blocks),
            torch.tensor([b.valid_tokens for b in blocks], dtype=torch.int32, device=device),
            [b.block for b in blocks],
        )

    @classmethod
    def from_store(cls, store, layer: int, device: torch.device | str,
                   verify_crc: bool = True) -> "DeviceBlockPool":
        """Loads every block of ``layer``: the raw records are read into one pinned buffer by
        the native reader (KVCacheStore.read_records), copied to the device in one transfer and
        decoded there (header checks and the payload
        CRC-32 on the GPU, ops.decode_records). Raises like kvssd's decode_record on a bad
        record: ValueError for a bad header or layout, IOError for a CRC mismatch."""
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError(f"DeviceBlockPool needs a CUDA device, got {device}")
        spec = store.spec
        ids = store.blocks_for_layer(layer)
        if not ids:
            raise ValueError(f"layer {layer} has no blocks")
        raw = store.read_records(layer, ids)  # one batch of the native reader, pinned
        dev = raw.to(device, non_blocking=True)
        kp, vp, ks, vs, valid, status = ops.decode_records(
            dev, spec, layer, torch.tensor(ids, dtype=torch.int32))
        bad = status.cpu()
        if verify_crc is False:
            bad &= ~ops.RECORD_BAD_CRC
        for i, st in enumerate(bad.tolist()):
            if st & (ops.RECORD_BAD_HEADER | ops.RECORD_BAD_ID):
                raise ValueError(f"invalid KVSSD record header (layer={layer}, block={ids[i]})")
            if st & (ops.RECORD_BAD_GEOMETRY | ops.RECORD_BAD_LENGTH):
                raise ValueError("record layout does not match manifest")
            if st & ops.RECORD_BAD_CRC:
                raise IOError(f"CRC mismatch for layer={layer}, block={ids[i]}")
        return cls(spec, kp, vp, ks, vs, valid, ids)

    @property
    def n_blocks(self) -> int:
        return self.packed_k.shape[0]

    def block_table(self, block_ids: Sequence[int]) -> torch.Tensor:
        """int32 pool-slot table for the given block ids (KeyError for unknown ids)."""
        try:
            slots = [self._slot_of[b] for b in block_ids]
        except KeyError as exc:
            raise KeyError(f"block {exc.args[0]} is not resident in this pool") from exc
        return torch.tensor(slots, dtype=torch.int32).to(self.device, non_blocking=True)

    def packed_bytes(self, block_ids: Sequence[int] | None = None) -> int:
        n = self.n_blocks if block_ids is None else len(block_ids)
        return n * self.spec.packed_kv_bytes_per_block

    def decode_table(self, query: torch.Tensor, table: torch.Tensor | None,
                     sm_scale: float | None = None, out: torch.Tensor | None = None,
                     lse: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """(out fp32, lse fp32) over the pool slots in ``table`` (None = every slot).

        Asynchronous; a kernel failure (a table entry outside the pool is skipped and flagged;
        after a wait that gave up the call's result is NaN) raises ops.DeviceFailure on a later
        decode on this stream once the status read has landed (at the latest four calls on),
        or on ``check()``, which waits for it."""
        scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(query.shape[-1])
        watch = ops.status_watch(self.device)
        watch.poll("DeviceBlockPool.decode (an earlier call)")
        result = ops.decode(query, self.packed_k, self.packed_v, self.scales_k, self.scales_v,
                            self.valid_tokens, self.spec.bits, self.spec.group_size, scale,
                            block_table=table, out=out, lse=lse)
        watch.arm("DeviceBlockPool.decode")
        return result

    def check(self) -> None:
        """Waits for the outstanding status reads of this device's current stream and raises
        ops.DeviceFailure if a decode flagged a failure."""
        ops.status_watch(self.device).check("DeviceBlockPool.decode")

    def decode(self, query: torch.Tensor, selector: BlockSelector | None = None,
               sm_scale: float | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        selector = selector or AllBlocks()
        chosen = selector.select(list(self.block_ids))
        if not chosen:
            raise ValueError("selector returned no blocks")
        if chosen == self.block_ids:
            return self.decode_table(query.to(self.device), None, sm_scale)
        return self.decode_table(query.to(self.device), self.block_table(chosen), sm_scale)
