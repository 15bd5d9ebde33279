"""Multi-rank host logic of kvssd_b200.sharding on CPU: gloo process groups of 2 and 4 ranks.

Each rank decodes its shard with the oracle (the checker stands in for the CUDA kernel on a
host without a GPU) and the ShardedDecoder does the partition, the all-gather and the merge
order exactly as it does over NCCL; rank 0 compares the result with the reference backend's
golden output for the whole batch.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from conftest import f16, load_npz

from kvssd_b200 import PackedBatch
from kvssd_b200.sharding import (
    ShardedDecoder,
    block_range,
    head_shard,
    shard_batch_by_blocks,
    shard_batch_by_heads,
)
from oracle import kvssd_oracle as oracle

GOLDEN = "backend_gqa4_b4_32_8_128.npz"


def _batch(g) -> tuple[torch.Tensor, PackedBatch]:
    batch = PackedBatch(
        torch.from_numpy(g["packed_k"]), torch.from_numpy(g["packed_v"]),
        torch.from_numpy(f16(g["scales_k"]).copy()), torch.from_numpy(f16(g["scales_v"]).copy()),
        torch.from_numpy(g["valid"]), int(g["bits"]), int(g["group"]))
    return torch.from_numpy(g["query"]).float(), batch


def _oracle_decode(query, batch: PackedBatch, sm_scale: float):
    out, lse = oracle.decode(query.numpy(), batch.packed_k.numpy(), batch.packed_v.numpy(),
                             batch.scales_k.numpy(), batch.scales_v.numpy(),
                             batch.valid_tokens.numpy(), batch.bits, batch.group_size,
                             sm_scale, threads=1)
    return torch.from_numpy(out), torch.from_numpy(lse)


def _oracle_merge(outs, lses):
    out, lse = oracle.merge_chunks(outs.numpy(), lses.numpy())
    return torch.from_numpy(out), torch.from_numpy(lse)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, mode: str, results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = load_npz(GOLDEN)
        query, batch = _batch(g)
        if mode == "tokens":
            local = shard_batch_by_blocks(batch, rank, world)
        else:
            local = shard_batch_by_heads(batch, rank, world, query.shape[0])
        dec = ShardedDecoder(mode, decode_fn=_oracle_decode, merge_fn=_oracle_merge)
        for _ in range(2):  # the receive buffer is reused across calls
            out, lse = dec.run(query, local, float(g["sm_scale"]))
        results[rank] = (out.numpy().copy(), lse.numpy().copy(), local.packed_k.shape[0])
    finally:
        dist.destroy_process_group()


def _run(world: int, mode: str):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        mp.start_processes(_rank_main, args=(world, _free_port(), mode, results),
                           nprocs=world, join=True, start_method="spawn")
        return dict(results)


def test_block_range_is_balanced_and_covers_everything():
    for n in (0, 1, 3, 7, 1024, 8192):
        for world in (1, 2, 3, 4, 8):
            ranges = [block_range(n, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        block_range(4, 2, 2)


def test_head_shard_follows_gqa_mapping():
    # kvssd's GQA rule: query head h reads KV head h // (QH / KVH)
    qh, kvh = 32, 8
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            kv_lo, kv_hi, q_lo, q_hi = head_shard(kvh, qh, r, world)
            assert all(kv_lo <= h // (qh // kvh) < kv_hi for h in range(q_lo, q_hi))
            seen.extend(range(q_lo, q_hi))
        assert seen == list(range(qh))
    with pytest.raises(ValueError, match="divide"):
        head_shard(8, 32, 0, 3)


def test_head_shard_batch_is_head_contiguous_copy():
    _, batch = _batch(load_npz(GOLDEN))
    shard = shard_batch_by_heads(batch, 1, 2, 32)
    assert shard.packed_k.is_contiguous() and shard.packed_k.shape[2] == 4
    assert torch.equal(shard.packed_k, batch.packed_k[:, :, 4:8])
    assert torch.equal(shard.scales_v, batch.scales_v[:, :, 4:8])


@pytest.mark.parametrize("world,mode", [(2, "tokens"), (2, "heads"), (4, "tokens"), (4, "heads")])
def test_sharded_decode_matches_whole_batch(world, mode):
    g = load_npz(GOLDEN)
    results = _run(world, mode)
    assert sorted(results) == list(range(world))
    if mode == "tokens" and world == 4:
        assert results[3][2] == 0  # three blocks over four ranks: the last shard is empty
    for rank in range(world):
        out, lse, _ = results[rank]
        np.testing.assert_allclose(out, g["out"], atol=2e-5, rtol=1e-5)
        np.testing.assert_allclose(lse, g["lse"], atol=2e-5, rtol=1e-6)


def test_peer_transport_choice_ignores_the_local_shard(monkeypatch):
    """Every rank of a token-sharded group takes the same transport: the choice rests on the
    geometry the ranks share, never on this rank's block count, alignment or emptiness (a rank
    that took the all-gather while the others ran the exchange kernel would leave both waiting).
    The planner is stubbed and the query is a CUDA-typed stand-in; nothing runs on a device."""
    from types import SimpleNamespace

    from kvssd_b200 import ops
    from kvssd_b200.sharding import ShardedDecoder

    g = load_npz(GOLDEN)
    _, batch = _batch(g)
    calls = []

    def plan(*args):
        calls.append(args)
        return {"kernel": "tensor_core_tma"}

    monkeypatch.setattr(ops, "decode_plan", plan)
    monkeypatch.setattr(ShardedDecoder, "world", property(lambda self: 2))
    query = SimpleNamespace(device=torch.device("cuda", 0), shape=(32, 128))
    raw = torch.empty(batch.packed_k.numel() + 8, dtype=torch.uint8)
    misaligned = raw[8:].view(batch.packed_k.shape)
    n = batch.packed_k.shape[0]
    shards = [batch, shard_batch_by_blocks(batch, 2 * n - 1, 2 * n),  # the last rank's: empty
              PackedBatch(misaligned, *(getattr(batch, f) for f in
                                        ("packed_v", "scales_k", "scales_v", "valid_tokens",
                                         "bits", "group_size")))]
    assert shards[1].packed_k.shape[0] == 0
    for transport in ("auto", "peer"):
        dec = ShardedDecoder("tokens", transport=transport)
        assert [dec._use_peer(query, s) for s in shards] == [True] * 3
    assert len(set(calls)) == 1  # the same question on every rank, whatever its shard holds
    monkeypatch.setattr(ops, "decode_plan", lambda *a: {"kernel": "tensor_core_regs"})
    assert not ShardedDecoder("tokens")._use_peer(query, shards[1])
    with pytest.raises(RuntimeError, match="peer transport"):
        ShardedDecoder("tokens", transport="peer")._use_peer(query, shards[0])


def test_peer_operands_stand_in_for_empty_and_unaligned_shards():
    """What the exchange kernel is given: an empty shard becomes one block with no valid tokens
    (the kernel returns out 0 and lse -inf for it, no weight in the merge), kept for later calls;
    operands that are not 16-byte aligned or not contiguous are copied; the rest pass as they
    are."""
    from kvssd_b200.sharding import ShardedDecoder

    g = load_npz(GOLDEN)
    _, batch = _batch(g)
    dec = ShardedDecoder("tokens")
    n = batch.packed_k.shape[0]
    empty = shard_batch_by_blocks(batch, 2 * n - 1, 2 * n)  # the last rank's shard: no blocks
    stand_in = dec._peer_operands(empty)
    _, bt, kvh, pd = batch.packed_k.shape
    assert stand_in.packed_k.shape == (1, bt, kvh, pd) and stand_in.packed_v.shape == (1, bt, kvh, pd)
    assert stand_in.scales_k.shape == (1, bt, kvh, batch.scales_k.shape[3])
    assert stand_in.scales_k.dtype == batch.scales_k.dtype
    assert stand_in.valid_tokens.tolist() == [0] and stand_in.valid_tokens.dtype == torch.int32
    assert (stand_in.bits, stand_in.group_size) == (batch.bits, batch.group_size)
    assert dec._peer_operands(empty) is stand_in  # reused, not reallocated per call

    same = dec._peer_operands(batch)
    for f in ("packed_k", "packed_v", "scales_k", "scales_v"):
        assert getattr(same, f) is getattr(batch, f)
    raw = torch.empty(batch.packed_k.numel() + 8, dtype=torch.uint8)
    misaligned = raw[8:].view(batch.packed_k.shape)
    misaligned.copy_(batch.packed_k)
    strided = batch.scales_v.transpose(1, 2).contiguous().transpose(1, 2)
    fixed = dec._peer_operands(PackedBatch(misaligned, batch.packed_v, batch.scales_k, strided,
                                           batch.valid_tokens.long(), batch.bits,
                                           batch.group_size))
    assert fixed.packed_k.data_ptr() % 16 == 0 and torch.equal(fixed.packed_k, batch.packed_k)
    assert fixed.scales_v.is_contiguous() and torch.equal(fixed.scales_v, batch.scales_v)
    assert fixed.packed_v is batch.packed_v
    assert fixed.valid_tokens.dtype == torch.int32
