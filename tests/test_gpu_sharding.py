"""Multi-GPU decode (needs >= 2 GPUs; each case is skipped when fewer GPUs than its ranks are
visible): the c1 configuration split over 2, 4 and 8 ranks, one process per GPU, against the
reference backend's frozen output for the whole context -- token shards through the fused
peer-memory exchange kernel and through NCCL, and KV-head shards -- and the c2 configuration
(1024 blocks) split over 2, 4 and 8 ranks through the peer exchange against its frozen output.
Every call on every rank must give the same bits. Also: the peer exchange under CUDA-graph
replay, ranks whose shards are empty or unaligned (they take the exchange like the others),
and a rank that skips a call (the other rank's kernel gives up after about a second, flags
status bit 8 and returns NaN; the group's collective check raises on every rank and re-arms
the buffers; nothing faults or hangs; NVLS is off)."""

from __future__ import annotations

import datetime
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from conftest import load_npz

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank: int, world: int, port: int, config: str = "c1"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    from kvssd_b200 import PackedBatch
    from kvssd_b200.workloads import WORKLOADS, make_layer

    w = WORKLOADS[config]
    layer = make_layer(w, 0, "cpu")
    batch = PackedBatch(*(t.to(device) for t in (layer.packed_k, layer.packed_v, layer.scales_k,
                                                 layer.scales_v, layer.valid_tokens)),
                        w.bits, w.group_size)
    return device, w, batch, layer.query.to(device)


def _rank_main(rank: int, world: int, port: int, mode: str, transport: str, config: str,
               results) -> None:
    device, w, batch, q = _setup(rank, world, port, config)
    try:
        from kvssd_b200.sharding import ShardedDecoder, shard_batch_by_blocks, shard_batch_by_heads

        if mode == "tokens":
            local = shard_batch_by_blocks(batch, rank, world)
        else:
            local = shard_batch_by_heads(batch, rank, world, q.shape[0])
        dec = ShardedDecoder(mode, transport=transport)
        outs = []
        for _ in range(3):  # consecutive calls reuse the exchange buffers (both halves)
            out, lse = dec.run(q, local, 1.0 / math.sqrt(w.head_dim))
            outs.append((out.cpu().numpy().copy(), lse.cpu().numpy().copy()))
        torch.cuda.synchronize(device)
        results[rank] = (outs, dec._peer is not None)
        dec.close()
    finally:
        dist.destroy_process_group()


def _spawn(fn, *args, world: int = 2):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        mp.start_processes(fn, args=(world, _free_port(), *args, results), nprocs=world,
                           join=True, start_method="spawn")
        return dict(results)


def _needs(world: int):
    return pytest.mark.skipif(torch.cuda.device_count() < world,
                              reason=f"needs {world} GPUs")


def _check(out, lse, g):
    np.testing.assert_allclose(out.astype(np.float16).astype(np.float32),
                               g["out"].astype(np.float16).astype(np.float32), atol=2e-3, rtol=1e-2)
    np.testing.assert_allclose(lse, g["lse"], atol=5e-3, rtol=1e-3)


def _check_group(results, world: int, g, transport: str) -> None:
    for rank in range(world):
        outs, used_peer = results[rank]
        assert used_peer == (transport == "peer")
        for out, lse in outs:
            _check(out, lse, g)
        # every call, and every rank, give the same bits
        assert all(np.array_equal(o, outs[0][0]) for o, _ in outs)
        assert np.array_equal(outs[0][0], results[0][0][0][0])


@pytest.mark.parametrize("world", [pytest.param(n, marks=_needs(n)) for n in (2, 4, 8)])
@pytest.mark.parametrize("mode,transport", [("tokens", "peer"), ("tokens", "nccl"),
                                            ("heads", "auto")])
def test_sharded_decode_matches_reference(mode, transport, world):
    g = load_npz("config_c1.npz")
    _check_group(_spawn(_rank_main, mode, transport, "c1", world=world), world, g, transport)


@pytest.mark.parametrize("world", [pytest.param(n, marks=_needs(n)) for n in (2, 4, 8)])
def test_sharded_c2_peer_exchange_matches_reference(world):
    g = load_npz("config_c2.npz")
    _check_group(_spawn(_rank_main, "tokens", "peer", "c2", world=world), world, g, "peer")


def _graph_main(rank: int, world: int, port: int, results) -> None:
    device, w, batch, q = _setup(rank, world, port)
    try:
        from kvssd_b200.sharding import ShardedDecoder, shard_batch_by_blocks

        local = shard_batch_by_blocks(batch, rank, world)
        dec = ShardedDecoder("tokens", transport="peer")
        scale = 1.0 / math.sqrt(w.head_dim)
        eager = dec.run(q, local, scale)[0].clone()
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            dec.run(q, local, scale)
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        dist.barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            out, _ = dec.run(q, local, scale)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize(device)
        from kvssd_b200 import ops

        results[rank] = (torch.equal(out, eager), ops.read_device_status_all(device))
        del g
        dec.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_replays_in_cuda_graph():
    results = _spawn(_graph_main)
    for rank in (0, 1):
        same, status = results[rank]
        assert same and status == 0


def _uneven_main(rank: int, world: int, port: int, results) -> None:
    """One selected block over the ranks: every rank but 0 holds an empty shard, and rank 0's
    codes are a view 8 bytes off 16-byte alignment. Every rank still takes the peer exchange
    (the choice rests on the shared geometry), and the result is rank 0's block alone."""
    device, w, batch, q = _setup(rank, world, port)
    try:
        from dataclasses import replace

        from kvssd_b200 import ops
        from kvssd_b200.sharding import ShardedDecoder, shard_batch_by_blocks

        scale = 1.0 / math.sqrt(w.head_dim)
        one = replace(batch, packed_k=batch.packed_k[:1], packed_v=batch.packed_v[:1],
                      scales_k=batch.scales_k[:1], scales_v=batch.scales_v[:1],
                      valid_tokens=batch.valid_tokens[:1])
        local = shard_batch_by_blocks(one, rank, world)
        if rank == 0:
            raw = torch.empty(local.packed_k.numel() + 8, dtype=torch.uint8, device=device)
            view = raw[8:].view(local.packed_k.shape)
            view.copy_(local.packed_k)
            local = replace(local, packed_k=view)
        dec = ShardedDecoder("tokens")
        runs = [tuple(t.clone() for t in dec.run(q, local, scale)) for _ in range(2)]
        ref_out, ref_lse = ops.decode(q, *(t.contiguous() for t in (
            one.packed_k, one.packed_v, one.scales_k, one.scales_v)),
            one.valid_tokens.to(torch.int32).contiguous(), w.bits, w.group_size, scale)
        torch.cuda.synchronize(device)
        close = all(torch.allclose(o, ref_out, atol=1e-5, rtol=1e-5) and
                    torch.allclose(lse, ref_lse, atol=1e-5, rtol=1e-5) for o, lse in runs)
        results[rank] = (close, dec._peer is not None, ops.read_device_status_all(device))
        dec.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [pytest.param(n, marks=_needs(n)) for n in (2, 4)])
def test_peer_exchange_with_empty_and_unaligned_shards(world):
    results = _spawn(_uneven_main, world=world)
    for rank in range(world):
        close, used_peer, status = results[rank]
        assert used_peer and status == 0 and close


def _skip_main(rank: int, world: int, port: int, results) -> None:
    device, w, batch, q = _setup(rank, world, port)
    try:
        from kvssd_b200 import ops
        from kvssd_b200.sharding import ShardedDecoder, shard_batch_by_blocks

        local = shard_batch_by_blocks(batch, rank, world)
        dec = ShardedDecoder("tokens", transport="peer")
        scale = 1.0 / math.sqrt(w.head_dim)
        dec.run(q, local, scale)  # both ranks: creates the exchange, one good call
        dec.check()  # collective: nothing flagged
        nan_result = None
        if rank == 0:  # rank 1 skips this call: rank 0 must give up, not hang, and return NaN
            out, lse = dec.run(q, local, scale)
            torch.cuda.synchronize(device)
            nan_result = bool(torch.isnan(out).all()) and bool(torch.isnan(lse).all())
        raised = None
        try:
            dec.check()  # collective: rank 0 flagged bit 8, so both ranks raise; buffers re-armed
        except ops.DeviceFailure as exc:
            raised = exc.status
        out, lse = dec.run(q, local, scale)
        torch.cuda.synchronize(device)
        results[rank] = (raised, nan_result, ops.read_device_status_all(device),
                         out.cpu().numpy(), lse.cpu().numpy())
        dec.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_times_out_when_a_rank_skips_a_call():
    g = load_npz("config_c1.npz")
    results = _spawn(_skip_main)
    assert results[0][1] is True  # the timed-out call returned NaN, not a plausible number
    for rank in (0, 1):
        raised, _, status, out, lse = results[rank]
        assert raised is not None and raised & 8  # every rank learns of the failure
        assert status == 0
        _check(out, lse, g)  # the re-armed group decodes correctly again
