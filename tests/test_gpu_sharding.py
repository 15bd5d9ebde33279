"""Multi-GPU decode (needs >= 2 GPUs; skipped otherwise): the c1 configuration split over 2
ranks, one process per GPU, against the reference backend's frozen output for the whole
context -- token shards through the fused peer-memory exchange kernel and through NCCL, and
KV-head shards. Also: the peer exchange under CUDA-graph replay, and a rank that skips a call
(the other rank's kernel gives up after about a second and flags status bit 8; nothing faults
or hangs; NVLS is off)."""

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


def _setup(rank: int, world: int, port: int):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    from kvssd_b200 import PackedBatch
    from kvssd_b200.workloads import WORKLOADS, make_layer

    w = WORKLOADS["c1"]
    layer = make_layer(w, 0, "cpu")
    batch = PackedBatch(*(t.to(device) for t in (layer.packed_k, layer.packed_v, layer.scales_k,
                                                 layer.scales_v, layer.valid_tokens)),
                        w.bits, w.group_size)
    return device, w, batch, layer.query.to(device)


def _rank_main(rank: int, world: int, port: int, mode: str, transport: str, results) -> None:
    device, w, batch, q = _setup(rank, world, port)
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


def _spawn(fn, *args):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        mp.start_processes(fn, args=(2, _free_port(), *args, results), nprocs=2, join=True,
                           start_method="spawn")
        return dict(results)


def _check(out, lse, g):
    np.testing.assert_allclose(out.astype(np.float16).astype(np.float32),
                               g["out"].astype(np.float16).astype(np.float32), atol=2e-3, rtol=1e-2)
    np.testing.assert_allclose(lse, g["lse"], atol=5e-3, rtol=1e-3)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode,transport", [("tokens", "peer"), ("tokens", "nccl"),
                                            ("heads", "auto")])
def test_two_gpu_sharded_decode_matches_reference(mode, transport):
    g = load_npz("config_c1.npz")
    results = _spawn(_rank_main, mode, transport)
    for rank in (0, 1):
        outs, used_peer = results[rank]
        assert used_peer == (transport == "peer")
        for out, lse in outs:
            _check(out, lse, g)
        # every call, and both ranks, give the same bits
        assert all(np.array_equal(o, outs[0][0]) for o, _ in outs)
        assert np.array_equal(outs[0][0], results[0][0][0][0])


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

        results[rank] = (torch.equal(out, eager), ops.read_device_status(device))
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


def _skip_main(rank: int, world: int, port: int, results) -> None:
    device, w, batch, q = _setup(rank, world, port)
    try:
        from kvssd_b200 import ops
        from kvssd_b200.sharding import ShardedDecoder, shard_batch_by_blocks

        local = shard_batch_by_blocks(batch, rank, world)
        dec = ShardedDecoder("tokens", transport="peer")
        scale = 1.0 / math.sqrt(w.head_dim)
        dec.run(q, local, scale)  # both ranks: creates the exchange, one good call
        torch.cuda.synchronize(device)
        ops.read_device_status(device)
        dist.barrier()
        if rank == 0:  # rank 1 skips this call: rank 0 must give up, not hang
            dec.run(q, local, scale)
            torch.cuda.synchronize(device)
        status = ops.read_device_status(device)
        dist.barrier()
        dec._peer.reset()  # call numbers differ now: re-zero the buffers collectively
        out, lse = dec.run(q, local, scale)
        torch.cuda.synchronize(device)
        results[rank] = (status, ops.read_device_status(device), out.cpu().numpy(),
                         lse.cpu().numpy())
        dec.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_times_out_when_a_rank_skips_a_call():
    g = load_npz("config_c1.npz")
    results = _spawn(_skip_main)
    assert results[0][0] & 8 and results[1][0] == 0
    for rank in (0, 1):
        assert results[rank][1] == 0
        _check(results[rank][2], results[rank][3], g)
