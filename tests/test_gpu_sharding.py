"""Multi-GPU decode over NCCL (needs >= 2 GPUs; skipped otherwise): token-block-range and
KV-head shards of the c1 configuration decoded on 2 ranks by ShardedDecoder with the CUDA
kernels, against the reference backend's frozen output for the whole context."""

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


def _rank_main(rank: int, world: int, port: int, mode: str, results) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from kvssd_b200 import PackedBatch
        from kvssd_b200.sharding import ShardedDecoder, shard_batch_by_blocks, shard_batch_by_heads
        from kvssd_b200.workloads import WORKLOADS, make_layer

        w = WORKLOADS["c1"]
        layer = make_layer(w, 0, "cpu")
        batch = PackedBatch(*(t.to(device) for t in (layer.packed_k, layer.packed_v,
                                                     layer.scales_k, layer.scales_v,
                                                     layer.valid_tokens)), w.bits, w.group_size)
        q = layer.query.to(device)
        if mode == "tokens":
            local = shard_batch_by_blocks(batch, rank, world)
        else:
            local = shard_batch_by_heads(batch, rank, world, q.shape[0])
        dec = ShardedDecoder(mode)
        for _ in range(2):
            out, lse = dec.run(q, local, 1.0 / math.sqrt(w.head_dim))
        torch.cuda.synchronize(device)
        results[rank] = (out.cpu().numpy(), lse.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["tokens", "heads"])
def test_two_gpu_sharded_decode_matches_reference(mode):
    g = load_npz("config_c1.npz")
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        mp.start_processes(_rank_main, args=(2, _free_port(), mode, results), nprocs=2,
                           join=True, start_method="spawn")
        results = dict(results)
    for rank in (0, 1):
        out, lse = results[rank]
        np.testing.assert_allclose(out.astype(np.float16).astype(np.float32),
                                   g["out"].astype(np.float16).astype(np.float32),
                                   atol=2e-3, rtol=1e-2)
        np.testing.assert_allclose(lse, g["lse"], atol=5e-3, rtol=1e-3)
