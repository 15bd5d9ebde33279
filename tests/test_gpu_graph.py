"""One fused decode captured in a CUDA graph and replayed with new query contents: every
replay gets a fresh epoch from the workspace header on the device, so its combine folds its own
parts (a stale epoch would let it fold the previous replay's parts and return the previous
query's output). Each replay equals an eager decode of the same query."""

from __future__ import annotations

import math

import pytest
import torch

from kvssd_b200 import ops
from kvssd_b200.workloads import WORKLOADS, make_layer

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("name", ["c1", "c3"])
def test_graph_replays_fold_their_own_parts(name):
    w = WORKLOADS[name]
    lay = make_layer(w, 0, DEV)
    pool = [lay.packed_k, lay.packed_v, lay.scales_k, lay.scales_v, lay.valid_tokens]
    scale = 1.0 / math.sqrt(w.head_dim)
    q = lay.query.clone()
    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):
        ops.decode(q, *pool, w.bits, w.group_size, scale)  # workspace of the capture stream
    torch.cuda.current_stream(DEV).wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        out, lse = ops.decode(q, *pool, w.bits, w.group_size, scale)
    gen = torch.Generator(device="cpu").manual_seed(7)
    previous = None
    for _ in range(3):
        q.copy_(torch.randn(q.shape, generator=gen).to(DEV, q.dtype))
        g.replay()
        torch.cuda.synchronize()
        ref_out, ref_lse = ops.decode(q, *pool, w.bits, w.group_size, scale)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
        if previous is not None:
            assert not torch.equal(out, previous)
        previous = out.clone()
    assert ops.read_device_status(DEV, stream=side) == 0
