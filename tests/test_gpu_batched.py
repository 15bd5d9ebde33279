"""Batched decode (kvssd_b200_decode_batched): several independent decodes in one launch --
separate pools (layers) or one pool with per-problem block tables (a batch of sequences) --
against the CPU oracle at the parity tolerance and against single decodes (these split the
tokens differently, so the FP16 probabilities are rounded against different running maxima:
agreement within 5e-4); a refused descriptor is flagged without touching the other problems."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from kvssd_b200 import _native, ops
from kvssd_b200.quant import quantize_tensor
from oracle import kvssd_oracle as orc

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
SCALE = 1.0 / math.sqrt(128)
NEAR = dict(atol=5e-4, rtol=5e-3)  # batched vs single decode of the same problem


def _check_oracle(q, pool, table, out, lse):
    kp, vp, ks, vs, valid = [x.cpu().numpy() for x in pool]
    ro, rl = orc.decode(q.float().cpu().numpy(), kp, vp, ks, vs, valid, 4, 32, SCALE,
                        block_table=None if table is None else table.cpu().numpy())
    np.testing.assert_allclose(out.cpu().numpy().astype(np.float16).astype(np.float32),
                               ro.astype(np.float16).astype(np.float32), atol=2e-3, rtol=1e-2)
    np.testing.assert_allclose(lse.cpu().numpy(), rl, atol=5e-3, rtol=1e-3)


def _pool(nb, seed, valid=None, kvh=8, group=32):
    gen = torch.Generator().manual_seed(seed)
    k = torch.randn(nb, 128, kvh, 128, generator=gen).half()
    v = torch.randn(nb, 128, kvh, 128, generator=gen).half()
    kq, vq = quantize_tensor(k, 4, group), quantize_tensor(v, 4, group)
    valid = torch.tensor(valid if valid is not None else [128] * nb, dtype=torch.int32)
    return [t.to(DEV) for t in (kq.packed, vq.packed, kq.scales, vq.scales, valid)]


def _query(seed, qh=32):
    return torch.randn(qh, 128, generator=torch.Generator().manual_seed(seed)).half().to(DEV)


def test_batched_layers_match_single_decodes_and_oracle():
    pools = [_pool(nb, 10 + i, valid=[128] * (nb - 1) + [37]) for i, nb in enumerate((3, 9, 1, 20))]
    queries = [_query(100 + i) for i in range(len(pools))]
    tables = [None, torch.tensor([8, 0, 3, 3, 5], dtype=torch.int32, device=DEV), None, None]
    problems = [(q, *p, t) for q, p, t in zip(queries, pools, tables)]
    outs = ops.decode_batched(problems, 4, 32, SCALE)
    torch.cuda.synchronize()
    assert ops.read_device_status(DEV) == 0
    for (q, *p, t), (out, lse) in zip(problems, outs):
        ref_out, ref_lse = ops.decode(q, *p, 4, 32, SCALE, block_table=t)
        torch.testing.assert_close(out, ref_out, **NEAR)
        torch.testing.assert_close(lse, ref_lse, atol=1e-4, rtol=1e-5)
        _check_oracle(q, p, t, out, lse)


def test_batch_of_sequences_over_one_pool():
    pool = _pool(12, 7)
    seqs = [[0, 1, 2, 3], [4, 5], [6, 7, 8, 9, 10, 11], [11], [2, 4, 6, 8, 10]]
    problems = [(_query(200 + i), *pool, torch.tensor(s, dtype=torch.int32, device=DEV))
                for i, s in enumerate(seqs)]
    outs = ops.decode_batched(problems, 4, 32, SCALE)
    torch.cuda.synchronize()
    for (q, *p, t), (out, lse) in zip(problems, outs):
        ref_out, ref_lse = ops.decode(q, *p, 4, 32, SCALE, block_table=t)
        torch.testing.assert_close(out, ref_out, **NEAR)
        torch.testing.assert_close(lse, ref_lse, atol=1e-4, rtol=1e-5)
        _check_oracle(q, p, t, out, lse)


def test_refused_descriptor_is_flagged_and_others_decode():
    good = _pool(4, 3)
    raw = torch.empty(good[0].numel() + 8, dtype=torch.uint8, device=DEV)
    misaligned = raw[8:].view(good[0].shape)  # 8-byte aligned: the 16-byte copies refuse it
    misaligned.copy_(good[0])
    q = _query(5)
    problems = [(q, *good, None), (q, misaligned, *good[1:], None), (q, *good, None)]
    batch = ops.BatchedDecode(problems, 4, 32, SCALE)
    outs = batch.run()
    torch.cuda.synchronize()
    assert batch.read_status() & _native.DEV_BAD_PROBLEM
    ref_out, _ = ops.decode(q, *good, 4, 32, SCALE)
    torch.testing.assert_close(outs[0][0], ref_out, **NEAR)
    torch.testing.assert_close(outs[2][0], ref_out, **NEAR)
    # The refused problem's combining CTAs still count themselves, so the grid's epoch moves
    # on: later calls read this call's parts, not the previous call's (new query each time).
    for _ in range(2):
        q.neg_()
        outs = batch.run()
        torch.cuda.synchronize()
        ref_out, _ = ops.decode(q, *good, 4, 32, SCALE)
        torch.testing.assert_close(outs[0][0], ref_out, **NEAR)
        torch.testing.assert_close(outs[2][0], ref_out, **NEAR)


def test_batched_refuses_other_shapes():
    pool = _pool(2, 1, group=16)
    with pytest.raises(_native.NativeError, match="streaming kernel"):
        ops.decode_batched([(_query(1), *pool, None)], 4, 16, SCALE)


def test_batched_decode_replays_in_cuda_graph():
    pools = [_pool(3, 40 + i) for i in range(6)]
    queries = [_query(300 + i) for i in range(6)]
    batch = ops.BatchedDecode([(q, *p, None) for q, p in zip(queries, pools)], 4, 32, SCALE)
    eager = [o.clone() for o, _ in batch.run()]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        batch.run()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        batch.run()
    for q in queries:  # refill the queries in place: the replay decodes the new ones
        q.neg_()
    g.replay()
    torch.cuda.synchronize()
    for (q, *p), (out, _), before in zip(zip(queries, *zip(*pools)), batch.outs, eager):
        ref, _ = ops.decode(q, *p, 4, 32, SCALE)
        torch.testing.assert_close(out, ref, **NEAR)
        assert not torch.allclose(out, before)
    assert batch.read_status() == 0
