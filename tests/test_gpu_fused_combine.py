"""The streaming kernel's fused split-KV combine: equality with the two-launch path, the
epoch advancing by one per call, and the bounded wait (the header's test hook makes the
combining CTAs expect a tag of part 0 that no CTA writes, so they give up after about a second
and flag status bit 4; nothing faults or hangs). A call that gave up returns NaN, later calls on the workspace return
NaN until the status word is cleared, and the public entry points (the ``cuda`` backend's run,
DeviceBlockPool) raise ops.DeviceFailure on the next call instead of returning a number."""

from __future__ import annotations

import math
import time

import pytest
import torch

from kvssd_b200 import _native, ops
from kvssd_b200.workloads import WORKLOADS, make_layer

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
EPOCH = 128  # byte offset of the fused combine's epoch in the workspace header
HOOK = 132   # the test hook word after it (zero in normal use)


def _word(ws, off) -> int:
    return int(ws[off:off + 4].cpu().view(torch.int32)[0])


def _plant_hook(ws) -> None:
    ws[HOOK:HOOK + 4] = torch.tensor([1, 0, 0, 0], dtype=torch.uint8, device=ws.device)


@pytest.fixture(scope="module")
def layer():
    w = WORKLOADS["c1"]
    cpu = make_layer(w, 0, "cpu")
    return w, [t.to(DEV) for t in (cpu.query, cpu.packed_k, cpu.packed_v, cpu.scales_k,
                                   cpu.scales_v, cpu.valid_tokens)]


def _workspace(w, tensors) -> torch.Tensor:
    q, kp = tensors[0], tensors[1]
    n, bt, kvh, _ = kp.shape
    import ctypes
    need = ctypes.c_size_t()
    _native.check(_native.library().kvssd_b200_decode_workspace_size(
        n, bt, q.shape[0], kvh, q.shape[1], w.bits, w.group_size, ctypes.byref(need)), "size")
    return torch.zeros(need.value, dtype=torch.uint8, device=DEV)


def _abi_decode(w, tensors, ws):
    q, kp, vp, ks, vs, valid = tensors
    n, bt, kvh, _ = kp.shape
    qh, d = q.shape
    out = torch.full((qh, d), float("nan"), device=DEV)
    lse = torch.full((qh,), float("nan"), device=DEV)
    _native.check(_native.library().kvssd_b200_decode(
        q.data_ptr(), _native.Q_F16, kp.data_ptr(), vp.data_ptr(), ks.data_ptr(), vs.data_ptr(),
        valid.data_ptr(), None, n, n, bt, qh, kvh, d, w.bits, w.group_size,
        1.0 / math.sqrt(d), out.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream().cuda_stream), "kvssd_b200_decode")
    return out, lse


def _status(ws) -> int:
    import ctypes
    st = ctypes.c_uint()
    _native.library().kvssd_b200_read_status(ws.data_ptr(), 1, ctypes.byref(st),
                                             torch.cuda.current_stream().cuda_stream)
    return st.value


def test_streaming_plan_fuses_the_combine(layer):
    w, t = layer
    plan = ops.decode_plan(t[1].shape[0], w.block_tokens, w.query_heads, w.kv_heads, w.head_dim,
                           w.bits, w.group_size)
    assert plan["kernel"] in ops.STREAMING_KERNELS


def test_fused_combine_equals_two_launch_combine_and_advances_the_epoch(layer):
    w, t = layer
    ws = _workspace(w, t)
    fused = _abi_decode(w, t, ws)
    torch.cuda.synchronize()
    assert _word(ws, EPOCH) == 1 and _word(ws, HOOK) == 0  # a zeroed workspace starts at 1
    assert _status(ws) == 0
    args = (t[0], *t[1:], w.bits, w.group_size, 1.0 / math.sqrt(w.head_dim))
    n_parts, wsp = ops.decode_split(*args)
    two = ops.decode_combine(wsp, n_parts, w.query_heads, w.head_dim)
    torch.cuda.synchronize()
    torch.testing.assert_close(fused[0], two[0], atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(fused[1], two[1], atol=1e-6, rtol=1e-6)
    for call in (2, 3):  # the parts of the previous call carry an older tag
        again = _abi_decode(w, t, ws)
        torch.cuda.synchronize()
        assert _word(ws, EPOCH) == call
        assert torch.equal(again[0], fused[0]) and torch.equal(again[1], fused[1])


def test_fused_combine_wait_is_bounded_and_flagged(layer):
    w, t = layer
    ws = _workspace(w, t)
    _abi_decode(w, t, ws)
    _plant_hook(ws)  # part 0 is expected with a tag that no CTA writes
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    bad_out, bad_lse = _abi_decode(w, t, ws)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert torch.isnan(bad_out).all() and torch.isnan(bad_lse).all()
    assert _word(ws, HOOK) == 0  # the combiners cleared the hook after giving up
    # the word is sticky: until it is cleared, every call on this workspace fails closed
    again_out, _ = _abi_decode(w, t, ws)
    torch.cuda.synchronize()
    assert torch.isnan(again_out).all()
    assert _status(ws) & 4
    assert elapsed < 30
    out, lse = _abi_decode(w, t, ws)  # _status cleared the word
    ref = ops.decode(*t, w.bits, w.group_size, 1.0 / math.sqrt(w.head_dim))
    torch.cuda.synchronize()
    assert _status(ws) == 0
    torch.testing.assert_close(out, ref[0], atol=1e-6, rtol=1e-6)


def _plant_unreachable_count(device=DEV):
    """Plants the test hook in the current stream's ops workspace: the next fused combine
    waits for a part 0 tag that no CTA writes."""
    ws = ops._workspaces.get(device, torch.cuda.current_stream(device), 1 << 20)
    _plant_hook(ws)
    torch.cuda.synchronize()


def test_backend_run_raises_after_a_failed_call(layer):
    from kvssd_b200 import B200AttentionBackend, PackedBatch

    w, t = layer
    backend = B200AttentionBackend()
    batch = PackedBatch(*t[1:], w.bits, w.group_size)
    scale = 1.0 / math.sqrt(w.head_dim)
    good, _ = backend.run(t[0], batch, scale)
    backend.check(DEV)
    good = good.clone()
    _plant_unreachable_count()
    bad, bad_lse = backend.run(t[0], batch, scale)  # gives up after about a second
    torch.cuda.synchronize()
    assert torch.isnan(bad).all() and torch.isnan(bad_lse).all()
    with pytest.raises(ops.DeviceFailure) as info:
        backend.run(t[0], batch, scale)  # the earlier call's failure surfaces here
    assert info.value.status & 4
    # raising cleared the word and re-armed the workspace: the next call is good again
    out, _ = backend.run(t[0], batch, scale)
    backend.check(DEV)
    torch.testing.assert_close(out, good, atol=0, rtol=0)


def test_pool_check_raises_after_a_failed_call(layer):
    from kvssd_b200 import CacheSpec
    from kvssd_b200.pool import DeviceBlockPool

    w, t = layer
    spec = CacheSpec(1, w.kv_heads, w.head_dim, w.block_tokens, w.bits, w.group_size)
    pool = DeviceBlockPool(spec, *t[1:])
    good, _ = pool.decode(t[0])
    pool.check()
    good = good.clone()
    _plant_unreachable_count()
    bad, _ = pool.decode(t[0])
    with pytest.raises(ops.DeviceFailure):
        pool.check()
    assert torch.isnan(bad).all()
    out, _ = pool.decode(t[0])
    pool.check()
    torch.testing.assert_close(out, good, atol=0, rtol=0)


def test_out_of_pool_table_entry_raises_on_the_next_call(layer):
    from kvssd_b200 import CacheSpec
    from kvssd_b200.pool import DeviceBlockPool

    w, t = layer
    spec = CacheSpec(1, w.kv_heads, w.head_dim, w.block_tokens, w.bits, w.group_size)
    pool = DeviceBlockPool(spec, *t[1:])
    table = torch.tensor([0, 1, 10_000], dtype=torch.int32, device=DEV)
    out, _ = pool.decode_table(t[0], table)  # the bad entry is skipped, never read
    torch.cuda.synchronize()  # the status read of that call has landed in pinned memory
    with pytest.raises(ops.DeviceFailure) as info:
        pool.decode_table(t[0], table[:2].contiguous())
    assert info.value.status & 1
    assert torch.isfinite(out).all()
