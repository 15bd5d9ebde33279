"""kvssd_b200_decode_static (the allocation-free decode entry) against kvssd_b200_decode.

Called through the C ABI with ctypes, the way a host without a device allocator binds it.
The file sorts last so the entry point is also exercised after every other GPU test has run
in the same process.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from kvssd_b200 import _native, ops
from kvssd_b200.workloads import WORKLOADS, make_layer

pytestmark = pytest.mark.gpu


def _static_decode(layer, w, out, lse, scratch: ctypes.c_void_p) -> int:
    q = layer.query
    n, bt, kvh, _ = layer.packed_k.shape
    qh, d = q.shape
    return _native.library().kvssd_b200_decode_static(
        q.data_ptr(), _native.Q_F16,
        layer.packed_k.data_ptr(), layer.packed_v.data_ptr(),
        layer.scales_k.data_ptr(), layer.scales_v.data_ptr(),
        layer.valid_tokens.data_ptr(), None,
        n, n, bt, qh, kvh, d, w.bits, w.group_size, 1.0 / math.sqrt(d),
        out.data_ptr(), lse.data_ptr(), ctypes.byref(scratch),
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_static_scratch_decode_matches_workspace_decode(name):
    w = WORKLOADS[name]
    layer = make_layer(w, 0, "cuda")
    ref_out, ref_lse = ops.decode(layer.query, layer.packed_k, layer.packed_v, layer.scales_k,
                                  layer.scales_v, layer.valid_tokens, w.bits, w.group_size,
                                  1.0 / math.sqrt(w.head_dim))
    scratch = ctypes.c_void_p()
    for _ in range(2):  # two calls in a row reuse the same device scratch
        out = torch.full_like(ref_out, float("nan"))
        lse = torch.full_like(ref_lse, float("nan"))
        _native.check(_static_decode(layer, w, out, lse, scratch), "kvssd_b200_decode_static")
        torch.cuda.synchronize()
        torch.testing.assert_close(out.half(), ref_out.half(), atol=2e-3, rtol=1e-2)
        torch.testing.assert_close(lse, ref_lse, atol=5e-3, rtol=1e-3)
    assert scratch.value is not None and scratch.value % 256 == 0
    status = ctypes.c_uint(99)
    _native.check(_native.library().kvssd_b200_read_status(
        scratch.value, 1, ctypes.byref(status), torch.cuda.current_stream().cuda_stream),
        "kvssd_b200_read_status")
    assert status.value == 0


def test_static_scratch_rejects_geometry_beyond_its_size():
    # 128 query heads x (128 + 2) floats per part over 148 parts exceeds the 8 MiB scratch;
    # the call must refuse before launching anything.
    qh, kvh, d, bt, n = 128, 16, 128, 128, 64
    dev = torch.device("cuda")
    q = torch.zeros((qh, d), dtype=torch.float16, device=dev)
    pk = torch.zeros((n, bt, kvh, d // 2), dtype=torch.uint8, device=dev)
    sk = torch.zeros((n, bt, kvh, d // 32), dtype=torch.float16, device=dev)
    valid = torch.full((n,), bt, dtype=torch.int32, device=dev)
    out = torch.zeros((qh, d), dtype=torch.float32, device=dev)
    lse = torch.zeros((qh,), dtype=torch.float32, device=dev)
    status = _native.library().kvssd_b200_decode_static(
        q.data_ptr(), _native.Q_F16, pk.data_ptr(), pk.data_ptr(), sk.data_ptr(), sk.data_ptr(),
        valid.data_ptr(), None, n, n, bt, qh, kvh, d, 4, 32, 1.0, out.data_ptr(),
        lse.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    assert status == _native.ERR_WORKSPACE
    detail = _native.library().kvssd_b200_last_error().decode()
    assert "static scratch holds" in detail and str(8 << 20) in detail
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0


class _DeviceBytes:
    """A raw device address exposed to torch without a copy (CUDA array interface)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def test_static_scratch_recovers_after_a_wait_that_gave_up():
    # A caller without an allocator cannot re-zero the scratch itself: reading the status with
    # clear = 1 after a failed call must leave the scratch ready for the next call.
    w = WORKLOADS["c1"]
    layer = make_layer(w, 0, "cuda")
    ref_out, ref_lse = ops.decode(layer.query, layer.packed_k, layer.packed_v, layer.scales_k,
                                  layer.scales_v, layer.valid_tokens, w.bits, w.group_size,
                                  1.0 / math.sqrt(w.head_dim))
    scratch = ctypes.c_void_p()
    out = torch.empty_like(ref_out)
    lse = torch.empty_like(ref_lse)
    _native.check(_static_decode(layer, w, out, lse, scratch), "kvssd_b200_decode_static")
    torch.cuda.synchronize()
    header = torch.as_tensor(_DeviceBytes(scratch.value, 2048), device="cuda")
    # the fused combine's test hook: part 0 is expected with a tag no CTA writes, it gives up
    header[132:136] = torch.tensor([1, 0, 0, 0], dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    _native.check(_static_decode(layer, w, out, lse, scratch), "kvssd_b200_decode_static")
    torch.cuda.synchronize()
    assert torch.isnan(out).all() and torch.isnan(lse).all()
    status = ctypes.c_uint()
    rc = _native.library().kvssd_b200_read_status(
        scratch.value, 1, ctypes.byref(status), torch.cuda.current_stream().cuda_stream)
    assert rc == _native.ERR_DEVICE_STATUS and status.value & 4
    torch.cuda.synchronize()
    assert torch.count_nonzero(header[:4]) == 0  # status word cleared
    assert torch.count_nonzero(header[132:140]) == 0  # hook and batched counter at zero
    for _ in range(2):
        _native.check(_static_decode(layer, w, out, lse, scratch), "kvssd_b200_decode_static")
        torch.cuda.synchronize()
        torch.testing.assert_close(out.half(), ref_out.half(), atol=2e-3, rtol=1e-2)
        torch.testing.assert_close(lse, ref_lse, atol=5e-3, rtol=1e-3)
