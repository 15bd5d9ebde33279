"""Our decode against the reference's own CUDA kernel (kvssd `csrc/fused_decode.cu`, built for
sm_100a by oracle/ref_cuda.py) on the same device inputs: outputs within the parity tolerance
of each other and of the CPU oracle, on a golden case and on the c1 configuration. The c1 test
also times both kernels (CUDA events, warm) and prints the ratio; the reference kernel runs one
CTA per query head and walks the tokens serially, so it is slower by orders of magnitude."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from kvssd_b200 import ops
from kvssd_b200.workloads import WORKLOADS, make_layer
from oracle import kvssd_oracle as orc
from oracle import ref_cuda

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
REF = ref_cuda.load()
needs_ref = pytest.mark.skipif(REF is None, reason="reference CUDA extension not built")


def _np(x) -> np.ndarray:
    if torch.is_tensor(x):
        return x.detach().cpu().float().numpy()
    return np.asarray(x, dtype=np.float32)


def _close(out, lse, ref_out, ref_lse):
    """FP16-rounded outputs within max-abs 2e-3 / rel 1e-2; LSE within 5e-3 / 1e-3."""
    got = _np(out).astype(np.float16).astype(np.float32)
    exp = _np(ref_out).astype(np.float16).astype(np.float32)
    np.testing.assert_allclose(got, exp, atol=2e-3, rtol=1e-2)
    np.testing.assert_allclose(_np(lse), _np(ref_lse), atol=5e-3, rtol=1e-3)


def _both(layer, bits, group, scale):
    t = [x.to(DEV) for x in (layer.query, layer.packed_k, layer.packed_v, layer.scales_k,
                             layer.scales_v, layer.valid_tokens)]
    ours = ops.decode(*t, bits, group, scale)
    theirs = REF.fused_decode(*t, bits, group, scale)
    torch.cuda.synchronize()
    return t, ours, theirs


@needs_ref
def test_reference_kernel_and_ours_agree_on_c1():
    w = WORKLOADS["c1"]
    layer = make_layer(w, 0, "cpu")
    scale = 1 / math.sqrt(w.head_dim)
    t, (out, lse), (rout, rlse) = _both(layer, w.bits, w.group_size, scale)
    _close(out, lse, rout, rlse)
    ro, rl = orc.decode(layer.query.float().numpy(), layer.packed_k.numpy(),
                        layer.packed_v.numpy(), layer.scales_k.numpy(), layer.scales_v.numpy(),
                        layer.valid_tokens.numpy(), w.bits, w.group_size, scale)
    _close(out, lse, ro, rl)
    _close(rout, rlse, ro, rl)

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps * 1e3

    ours_us = timed(lambda: ops.decode(*t, w.bits, w.group_size, scale), 50)
    ref_us = timed(lambda: REF.fused_decode(*t, w.bits, w.group_size, scale), 3)
    print(f"\nc1 decode on {torch.cuda.get_device_name(0)}: reference kernel {ref_us:.1f} us, "
          f"kvssd_b200 {ours_us:.1f} us (eager launches), ratio {ref_us / ours_us:.0f}x")
    assert ours_us < ref_us


@needs_ref
@pytest.mark.parametrize("bits", [2, 4])
def test_reference_kernel_and_ours_agree_on_a_ragged_case(bits):
    gen = torch.Generator().manual_seed(bits)
    from kvssd_b200.quant import quantize_tensor
    from kvssd_b200.workloads import LayerData

    k = torch.randn(5, 128, 8, 128, generator=gen).half()
    v = torch.randn(5, 128, 8, 128, generator=gen).half()
    kq, vq = quantize_tensor(k, bits, 32), quantize_tensor(v, bits, 32)
    layer = LayerData(torch.randn(32, 128, generator=gen).half(), kq.packed, vq.packed,
                      kq.scales, vq.scales, torch.tensor([128, 3, 128, 0, 77], dtype=torch.int32))
    scale = 1 / math.sqrt(128)
    _, (out, lse), (rout, rlse) = _both(layer, bits, 32, scale)
    _close(out, lse, rout, rlse)
