"""GPU parity of the fused decode kernels against the reference's golden outputs and the CPU
oracle. Tolerance (the parity target of this path): outputs cast to FP16 within max-abs 2e-3 and
rel 1e-2 of the reference CPU decode; LSE within 5e-3 abs + 1e-3 rel. Unpacked codes and FP16
dequantized values are bit-exact."""

from __future__ import annotations

import hashlib
import math

import numpy as np
import pytest
import torch
from conftest import QUERY_DTYPES, f16, golden_names, load_npz

from kvssd_b200 import B200AttentionBackend, PackedBatch, ops
from kvssd_b200 import _native
from kvssd_b200.workloads import WORKLOADS, make_layer
from oracle import kvssd_oracle as orc

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
OUT_ATOL, OUT_RTOL = 2e-3, 1e-2
LSE_ATOL, LSE_RTOL = 5e-3, 1e-3


def assert_parity(out, lse, ref_out, ref_lse):
    out = out.detach().float().cpu()
    lse = lse.detach().float().cpu()
    ref_out = torch.as_tensor(np.asarray(ref_out), dtype=torch.float32)
    ref_lse = torch.as_tensor(np.asarray(ref_lse), dtype=torch.float32)
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out.half().float(), ref_out.half().float(), atol=OUT_ATOL,
                               rtol=OUT_RTOL)
    assert torch.equal(torch.isneginf(lse), torch.isneginf(ref_lse))
    fin = torch.isfinite(ref_lse)
    torch.testing.assert_close(lse[fin], ref_lse[fin], atol=LSE_ATOL, rtol=LSE_RTOL)


def golden_batch(g):
    q = torch.from_numpy(g["query"]).to(QUERY_DTYPES[str(g["query_dtype"])]).to(DEV)
    batch = PackedBatch(
        torch.from_numpy(g["packed_k"]).to(DEV), torch.from_numpy(g["packed_v"]).to(DEV),
        torch.from_numpy(f16(g["scales_k"]).copy()).to(DEV),
        torch.from_numpy(f16(g["scales_v"]).copy()).to(DEV),
        torch.from_numpy(g["valid"]).to(DEV), int(g["bits"]), int(g["group"]),
    )
    return q, batch


@pytest.fixture
def path_override():
    def set_path(p):
        ops.set_path_override(p)
    yield set_path
    ops.set_path_override(_native.PATH_AUTO)


@pytest.mark.parametrize("name", golden_names("backend_"))
@pytest.mark.parametrize("path", [_native.PATH_AUTO, _native.PATH_TENSOR_CORE_CPASYNC,
                                  _native.PATH_TENSOR_CORE_REGS, _native.PATH_GENERIC])
def test_backend_matches_reference_golden(name, path, path_override):
    g = load_npz(name)
    q, batch = golden_batch(g)
    if path in (_native.PATH_TENSOR_CORE_REGS, _native.PATH_TENSOR_CORE_CPASYNC) and \
            ops.decode_path(q.shape[1], batch.bits, batch.group_size) != 1:
        pytest.skip("shape outside the tensor-core kernels")
    path_override(path)
    out, lse = B200AttentionBackend().run(q, batch, float(g["sm_scale"]))
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and lse.dtype == torch.float32
    assert out.shape == q.shape and lse.shape == (q.shape[0],)
    assert_parity(out, lse, g["out"], g["lse"])
    assert ops.read_device_status(DEV) == 0


def test_tensor_core_path_covers_benchmark_shapes():
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for bits in (2, 4):
        assert ops.decode_path(128, bits, 32) == _native.PATH_TENSOR_CORE
    plan = ops.decode_plan(1024, 128, 32, 8, 128, 4, 32)  # the 128K-token INT4 configuration
    assert plan["kernel"] == "tensor_core_tma", plan
    assert plan["n_parts"] == plan["n_splits"] <= sms
    assert ops.decode_plan(33, 128, 32, 8, 128, 2, 32)["kernel"] == "tensor_core_tma"  # INT2
    assert ops.decode_plan(33, 128, 32, 8, 64, 4, 32)["kernel"] == "tensor_core_regs"  # D = 64


@pytest.mark.parametrize("path", [_native.PATH_AUTO, _native.PATH_TENSOR_CORE_CPASYNC,
                                  _native.PATH_TENSOR_CORE_REGS, _native.PATH_GENERIC])
@pytest.mark.parametrize("kvh,qh,bits", [(8, 32, 4), (8, 32, 2), (4, 16, 4), (4, 16, 2),
                                         (16, 32, 2), (2, 16, 4),
                                         (1, 8, 4), (8, 8, 4), (16, 32, 4)])
def test_kernels_agree_with_oracle_across_head_layouts(kvh, qh, bits, path, path_override):
    """Every decode kernel against the oracle for KV-head counts that change the streaming ring
    layout (row bytes 64..1024) and the warps-per-head split, including partial tiles."""
    pool = _pool(nb=9, kvh=kvh, bits=bits, valid=[128, 128, 100, 128, 3, 128, 128, 64, 17])
    q = torch.randn(qh, 128, generator=torch.Generator().manual_seed(kvh * 100 + qh)).half()
    path_override(path)
    out, lse = _run(q, pool, bits, 32, [8, 0, 1, 2, 3, 4, 5, 6, 7, 2])
    assert_parity(out, lse, *_oracle(q, pool, bits, 32, [8, 0, 1, 2, 3, 4, 5, 6, 7, 2]))
    assert ops.read_device_status(DEV) == 0


@pytest.mark.parametrize("name", golden_names("quant_"))
@pytest.mark.parametrize("mode", [0, 1])
def test_register_unpacker_bit_exact_vs_reference(name, mode):
    g = load_npz(name)
    bits = int(name.split("_b")[1][0])
    group = int(name.split("_g")[1].split(".")[0])
    for tag in ("f32", "f16"):
        packed = torch.from_numpy(g[f"packed_{tag}"]).reshape(15, -1)
        scales = torch.from_numpy(f16(g[f"scales_{tag}"]).copy()).reshape(15, -1)
        rows = 14 if mode == 1 else 15
        codes, values = ops.dequantize_packed(packed[:rows].to(DEV), scales[:rows].to(DEV), bits,
                                              group, mode)
        np.testing.assert_array_equal(codes.cpu().numpy(), g[f"codes_{tag}"].reshape(15, -1)[:rows])
        np.testing.assert_array_equal(values.cpu().view(torch.int16).numpy().view(np.uint16),
                                      g[f"deq16_{tag}"].reshape(15, -1)[:rows])


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("d,group", [(64, 16), (128, 32), (128, 16), (256, 64), (128, 128)])
@pytest.mark.parametrize("mode", [0, 1])
def test_register_unpacker_bit_exact_exhaustive(bits, d, group, mode):
    """Every code value in every lane position, with scales spanning subnormal to large FP16."""
    rng = np.random.default_rng(7 + bits + d + group + mode)
    rows = 4096
    packed = rng.integers(0, 256, size=(rows, d * bits // 8), dtype=np.uint8)
    sbits = rng.integers(0, 0x7C00, size=(rows, d // group), dtype=np.uint16)  # finite, >= 0
    sbits[:64] = rng.integers(0, 0x0400, size=(64, d // group))  # subnormal scales
    scales = sbits.view(np.float16)
    codes, values = ops.dequantize_packed(torch.from_numpy(packed).to(DEV),
                                          torch.from_numpy(scales.copy()).to(DEV), bits, group, mode)
    np.testing.assert_array_equal(codes.cpu().numpy(), orc.unpack_codes(packed, bits, d))
    expect = orc.dequantize(packed, scales, bits, group, d, np.float16)
    np.testing.assert_array_equal(values.cpu().view(torch.int16).numpy().view(np.uint16),
                                  expect.view(np.uint16))


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("config", ["c1", "c3", "c2"])
def test_benchmark_configs_match_reference_decode(config):
    """Full-size C1/C3/C2 inputs (seeded, quantized on the CPU) against the reference
    backend's own output for the same inputs."""
    g = load_npz(f"config_{config}.npz")
    w = WORKLOADS[config]
    layer = make_layer(w, 0, "cpu")
    assert _sha(layer.packed_k) == str(g["sha_packed_k"])
    assert _sha(layer.scales_v) == str(g["sha_scales_v"])
    sel = torch.tensor(g["selected"].tolist(), dtype=torch.int32)
    out, lse = ops.decode(layer.query.to(DEV), layer.packed_k.to(DEV), layer.packed_v.to(DEV),
                          layer.scales_k.to(DEV), layer.scales_v.to(DEV),
                          layer.valid_tokens.to(DEV), w.bits, w.group_size,
                          1.0 / math.sqrt(w.head_dim), block_table=sel.to(DEV))
    torch.cuda.synchronize()
    assert_parity(out, lse, g["out"], g["lse"])


def _pool(nb=12, bt=128, kvh=8, d=128, bits=4, group=32, seed=0, valid=None):
    gen = torch.Generator().manual_seed(seed)
    k = torch.randn(nb, bt, kvh, d, generator=gen).half()
    v = torch.randn(nb, bt, kvh, d, generator=gen).half()
    from kvssd_b200.quant import quantize_tensor
    kq, vq = quantize_tensor(k, bits, group), quantize_tensor(v, bits, group)
    if valid is None:
        valid = [bt] * nb
    return [kq.packed, vq.packed, kq.scales, vq.scales, torch.tensor(valid, dtype=torch.int32)]


def _oracle(q, pool, bits, group, table=None):
    kp, vp, ks, vs, valid = [t.cpu().numpy() for t in pool]
    return orc.decode(q.float().cpu().numpy(), kp, vp, ks, vs, valid, bits, group,
                      1.0 / math.sqrt(q.shape[1]), block_table=table)


def _run(q, pool, bits, group, table=None):
    dev = [t.to(DEV) for t in pool]
    tab = None if table is None else torch.tensor(table, dtype=torch.int32, device=DEV)
    out, lse = ops.decode(q.to(DEV), *dev, bits, group, 1.0 / math.sqrt(q.shape[1]), block_table=tab)
    torch.cuda.synchronize()
    return out, lse


@pytest.mark.parametrize("bits", [2, 4])
def test_block_table_selection_order_and_duplicates(bits):
    pool = _pool(bits=bits, valid=[128, 77, 128, 0, 5, 128, 128, 1, 128, 128, 16, 17])
    q = torch.randn(32, 128, generator=torch.Generator().manual_seed(3)).half()
    for table in ([0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11], [11, 3, 5, 0], [7], [2, 2, 9, 2],
                  list(range(11, -1, -1)), [3]):
        out, lse = _run(q, pool, bits, 32, table)
        ref = _oracle(q, pool, bits, 32, table)
        assert_parity(out, lse, *ref)
    assert ops.read_device_status(DEV) == 0


def test_all_selected_blocks_empty_gives_zero_and_neg_inf():
    pool = _pool(nb=3, valid=[0, 0, 0])
    q = torch.randn(32, 128).half()
    out, lse = _run(q, pool, 4, 32)
    assert torch.all(out == 0) and torch.all(torch.isneginf(lse))


def test_invalid_block_table_and_valid_entries_are_flagged_not_read():
    pool = _pool(nb=4, valid=[128, 300, -5, 64])
    q = torch.randn(32, 128, generator=torch.Generator().manual_seed(1)).half()
    ops.read_device_status(DEV)  # clear
    out, lse = _run(q, pool, 4, 32, [0, 7, -1, 3, 1, 2])
    status = ops.read_device_status(DEV)
    assert status & 1 and status & 2
    clamped = [t.clone() for t in pool]
    clamped[4] = torch.tensor([128, 128, 0, 64], dtype=torch.int32)
    ref = _oracle(q, clamped, 4, 32, [0, 3, 1, 2])
    assert_parity(out, lse, *ref)
    assert ops.read_device_status(DEV) == 0


@pytest.mark.parametrize("qdtype", [torch.float16, torch.bfloat16, torch.float32, torch.float64])
def test_query_dtypes(qdtype):
    pool = _pool(nb=6)
    q = torch.randn(32, 128, generator=torch.Generator().manual_seed(9)).to(qdtype)
    out, lse = _run(q, pool, 4, 32)
    assert_parity(out, lse, *_oracle(q, pool, 4, 32))


def test_unaligned_pool_views_use_generic_kernel():
    pool = _pool(nb=3)
    dev = [t.to(DEV) for t in pool]
    raw = torch.empty(dev[0].numel() + 4, dtype=torch.uint8, device=DEV)
    kp_view = raw[4:].view(dev[0].shape)  # 4-byte aligned, not 16
    kp_view.copy_(dev[0])
    q = torch.randn(32, 128).half()
    out, lse = ops.decode(q.to(DEV), kp_view, dev[1], dev[2], dev[3], dev[4], 4, 32,
                          1 / math.sqrt(128))
    torch.cuda.synchronize()
    assert_parity(out, lse, *_oracle(q, pool, 4, 32))


def test_single_token_and_single_block():
    pool = _pool(nb=1, valid=[1])
    q = torch.randn(32, 128).half()
    out, lse = _run(q, pool, 4, 32)
    assert_parity(out, lse, *_oracle(q, pool, 4, 32))


def test_many_blocks_cross_block_cache_refills():
    pool = _pool(nb=100, bt=16, valid=[16 if i % 7 else i % 16 for i in range(100)], seed=4)
    q = torch.randn(32, 128).half()
    table = list(range(99, -1, -3)) + list(range(0, 100, 5))
    out, lse = _run(q, pool, 4, 32, table)
    assert_parity(out, lse, *_oracle(q, pool, 4, 32, table))


def test_decode_is_deterministic():
    pool = _pool(nb=20)
    q = torch.randn(32, 128).half()
    a = _run(q, pool, 4, 32)
    b = _run(q, pool, 4, 32)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_merge_kernels_match_reference():
    g = load_npz("merge.npz")
    t = {k: torch.from_numpy(v).to(DEV) for k, v in g.items()}
    out, lse = ops.merge_pair(t["lo"], t["ll"], t["ro"], t["rl"])
    torch.testing.assert_close(out.cpu(), torch.from_numpy(g["out"]), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(lse.cpu(), torch.from_numpy(g["lse"]), atol=1e-6, rtol=1e-5)
    out, lse = ops.merge_chunks(torch.stack([t["lo"], t["ro"]]), torch.stack([t["ll"], t["rl"]]))
    torch.testing.assert_close(out.cpu(), torch.from_numpy(g["out"]), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(lse.cpu(), torch.from_numpy(g["lse"]), atol=1e-6, rtol=1e-5)


def test_split_merge_property_at_c2_size():
    """Size-independent property at the headline size: decoding two halves of the selection
    and merging their (out, lse) equals decoding the whole selection."""
    w = WORKLOADS["c2"]
    layer = make_layer(w, 0, DEV)
    args = (layer.packed_k, layer.packed_v, layer.scales_k, layer.scales_v, layer.valid_tokens,
            w.bits, w.group_size, 1 / math.sqrt(w.head_dim))
    whole = ops.decode(layer.query, *args)
    n = w.blocks_per_layer
    halves = [torch.arange(0, n // 3, dtype=torch.int32, device=DEV),
              torch.arange(n // 3, n, dtype=torch.int32, device=DEV)]
    parts = [ops.decode(layer.query, *args, block_table=h) for h in halves]
    merged = ops.merge_chunks(torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts]))
    rev = ops.decode(layer.query, *args, block_table=torch.arange(n - 1, -1, -1, dtype=torch.int32,
                                                                   device=DEV))
    torch.cuda.synchronize()
    # Re-ordering changes split boundaries and summation order only: agreement far inside the
    # parity tolerance (2e-3 abs), limited by FP32/FP16 rounding of the accumulation order.
    torch.testing.assert_close(merged[0], whole[0], atol=5e-5, rtol=1e-3)
    torch.testing.assert_close(merged[1], whole[1], atol=5e-5, rtol=1e-5)
    torch.testing.assert_close(rev[0], whole[0], atol=5e-5, rtol=1e-3)
    # linearity in V's scales: scaling every V scale by 2 scales the output by 2 exactly
    v2 = (layer.scales_v.float() * 2).half()
    doubled = ops.decode(layer.query, layer.packed_k, layer.packed_v, layer.scales_k, v2,
                         layer.valid_tokens, w.bits, w.group_size, 1 / math.sqrt(w.head_dim))
    torch.cuda.synchronize()
    torch.testing.assert_close(doubled[0], 2 * whole[0], atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("group", [32, 64])
def test_int2_streaming_kernel_matches_oracle(group):
    """INT2 through the TMA-fed streaming kernel (tiles dequantized in registers): both scale
    group sizes, identity selection with ragged blocks, and a block table."""
    pool = _pool(nb=11, bits=2, group=group, seed=group,
                 valid=[128, 5, 128, 128, 0, 128, 77, 128, 128, 16, 128])
    q = torch.randn(32, 128, generator=torch.Generator().manual_seed(group + 1)).half()
    assert ops.decode_plan(11, 128, 32, 8, 128, 2, group)["kernel"] == "tensor_core_tma"
    assert_parity(*_run(q, pool, 2, group), *_oracle(q, pool, 2, group))
    table = [10, 0, 3, 3, 9, 6]
    assert_parity(*_run(q, pool, 2, group, table), *_oracle(q, pool, 2, group, table))
    assert ops.read_device_status(DEV) == 0


def test_c3_shape_int2_outliers_recent_sink():
    """The c3 configuration's shape at a reduced size: INT2 with 1 % outlier channels x8 and a
    RecentSinkBlocks(1, 32) selection through a block table."""
    import dataclasses

    from kvssd_b200 import RecentSinkBlocks
    from kvssd_b200.workloads import WORKLOADS, make_layer

    w = dataclasses.replace(WORKLOADS["c3"], tokens=64 * 128, seed=33)
    layer = make_layer(w, 0, "cpu")
    sel = RecentSinkBlocks(w.sink, w.recent).select(list(range(layer.packed_k.shape[0])))
    pool = (layer.packed_k, layer.packed_v, layer.scales_k, layer.scales_v, layer.valid_tokens)
    out, lse = _run(layer.query, pool, 2, 32, sel)
    assert_parity(out, lse, *_oracle(layer.query, pool, 2, 32, sel))
    assert ops.read_device_status(DEV) == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32, torch.float64])
def test_unaligned_query_takes_the_element_load_path(dtype):
    """A query view that is not 16-byte aligned (offset by one element) is read element by
    element instead of through the per-CTA bulk copy / vector loads; results are identical to
    the aligned query's."""
    pool = _pool(nb=6, seed=5, valid=[128, 128, 90, 128, 1, 128])
    q = torch.randn(32, 128, generator=torch.Generator().manual_seed(6)).to(dtype)
    backing = torch.empty(32 * 128 + 1, dtype=dtype, device=DEV)
    unaligned = backing[1:].view(32, 128)
    unaligned.copy_(q.to(DEV))
    assert unaligned.data_ptr() % 16 != 0
    dev = [t.to(DEV) for t in pool]
    scale = 1.0 / math.sqrt(128)
    out_u, lse_u = ops.decode(unaligned, *dev, 4, 32, scale)
    out_a, lse_a = ops.decode(q.to(DEV).contiguous(), *dev, 4, 32, scale)
    torch.cuda.synchronize()
    assert torch.equal(out_u, out_a) and torch.equal(lse_u, lse_a)
    assert_parity(out_u, lse_u, *_oracle(q.float(), pool, 4, 32))
    assert ops.read_device_status(DEV) == 0


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("kvh,qh", [(4, 16), (16, 32)])
def test_streaming_group64_scale_row_layouts(kvh, qh, bits):
    """Group 64 with 4 and 16 KV heads: the streaming kernel's scale rows are then 16 and 64
    bytes (no swizzle / the 64-byte swizzle) -- layouts the group-32 cases do not reach."""
    pool = _pool(nb=7, kvh=kvh, bits=bits, group=64, seed=kvh + bits,
                 valid=[128, 128, 33, 128, 0, 128, 9])
    q = torch.randn(qh, 128, generator=torch.Generator().manual_seed(kvh * 7 + bits)).half()
    assert ops.decode_plan(7, 128, qh, kvh, 128, bits, 64)["kernel"] == "tensor_core_tma"
    assert_parity(*_run(q, pool, bits, 64), *_oracle(q, pool, bits, 64))
    table = [6, 1, 1, 3, 0]
    assert_parity(*_run(q, pool, bits, 64, table), *_oracle(q, pool, bits, 64, table))
    assert ops.read_device_status(DEV) == 0
