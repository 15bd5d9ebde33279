"""Pins the CPU oracle to golden vectors produced by the reference implementation."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import f16, golden_names, load_json, load_npz

from oracle import kvssd_oracle as orc

QUANT = golden_names("quant_")
BACKEND = golden_names("backend_")


@pytest.mark.parametrize("name", QUANT)
def test_oracle_quantizer_bit_exact(name):
    g = load_npz(name)
    bits = int(name.split("_b")[1][0])
    group = int(name.split("_g")[1].split(".")[0])
    for tag in ("f32", "f16"):
        x = g[f"x_{tag}"]
        packed, scales = orc.quantize(x, bits, group)
        np.testing.assert_array_equal(packed, g[f"packed_{tag}"])
        np.testing.assert_array_equal(scales.view(np.uint16), g[f"scales_{tag}"])
        np.testing.assert_array_equal(orc.unpack_codes(packed, bits, 128), g[f"codes_{tag}"])
        np.testing.assert_array_equal(orc.pack_codes(g[f"codes_{tag}"], bits), packed)
        deq32 = orc.dequantize(packed, scales, bits, group, 128)
        np.testing.assert_array_equal(deq32, g[f"deq32_{tag}"])
        deq16 = orc.dequantize(packed, scales, bits, group, 128, np.float16)
        np.testing.assert_array_equal(deq16.view(np.uint16), g[f"deq16_{tag}"])


@pytest.mark.parametrize("name", BACKEND)
def test_oracle_decode_matches_reference_backend(name):
    g = load_npz(name)
    out, lse = orc.decode(g["query"].astype(np.float32), g["packed_k"], g["packed_v"],
                          f16(g["scales_k"]), f16(g["scales_v"]), g["valid"], int(g["bits"]),
                          int(g["group"]), float(g["sm_scale"]))
    np.testing.assert_allclose(out, g["out"], atol=2e-6, rtol=2e-5)
    np.testing.assert_allclose(lse, g["lse"], atol=2e-6, rtol=2e-5)


def test_oracle_chunked_decode_equals_single_pass():
    g = load_npz("backend_gqa4_b4_32_8_128.npz")
    args = (g["query"].astype(np.float32), g["packed_k"], g["packed_v"], f16(g["scales_k"]),
            f16(g["scales_v"]), g["valid"], 4, int(g["group"]), float(g["sm_scale"]))
    whole = orc.decode(*args, chunk_blocks=1024)
    chunked = orc.decode(*args, chunk_blocks=1)
    np.testing.assert_allclose(chunked[0], whole[0], atol=1e-6, rtol=1e-5)
    np.testing.assert_allclose(chunked[1], whole[1], atol=1e-6, rtol=1e-5)


def test_oracle_merge_matches_reference():
    g = load_npz("merge.npz")
    out, lse = orc.merge_pair(g["lo"], g["ll"], g["ro"], g["rl"])
    np.testing.assert_allclose(out, g["out"], atol=1e-6, rtol=1e-5)
    np.testing.assert_allclose(lse, g["lse"], atol=1e-6, rtol=1e-5)


def test_oracle_selectors_match_reference():
    for case in load_json("selectors.json"):
        assert orc.recent_sink(case["available"], case["sink"], case["recent"]) == case["chosen"]
    with pytest.raises(ValueError):
        orc.recent_sink([1, 2], -1, 0)


@pytest.mark.parametrize("bits", [2, 4])
def test_oracle_dense_reference_matches_packed_attention(bits):
    g = load_npz(f"packed_attention_b{bits}.npz")
    keys, values = g["keys"][0], g["values"][0]
    bt, kvh, d = 8, 2, 32
    nb = -(-keys.shape[0] // bt)
    kpad = np.zeros((nb * bt, kvh, d), np.float32)
    vpad = np.zeros_like(kpad)
    kpad[: keys.shape[0]] = keys
    vpad[: keys.shape[0]] = values
    kp, ks = orc.quantize(kpad.reshape(nb, bt, kvh, d), bits, 16)
    vp, vs = orc.quantize(vpad.reshape(nb, bt, kvh, d), bits, 16)
    valid = np.array([8, 5], dtype=np.int32)
    out, _ = orc.decode(g["query"], kp, vp, ks, vs, valid, bits, 16, 1 / np.sqrt(d))
    np.testing.assert_allclose(out, g["out"], atol=2e-6, rtol=2e-5)
    kd = orc.dequantize(kp, ks, bits, 16, d).reshape(-1, kvh, d)[: keys.shape[0]]
    vd = orc.dequantize(vp, vs, bits, 16, d).reshape(-1, kvh, d)[: keys.shape[0]]
    np.testing.assert_allclose(orc.reference_attention(g["query"], kd, vd), g["out"],
                               atol=2e-6, rtol=2e-5)


def test_oracle_empty_selection_semantics():
    # All blocks empty: the reference returns lse = -inf and a zero output.
    g = load_npz("backend_mk_b4_1_1_32.npz")
    out, lse = orc.decode(g["query"], g["packed_k"], g["packed_v"], f16(g["scales_k"]),
                          f16(g["scales_v"]), np.zeros(2, np.int32), 4, 16, 0.1)
    assert np.all(out == 0) and np.all(np.isneginf(lse))
