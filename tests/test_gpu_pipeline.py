"""GPU end-to-end: store -> selector -> staging -> fused decode -> merge, against the
reference's golden packed_attention outputs and the CPU oracle."""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch
from conftest import load_npz
from test_gpu_decode import DEV, assert_parity

from kvssd_b200 import (
    AllBlocks,
    CacheSpec,
    DeviceBlockPool,
    KVCacheStore,
    KVSSDPipeline,
    RecentSinkBlocks,
    fused_attention_tensors,
    merge_attention_chunks,
    packed_attention,
    resolve_attention_backend,
)
from oracle import kvssd_oracle as orc

pytestmark = pytest.mark.gpu


def _store(tmp: Path, tokens=600, kvh=8, d=128, bt=16, bits=4, group=32, seed=11):
    gen = torch.Generator().manual_seed(seed)
    k = torch.randn(1, tokens, kvh, d, generator=gen)
    v = torch.randn(1, tokens, kvh, d, generator=gen)
    return KVCacheStore.create(tmp, k, v, CacheSpec(1, kvh, d, bt, bits, group))


def _oracle_for(store: KVCacheStore, q: torch.Tensor, selected: list[int]):
    blocks = [store.read(0, b) for b in selected]
    kp = np.stack([b.key.packed.numpy() for b in blocks])
    vp = np.stack([b.value.packed.numpy() for b in blocks])
    ks = np.stack([b.key.scales.numpy() for b in blocks])
    vs = np.stack([b.value.scales.numpy() for b in blocks])
    valid = np.array([b.valid_tokens for b in blocks], np.int32)
    s = store.spec
    return orc.decode(q.float().numpy(), kp, vp, ks, vs, valid, s.bits, s.group_size,
                      1 / math.sqrt(s.head_dim))


@pytest.mark.parametrize("bits", [2, 4])
def test_pipeline_and_packed_attention_match_reference(tmp_path: Path, bits: int):
    g = load_npz(f"packed_attention_b{bits}.npz")
    spec = CacheSpec(1, 2, 32, block_tokens=8, bits=bits, group_size=16)
    store = KVCacheStore.create(tmp_path, torch.from_numpy(g["keys"]), torch.from_numpy(g["values"]), spec)
    q = torch.from_numpy(g["query"])
    blocks = [store.read(0, i) for i in store.blocks_for_layer(0)]
    out = packed_attention(q.to(DEV), blocks, require_cuda_kernel=True)
    torch.testing.assert_close(out.cpu(), torch.from_numpy(g["out"]), atol=2e-3, rtol=1e-2)
    with KVSSDPipeline(store, device=DEV, require_cuda_kernel=True) as pipe:
        assert pipe.attention_backend.name == "cuda"
        out2 = pipe.decode(q, 0)
    assert out2.dtype == q.dtype and out2.device.type == "cuda"
    torch.testing.assert_close(out2.cpu(), torch.from_numpy(g["out"]), atol=2e-3, rtol=1e-2)
    store.close()


@pytest.mark.parametrize("stage_blocks", [1, 4, 64])
@pytest.mark.parametrize("selector", [AllBlocks(), RecentSinkBlocks(1, 8), RecentSinkBlocks(3, 2)])
def test_pipeline_selection_and_chunking(tmp_path: Path, stage_blocks, selector):
    store = _store(tmp_path)
    q = torch.randn(32, 128, generator=torch.Generator().manual_seed(2)).half()
    with KVSSDPipeline(store, device=DEV, io_depth=3, stage_blocks=stage_blocks) as pipe:
        out = pipe.decode(q, 0, selector)
        torch.cuda.synchronize()
    selected = selector.select(store.blocks_for_layer(0))
    ref_out, _ = _oracle_for(store, q, selected)
    torch.testing.assert_close(out.float().cpu().half().float(),
                               torch.from_numpy(ref_out).half().float(), atol=2e-3, rtol=1e-2)
    assert out.dtype == torch.float16
    store.close()


def test_pipeline_detects_corrupt_record_on_device(tmp_path: Path):
    store = _store(tmp_path, tokens=200)
    q = torch.randn(32, 128, generator=torch.Generator().manual_seed(3)).half()
    entry = store.entry(0, 5)
    store.close()
    path = tmp_path / "blocks.kvssd"
    data = bytearray(path.read_bytes())
    data[entry.offset + 52 + 1000] ^= 0x10  # one payload bit: only the CRC can tell
    path.write_bytes(bytes(data))
    store = KVCacheStore.open(tmp_path)
    with KVSSDPipeline(store, device=DEV, stage_blocks=4) as pipe:
        with pytest.raises(IOError, match="CRC mismatch for layer=0, block=5"):
            pipe.decode(q, 0)
        out = pipe.decode(q, 0, RecentSinkBlocks(2, 3))  # block 5 not selected: fine
        torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    store.close()


def test_pipeline_rejects_empty_selection(tmp_path: Path):
    store = _store(tmp_path, tokens=64)
    with KVSSDPipeline(store, device=DEV) as pipe:
        with pytest.raises(ValueError, match="no blocks"):
            pipe.decode(torch.randn(32, 128).half(), 0, RecentSinkBlocks(0, 0))
    store.close()


def test_device_pool_decode_with_selectors(tmp_path: Path):
    store = _store(tmp_path, tokens=1000, bt=32, bits=2)
    pool = DeviceBlockPool.from_store(store, 0, DEV)
    q = torch.randn(32, 128, generator=torch.Generator().manual_seed(5)).half()
    for selector in (AllBlocks(), RecentSinkBlocks(1, 4), RecentSinkBlocks(2, 100)):
        out, lse = pool.decode(q, selector)
        torch.cuda.synchronize()
        ref = _oracle_for(store, q, selector.select(store.blocks_for_layer(0)))
        assert_parity(out, lse, *ref)
    with pytest.raises(KeyError):
        pool.block_table([999])
    store.close()


def test_fused_attention_tensors_and_chunk_merge():
    g = load_npz("backend_gqa4_b4_32_8_128.npz")
    from test_gpu_decode import golden_batch
    q, b = golden_batch(g)
    out, lse = fused_attention_tensors(q, b.packed_k, b.packed_v, b.scales_k, b.scales_v,
                                       b.valid_tokens, b.bits, b.group_size, float(g["sm_scale"]))
    assert_parity(out, lse, g["out"], g["lse"])
    backend = resolve_attention_backend("auto", DEV)
    assert backend.name == "cuda" and backend.probe(DEV).accelerated
    halves = []
    for sl in (slice(0, 1), slice(1, 3)):
        from kvssd_b200 import PackedBatch
        halves.append(backend.run(q, PackedBatch(b.packed_k[sl], b.packed_v[sl], b.scales_k[sl],
                                                 b.scales_v[sl], b.valid_tokens[sl], 4, 32),
                                  float(g["sm_scale"])))
    mo, ml = merge_attention_chunks(halves[0][0], halves[0][1], halves[1][0], halves[1][1])
    torch.testing.assert_close(mo, out, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(ml, lse, atol=1e-5, rtol=1e-5)


def test_pipeline_runs_a_plugged_backend(tmp_path: Path):
    # kvssd's pipeline calls the resolved backend's run per chunk; a backend registered by the
    # caller must be the one that runs (here a wrapper that counts its calls).
    from kvssd_b200 import B200AttentionBackend, register_attention_backend

    calls = []

    class Counting(B200AttentionBackend):
        name = "counting"

        def run(self, query, batch, sm_scale):
            calls.append(batch.packed_k.shape[0])
            return super().run(query, batch, sm_scale)

    register_attention_backend("counting", Counting)
    store = _store(tmp_path, tokens=600)
    q = torch.randn(32, 128, generator=torch.Generator().manual_seed(5)).half()
    with KVSSDPipeline(store, device=DEV, stage_blocks=8, attention_backend="counting") as pipe:
        assert isinstance(pipe.attention_backend, Counting)
        out = pipe.decode(q.to(DEV), 0)
    selected = store.blocks_for_layer(0)
    assert sum(calls) == len(selected) and len(calls) == -(-len(selected) // 8)
    ref_out, _ = _oracle_for(store, q, selected)
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(ref_out).half().float(),
                               atol=2e-3, rtol=1e-2)
    with pytest.raises(ValueError, match="require_cuda_kernel conflicts"):
        KVSSDPipeline(store, device=DEV, require_cuda_kernel=True, attention_backend="counting")
