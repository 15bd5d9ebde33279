"""The "mapped" storage backend: the store file mapped read-only and page-locked with the CUDA
driver (kvssd_b200_host_register), records copied to the device by DMA
(kvssd_b200_copy_records_h2d). The device bytes equal the host reads (contiguous runs and a
scattered selection), single-record reads work into both host and device tensors, and
KVSSDPipeline over a mapped store equals the default store."""

from __future__ import annotations

import pytest
import torch

from kvssd_b200 import AllBlocks, CacheSpec, KVCacheStore, KVSSDPipeline, RecentSinkBlocks, ops
from kvssd_b200.format import PackedKVBlock
from kvssd_b200.quant import QuantizedTensor
from kvssd_b200.storage import MappedStorageBackend
from kvssd_b200.workloads import WORKLOADS, make_layer

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture
def stores(tmp_path):
    w = WORKLOADS["c1"]
    lay = make_layer(w, 0, "cpu")
    spec = CacheSpec(1, w.kv_heads, w.head_dim, w.block_tokens, w.bits, w.group_size)
    shape = (w.block_tokens, w.kv_heads, w.head_dim)
    blocks = [PackedKVBlock(0, b, int(lay.valid_tokens[b]),
                            QuantizedTensor(lay.packed_k[b], lay.scales_k[b], shape, w.bits,
                                            w.group_size),
                            QuantizedTensor(lay.packed_v[b], lay.scales_v[b], shape, w.bits,
                                            w.group_size))
              for b in range(24)]
    store = KVCacheStore.from_blocks(tmp_path / "s", spec, blocks)
    state = MappedStorageBackend(store.root / "blocks.kvssd").probe()
    if not state.available:
        store.close()
        pytest.skip(f"mapped backend unavailable: {state.reason}")
    mapped = KVCacheStore.open(store.root, storage_backend="mapped")
    yield store, mapped, lay
    mapped.close()
    store.close()


def test_mapped_device_reads_equal_host_reads(stores):
    store, mapped, lay = stores
    assert mapped.reads_to_device
    ids = store.blocks_for_layer(0)
    rb = store.spec.record_bytes
    host = store.read_records(0, ids)
    buf = torch.empty(len(ids) * rb, dtype=torch.uint8, device=DEV)
    for sel in (ids, ids[::-3], [5, 6, 7, 1, 2, 20]):  # runs, scattered, mixed
        dev = mapped.read_records(0, sel, destination=buf)
        torch.cuda.synchronize()
        assert torch.equal(dev.cpu(), host[torch.tensor(sel)])
    out = ops.decode_records(mapped.read_records(0, ids, destination=buf), store.spec, 0,
                             torch.tensor(ids))
    torch.cuda.synchronize()
    assert int(out[5].abs().sum()) == 0 and torch.equal(out[0].cpu(), lay.packed_k[:24])
    one = torch.empty(rb, dtype=torch.uint8, device=DEV)
    mapped.read_into(mapped.entry(0, 9), one)
    cpu = torch.empty(rb, dtype=torch.uint8)
    mapped.read_into(mapped.entry(0, 9), cpu)
    torch.cuda.synchronize()
    assert torch.equal(one.cpu(), host[9]) and torch.equal(cpu, host[9])
    assert mapped.read(0, 4).valid_tokens == store.read(0, 4).valid_tokens


@pytest.mark.parametrize("selector", [AllBlocks(), RecentSinkBlocks(1, 5)])
def test_pipeline_over_a_mapped_store_equals_the_default_store(stores, selector):
    store, mapped, lay = stores
    q = lay.query.to(DEV).float()
    with KVSSDPipeline(store, device=DEV, stage_blocks=7) as pipe:
        ref = pipe.decode(q, 0, selector)
    with KVSSDPipeline(mapped, device=DEV, stage_blocks=7) as pipe:
        for _ in range(2):  # the second call reuses the device ring behind its events
            got = pipe.decode(q, 0, selector)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
