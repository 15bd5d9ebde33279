"""cuFile (GPUDirect Storage) record reads into device memory (kvssd_b200_gds_*, the ``gds``
storage backend): the bytes equal the host reads, the on-GPU record decode of them equals the
CPU decode, and KVSSDPipeline over a gds store equals the default store. Skipped, with the
probe's reason, where cuFile cannot open the store file (no libcufile driver, or a file system
without O_DIRECT)."""

from __future__ import annotations

import shutil
from pathlib import Path

import pytest
import torch

from kvssd_b200 import AllBlocks, GDSStorageBackend, KVCacheStore, KVSSDPipeline, ops
from kvssd_b200.format import PackedKVBlock
from kvssd_b200.quant import QuantizedTensor
from kvssd_b200.workloads import WORKLOADS, make_layer

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture
def gds_store(tmp_path):
    store, lay, w, extra = _gds_store(tmp_path)
    yield store, lay, w
    store.close()
    if extra is not None:
        shutil.rmtree(extra, ignore_errors=True)


def _gds_store(tmp_path):
    w = WORKLOADS["c1"]
    lay = make_layer(w, 0, "cpu")
    from kvssd_b200 import CacheSpec

    spec = CacheSpec(1, w.kv_heads, w.head_dim, w.block_tokens, w.bits, w.group_size)
    shape = (w.block_tokens, w.kv_heads, w.head_dim)
    blocks = [PackedKVBlock(0, b, int(lay.valid_tokens[b]),
                            QuantizedTensor(lay.packed_k[b], lay.scales_k[b], shape, w.bits,
                                            w.group_size),
                            QuantizedTensor(lay.packed_v[b], lay.scales_v[b], shape, w.bits,
                                            w.group_size))
              for b in range(16)]
    reasons = []
    # tmpfs refuses O_DIRECT: try the test's directory, then one on the working directory's
    # file system (removed afterwards)
    for root in (tmp_path, Path.cwd() / ".gds_test_store"):
        store = KVCacheStore.from_blocks(root / "s", spec, blocks)
        state = GDSStorageBackend(store.root / "blocks.kvssd").probe()
        if state.available:
            return store, lay, w, (root if root != tmp_path else None)
        reasons.append(f"{root}: {state.reason}")
        store.close()
        if root != tmp_path:
            shutil.rmtree(root, ignore_errors=True)
    pytest.skip("cuFile unavailable: " + "; ".join(reasons))


def test_gds_reads_equal_host_reads_and_decode_on_device(gds_store):
    store, lay, w = gds_store
    gstore = KVCacheStore.open(store.root, storage_backend="gds")
    assert gstore.reads_to_device
    ids = gstore.blocks_for_layer(0)
    rb = gstore.spec.record_bytes
    host = store.read_records(0, ids)
    dev_buf = gstore.storage_backend.allocate_buffer(len(ids) * rb, device=DEV)
    dev = gstore.read_records(0, ids, destination=dev_buf)
    torch.cuda.synchronize()
    assert torch.equal(dev.cpu(), host)
    out = ops.decode_records(dev, gstore.spec, 0, torch.tensor(ids))
    torch.cuda.synchronize()
    assert int(out[5].abs().sum()) == 0
    assert torch.equal(out[0].cpu(), lay.packed_k[: len(ids)])
    # one record through read_into, as kvssd's backend does
    one = gstore.storage_backend.allocate_buffer(rb, device=DEV)
    gstore.read_into(gstore.entry(0, ids[3]), one)
    torch.cuda.synchronize()
    assert torch.equal(one.cpu(), host[3])
    gstore.close()


def test_pipeline_over_a_gds_store_equals_the_default_store(gds_store):
    store, lay, w = gds_store
    q = lay.query.to(DEV)
    with KVSSDPipeline(store, device=DEV, stage_blocks=5) as pipe:
        ref = pipe.decode(q.float(), 0, AllBlocks())
    gstore = KVCacheStore.open(store.root, storage_backend="gds")
    with KVSSDPipeline(gstore, device=DEV, stage_blocks=5) as pipe:
        got = pipe.decode(q.float(), 0, AllBlocks())
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    gstore.close()
