"""Storage backend selection with kvssd's storage API (src/kvssd/storage/registry.py:15-68):
names, ``auto`` order, refusals, and the cuFile (gds) backend's probe reporting why it is
unavailable on a host without a CUDA device. The gds read path itself is tested on the GPU
(tests/test_gpu_gds.py)."""

from __future__ import annotations

import pytest
import torch

from kvssd_b200 import (CacheSpec, GDSStorageBackend, KVCacheStore, available_storage_backends,
                        resolve_storage_backend)
from kvssd_b200.format import PackedKVBlock
from kvssd_b200.quant import quantize_tensor
from kvssd_b200.storage import BufferedStorageBackend


def _store(tmp_path, **kw):
    spec = CacheSpec(layers=1, kv_heads=2, head_dim=64, block_tokens=16, bits=4, group_size=32)
    gen = torch.Generator().manual_seed(3)
    blocks = []
    for b in range(3):
        x = torch.randn(2, 16, 2, 64, generator=gen).half()
        blocks.append(PackedKVBlock(0, b, 16, quantize_tensor(x[0], 4, 32),
                                    quantize_tensor(x[1], 4, 32)))
    return KVCacheStore.from_blocks(tmp_path / "s", spec, blocks, **kw)


def test_default_store_reads_with_positioned_reads(tmp_path):
    store = _store(tmp_path)
    assert isinstance(store.storage_backend, BufferedStorageBackend)
    assert not store.reads_to_device
    blk = store.read(0, 1)
    assert blk.valid_tokens == 16
    store.close()


def test_unknown_and_unavailable_backends_are_refused(tmp_path):
    store = _store(tmp_path)
    path = store.root / "blocks.kvssd"
    with pytest.raises(ValueError, match="unknown storage backend 'nvme'"):
        resolve_storage_backend("nvme", path)
    if not torch.cuda.is_available():
        state = GDSStorageBackend(path).probe()
        assert not state.available and "CUDA" in state.reason
        with pytest.raises(RuntimeError, match="storage backend 'gds' unavailable"):
            KVCacheStore.open(store.root, storage_backend="gds")
    names = [s.name for s in available_storage_backends(path)]
    assert names[:3] == ["gds", "direct", "buffered"]
    auto = resolve_storage_backend("auto", path)  # gds, else direct, else buffered
    assert auto.probe().available
    assert resolve_storage_backend(None, path).name in ("gds", "direct", "buffered")
    missing = tmp_path / "nothing.kvssd"
    assert not BufferedStorageBackend(missing).probe().available
    store.close()


def test_mapped_backend_and_record_copy_refusals_without_a_gpu(tmp_path):
    """The mapped backend reports why it is unavailable, and the C ABI refuses out-of-range
    record copies before it touches CUDA (no device is needed for either)."""
    import ctypes

    from kvssd_b200 import _native
    from kvssd_b200.storage import MappedStorageBackend

    store = _store(tmp_path)
    path = store.root / "blocks.kvssd"
    if not torch.cuda.is_available():
        state = MappedStorageBackend(path).probe()
        assert not state.available and "CUDA" in state.reason
    assert "mapped" in [s.name for s in available_storage_backends(path)]
    assert resolve_storage_backend("auto", path).name != "mapped"  # opt-in only
    lib = _native.library()
    host = (ctypes.c_uint8 * 8192)()
    offsets = (ctypes.c_longlong * 2)(0, 8192)  # the second record runs past the range
    st = lib.kvssd_b200_copy_records_h2d(ctypes.addressof(host), 8192, offsets, 2, 4096,
                                         ctypes.addressof(host), None)
    assert st == _native.ERR_INVALID_ARGUMENT
    assert "outside the mapped range" in lib.kvssd_b200_host_last_error().decode()
    wrap = (ctypes.c_longlong * 1)(4096)  # offset + record_bytes wraps around 2^64
    st = lib.kvssd_b200_copy_records_h2d(ctypes.addressof(host), 8192, wrap, 1, 2**64 - 4096,
                                         ctypes.addressof(host), None)
    assert st == _native.ERR_INVALID_ARGUMENT
    assert "outside the mapped range" in lib.kvssd_b200_host_last_error().decode()
    assert lib.kvssd_b200_host_register(None, 0, 1) == _native.ERR_INVALID_ARGUMENT
    store.close()


def test_backend_probes_are_closed_again(tmp_path, monkeypatch):
    """available_storage_backends and ``auto`` close every instance they probe and drop (a gds
    probe holds a cuFile handle and an O_DIRECT descriptor until closed)."""
    from kvssd_b200 import storage

    closed = []

    class Counting(BufferedStorageBackend):
        def close(self) -> None:
            closed.append(self.name)
            super().close()

    class Unavailable(Counting):
        name = "gds"

        def probe(self):
            return storage.StorageAvailability(self.name, False, True, True, "test stand-in")

    store = _store(tmp_path)
    path = store.root / "blocks.kvssd"
    table = storage.FactoryTable("storage")
    for name, factory in (("gds", Unavailable), ("direct", Counting), ("buffered", Counting)):
        table.add(name, factory, auto=True)
    monkeypatch.setattr(storage, "_table", table)
    states = available_storage_backends(path)
    assert [s.available for s in states] == [False, True, True]
    assert closed == ["gds", "buffered", "buffered"]  # Counting's name is "buffered"
    closed.clear()
    chosen = resolve_storage_backend("auto", path)
    assert closed == ["gds"] and chosen.probe().available  # the chosen one stays open
    chosen.close()
    store.close()


def test_registered_storage_backends_and_auto(tmp_path, monkeypatch):
    """As in kvssd, ``auto`` considers only gds, direct and buffered: a factory registered under
    one of those names replaces that step, one under a new name is chosen only by name. A
    backend that is built, found unavailable and not returned is closed."""
    from kvssd_b200 import register_storage_backend, storage

    table = storage.FactoryTable("storage")
    for name, factory in storage._table._entries.items():
        table.add(name, factory[0], auto=factory[1])
    monkeypatch.setattr(storage, "_table", table)
    store = _store(tmp_path)
    path = store.root / "blocks.kvssd"
    closed = []

    class Mine(BufferedStorageBackend):
        name = "mine"

        def close(self) -> None:
            closed.append(self.name)
            super().close()

    class Refused(Mine):
        name = "refused"

        def probe(self):
            return storage.StorageAvailability(self.name, False, False, False, "not today")

    register_storage_backend(" Mine ", Mine)
    assert resolve_storage_backend("auto", path).name in ("gds", "direct", "buffered")
    assert isinstance(resolve_storage_backend("MINE", path), Mine)
    register_storage_backend("refused", Refused)
    with pytest.raises(RuntimeError, match="storage backend 'refused' unavailable: not today"):
        resolve_storage_backend("refused", path)
    assert closed == ["refused"]
    for name in ("gds", "direct"):
        register_storage_backend(name, Refused)  # both steps of auto now refuse
    register_storage_backend("buffered", Mine)
    assert isinstance(resolve_storage_backend(None, path), Mine)
    assert closed == ["refused", "refused", "refused"]
    assert table.names()[:4] == ["gds", "direct", "buffered", "mapped"]  # places kept
    with pytest.raises(ValueError, match="cannot be 'auto'"):
        register_storage_backend("Auto", Mine)
    with pytest.raises(ValueError, match="choose one of: auto, gds, direct, buffered, mapped, mine"):
        resolve_storage_backend("nvme", path)
    store.close()


def test_builtin_backends_satisfy_the_storage_interface(tmp_path):
    """Every registered backend has kvssd's StorageBackend interface
    (src/kvssd/storage/base.py:21-39), and the package exports it under kvssd's name."""
    from kvssd_b200 import StorageBackend, storage

    path = tmp_path / "blocks.kvssd"
    for key in storage._table.names():
        backend = storage._table.factory(key)(path)
        assert isinstance(backend, StorageBackend), key
        backend.close()
