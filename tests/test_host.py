"""Host-side logic of kvssd_b200 against the reference's golden outputs (no GPU needed):
quantizer bits, record format bytes, store layout, selectors, validation and registry."""

from __future__ import annotations

import shutil
from pathlib import Path

import numpy as np
import pytest
import torch
from conftest import GOLDEN, f16, golden_names, load_json, load_npz

from kvssd_b200 import (
    AllBlocks,
    CacheSpec,
    KVCacheStore,
    PackedBatch,
    RecentSinkBlocks,
    available_attention_backends,
    dequantize_tensor,
    quantize_tensor,
    resolve_attention_backend,
)
from kvssd_b200.backends import register_attention_backend
from kvssd_b200.format import ALIGNMENT, HEADER, decode_record
from kvssd_b200.loader import AsyncBlockLoader
from kvssd_b200.quant import pack_codes, unpack_codes
from kvssd_b200.workloads import WORKLOADS, make_layer


@pytest.mark.parametrize("name", golden_names("quant_"))
def test_quantizer_is_bit_identical_to_reference(name):
    g = load_npz(name)
    bits = int(name.split("_b")[1][0])
    group = int(name.split("_g")[1].split(".")[0])
    for tag, dtype in (("f32", torch.float32), ("f16", torch.float16)):
        x = torch.from_numpy(g[f"x_{tag}"]).to(dtype)
        q = quantize_tensor(x, bits, group)
        np.testing.assert_array_equal(q.packed.numpy(), g[f"packed_{tag}"])
        np.testing.assert_array_equal(q.scales.view(torch.int16).numpy().view(np.uint16),
                                      g[f"scales_{tag}"])
        np.testing.assert_array_equal(unpack_codes(q.packed, bits, 128).numpy(), g[f"codes_{tag}"])
        np.testing.assert_array_equal(pack_codes(torch.from_numpy(g[f"codes_{tag}"]), bits).numpy(),
                                      g[f"packed_{tag}"])
        np.testing.assert_array_equal(dequantize_tensor(q).numpy(), g[f"deq32_{tag}"])
        d16 = dequantize_tensor(q, torch.float16).view(torch.int16).numpy().view(np.uint16)
        np.testing.assert_array_equal(d16, g[f"deq16_{tag}"])


def test_quantizer_refusals_match_reference():
    with pytest.raises(ValueError, match="divisible"):
        quantize_tensor(torch.randn(2, 31), 4, group_size=16)
    with pytest.raises(ValueError, match="bits"):
        quantize_tensor(torch.randn(2, 32), 3, group_size=16)
    with pytest.raises(ValueError, match="pack-aligned"):
        quantize_tensor(torch.randn(2, 30), 2, group_size=6)
    with pytest.raises(TypeError):
        quantize_tensor(torch.ones(2, 32, dtype=torch.int32), 4, group_size=16)


def test_cachespec_geometry_matches_reference():
    for row in load_json("cachespec.json"):
        s = CacheSpec(*row["spec"])
        for key in ("packed_dim", "scale_count", "packed_count", "payload_bytes", "record_bytes"):
            assert getattr(s, key) == row[key], key
    with pytest.raises(ValueError):
        CacheSpec(1, 2, 30, group_size=16).validate()
    with pytest.raises(ValueError):
        CacheSpec(1, 2, 32, bits=3).validate()


def test_store_bytes_identical_to_reference(tmp_path: Path):
    g = load_npz("store_small_inputs.npz")
    spec = CacheSpec(2, 2, 32, block_tokens=8, bits=4, group_size=16)
    store = KVCacheStore.create(tmp_path, torch.from_numpy(g["keys"]), torch.from_numpy(g["values"]), spec)
    ref = (GOLDEN / "store_small" / "blocks.kvssd").read_bytes()
    assert (tmp_path / "blocks.kvssd").read_bytes() == ref
    assert (tmp_path / "manifest.json").read_text() == (GOLDEN / "store_small" / "manifest.json").read_text()
    assert all(e.offset % ALIGNMENT == 0 for e in store.manifest.entries)
    block = store.read(1, 2)
    assert block.valid_tokens == 3
    assert torch.count_nonzero(dequantize_tensor(block.key)[3:]) == 0
    store.close()


def test_reads_reference_written_store(tmp_path: Path):
    shutil.copytree(GOLDEN / "store_small", tmp_path / "s")
    store = KVCacheStore.open(tmp_path / "s")
    assert store.blocks_for_layer(0) == [0, 1, 2] and store.blocks_for_layer(1) == [0, 1, 2]
    b = store.read(0, 2)
    raw = (tmp_path / "s" / "blocks.kvssd").read_bytes()
    e = store.entry(0, 2)
    fields = HEADER.unpack(raw[e.offset : e.offset + HEADER.size])
    assert fields[0] == b"KVSSD001" and fields[4] == b.valid_tokens == 3
    with pytest.raises(KeyError):
        store.entry(0, 9)
    store.close()


def test_crc_detects_corruption(tmp_path: Path):
    shutil.copytree(GOLDEN / "store_small", tmp_path / "s")
    store = KVCacheStore.open(tmp_path / "s")
    entry = store.entry(0, 0)
    with (tmp_path / "s" / "blocks.kvssd").open("r+b") as f:
        f.seek(entry.offset + 80)
        old = f.read(1)
        f.seek(entry.offset + 80)
        f.write(bytes([old[0] ^ 0xFF]))
    with pytest.raises(IOError, match="CRC"):
        store.read(0, 0)
    store.read(0, 0, verify_crc=False)
    store.close()


def test_record_layout_mismatch_rejected(tmp_path: Path):
    shutil.copytree(GOLDEN / "store_small", tmp_path / "s")
    store = KVCacheStore.open(tmp_path / "s")
    raw = torch.empty(store.entry(0, 0).length, dtype=torch.uint8)
    store.read_into(store.entry(0, 0), raw)
    with pytest.raises(ValueError, match="does not match"):
        decode_record(raw, CacheSpec(2, 2, 32, block_tokens=8, bits=2, group_size=16))
    store.close()


def test_loader_slots_do_not_alias(tmp_path: Path):
    shutil.copytree(GOLDEN / "store_small", tmp_path / "s")
    store = KVCacheStore.open(tmp_path / "s")
    with AsyncBlockLoader(store, depth=2, pinned=False) as loader:
        blocks = list(loader.iter_blocks(0, [0, 1, 2]))
    assert [b.block for b in blocks] == [0, 1, 2]
    for b in blocks:
        ref = store.read(0, b.block)
        assert torch.equal(b.key.packed, ref.key.packed)
        assert torch.equal(b.value.scales, ref.value.scales)
    with AsyncBlockLoader(store, depth=3, pinned=False) as loader:
        it = loader.iter_records(0, [0, 1, 2])
        next(it)
        it.close()  # early stop drains in-flight reads and recycles their slots
        assert loader.free.qsize() == 3
    store.close()


def test_selectors_match_reference():
    for case in load_json("selectors.json"):
        assert RecentSinkBlocks(case["sink"], case["recent"]).select(case["available"]) == case["chosen"]
    assert AllBlocks().select([3, 1, 2]) == [3, 1, 2]
    with pytest.raises(ValueError):
        RecentSinkBlocks(-1, 2).select([1])


def _batch(qh=4, kvh=2, d=32, bits=4, group=16):
    k = quantize_tensor(torch.randn(2, 8, kvh, d), bits, group)
    v = quantize_tensor(torch.randn(2, 8, kvh, d), bits, group)
    return torch.randn(qh, d), PackedBatch(k.packed, v.packed, k.scales, v.scales,
                                           torch.tensor([8, 5], dtype=torch.int32), bits, group)


def test_packed_batch_validation_messages():
    q, b = _batch()
    b.validate(q)
    with pytest.raises(ValueError, match="query must be"):
        b.validate(q[0])
    with pytest.raises(ValueError, match="divisible by KV heads"):
        b.validate(torch.randn(3, 32))
    with pytest.raises(ValueError, match="packed dimension"):
        b.validate(torch.randn(4, 64))
    bad = PackedBatch(b.packed_k, b.packed_v, b.scales_k, b.scales_v, b.valid_tokens[:1], 4, 16)
    with pytest.raises(ValueError, match="one count per block"):
        bad.validate(q)
    bad = PackedBatch(b.packed_k, b.packed_v[:1], b.scales_k, b.scales_v, b.valid_tokens, 4, 16)
    with pytest.raises(ValueError, match="packed KV must match"):
        bad.validate(q)
    bad = PackedBatch(b.packed_k, b.packed_v, b.scales_k, b.scales_v, b.valid_tokens, 3, 16)
    with pytest.raises(ValueError, match="bits"):
        bad.validate(q)


def test_registry_fails_closed_on_cpu():
    with pytest.raises(RuntimeError, match="CUDA extension requires"):
        resolve_attention_backend("cuda", "cpu")
    with pytest.raises(RuntimeError, match="no attention backend is available"):
        resolve_attention_backend("auto", "cpu")
    with pytest.raises(ValueError, match="unknown attention backend"):
        resolve_attention_backend("imaginary", "cpu")
    names = {a.name for a in available_attention_backends("cpu")}
    assert "cuda" in names
    cuda = next(a for a in available_attention_backends("cpu") if a.name == "cuda")
    assert not cuda.available and cuda.accelerated
    with pytest.raises(ValueError):
        register_attention_backend("auto", object)


def test_registry_accepts_plugged_backend_instance():
    class Fake:
        name = "fake"

        def probe(self, device):
            from kvssd_b200.backends import BackendAvailability
            return BackendAvailability("fake", True, False, False, "test double", "cpu")

        def run(self, query, batch, sm_scale):
            raise AssertionError

    fake = Fake()
    assert resolve_attention_backend(fake, "cpu") is fake


def test_pipeline_refuses_cpu_device(tmp_path: Path):
    from kvssd_b200 import KVSSDPipeline
    shutil.copytree(GOLDEN / "store_small", tmp_path / "s")
    store = KVCacheStore.open(tmp_path / "s")
    with pytest.raises(RuntimeError):
        KVSSDPipeline(store, device="cpu")
    with pytest.raises(ValueError, match="conflicts"):
        KVSSDPipeline(store, device="cpu", require_cuda_kernel=True, attention_backend="triton")
    store.close()


def test_workload_c1_matches_reference_quantized_inputs():
    """The seeded C1 generator + this package's quantizer reproduce the reference's bytes."""
    import hashlib
    g = load_npz("config_c1.npz")
    layer = make_layer(WORKLOADS["c1"], 0, "cpu")
    sha = lambda t: hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()  # noqa: E731
    assert sha(layer.packed_k) == str(g["sha_packed_k"])
    assert sha(layer.packed_v) == str(g["sha_packed_v"])
    assert sha(layer.scales_k) == str(g["sha_scales_k"])
    assert sha(layer.scales_v) == str(g["sha_scales_v"])
    np.testing.assert_array_equal(layer.query.view(torch.int16).numpy().view(np.uint16), g["query"])


def test_workload_geometry():
    w = WORKLOADS["c2"]
    assert w.blocks_per_layer == 1024 and w.bytes_per_block == 147456
    assert w.bytes_per_block * w.blocks_per_layer == 150994944
    c3 = WORKLOADS["c3"]
    assert c3.selected_blocks() == [0, *range(992, 1024)]
    assert c3.bytes_per_block * len(c3.selected_blocks()) == 2703360
    assert WORKLOADS["c5"].bytes_per_block * WORKLOADS["c5"].blocks_per_layer == 1207959552
    assert f16(np.array([0x3C00], np.uint16))[0] == 1.0


def test_native_record_reader_matches_pread(tmp_path: Path):
    shutil.copytree(GOLDEN / "store_small", tmp_path / "s")
    store = KVCacheStore.open(tmp_path / "s")
    for layer in range(store.spec.layers):
        ids = store.blocks_for_layer(layer)
        for direct in (True, False):
            raw = store.read_records(layer, list(reversed(ids)), threads=3, direct=direct)
            for i, b in enumerate(reversed(ids)):
                ref = torch.empty(store.spec.record_bytes, dtype=torch.uint8)
                store.read_into(store.entry(layer, b), ref)
                assert torch.equal(raw[i], ref)
    # a record past the end of the file is an error, not a short buffer
    entry = store.entry(0, store.blocks_for_layer(0)[-1])
    (tmp_path / "s" / "blocks.kvssd").write_bytes(
        (tmp_path / "s" / "blocks.kvssd").read_bytes()[: entry.offset + 100])
    store2 = KVCacheStore.open(tmp_path / "s")
    with pytest.raises(OSError, match="short read"):
        store2.read_records(0, [store.blocks_for_layer(0)[-1]])


PREAD_SHIM = r"""
#define _GNU_SOURCE
#include <dlfcn.h>
#include <errno.h>
#include <fcntl.h>
#include <sys/types.h>

/* pread that refuses every read of a descriptor opened with O_DIRECT, as a file system that
   accepts the O_DIRECT open but not its reads does */
static ssize_t refuse(int fd, void* buf, size_t n, off_t off, const char* name) {
  typedef ssize_t (*fn)(int, void*, size_t, off_t);
  fn real = (fn)dlsym(RTLD_NEXT, name);
  int fl = fcntl(fd, F_GETFL);
  if (fl >= 0 && (fl & O_DIRECT)) { errno = EINVAL; return -1; }
  return real(fd, buf, n, off);
}
ssize_t pread(int fd, void* buf, size_t n, off_t off) { return refuse(fd, buf, n, off, "pread"); }
ssize_t pread64(int fd, void* buf, size_t n, off_t off) {
  return refuse(fd, buf, n, off, "pread64");
}
"""

READER_CHILD = r"""
import ctypes, mmap, sys
from kvssd_b200 import _native
path, n = sys.argv[1], 6
lib = _native.library()
buf = mmap.mmap(-1, n * 4096)  # page aligned, as O_DIRECT wants
addr = ctypes.addressof(ctypes.c_char.from_buffer(buf))
offsets = (ctypes.c_longlong * n)(*[4096 * (n - 1 - i) for i in range(n)])  # reversed
used = ctypes.c_int(-1)
st = lib.kvssd_b200_read_records(path.encode(), offsets, n, 4096, addr, 3, 1, ctypes.byref(used))
ok = st == 0 and all(buf[i * 4096:(i + 1) * 4096] == bytes([n - 1 - i]) * 4096 for i in range(n))
print(st, used.value, int(ok), lib.kvssd_b200_io_last_error().decode())
"""


def test_native_reader_falls_back_when_direct_reads_are_refused(tmp_path: Path):
    """Where the O_DIRECT open succeeds but its reads fail with EINVAL, the native reader reads
    the batch again with buffered preads (the store's default backend is ``buffered``, which
    must not fail where kvssd's positioned reads succeed). The refusal comes from a preloaded
    fake of pread in a child process."""
    import os
    import subprocess
    import sys

    data = tmp_path / "records.bin"
    data.write_bytes(b"".join(bytes([i]) * 4096 for i in range(6)))
    try:
        os.close(os.open(data, os.O_RDONLY | os.O_DIRECT))
    except OSError:
        pytest.skip("this file system refuses O_DIRECT opens; the fallback is not reached")
    shim_src = tmp_path / "shim.c"
    shim_src.write_text(PREAD_SHIM)
    shim = tmp_path / "shim.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", str(shim_src), "-o", str(shim), "-ldl"],
                   check=True)
    package = str(Path(__file__).resolve().parents[1] / "kvssd-attention_b200")
    env = {**os.environ, "PYTHONPATH": package + os.pathsep + os.environ.get("PYTHONPATH", "")}

    def child(preload: bool) -> list[str]:
        run_env = {**env, "LD_PRELOAD": str(shim)} if preload else env
        done = subprocess.run([sys.executable, "-c", READER_CHILD, str(data)], env=run_env,
                              capture_output=True, text=True, timeout=120)
        assert done.returncode == 0, done.stderr
        return done.stdout.strip().split(" ", 3)

    st, used, ok, *_ = child(preload=False)
    assert (st, used, ok) == ("0", "1", "1")  # O_DIRECT reads where the file system allows
    st, used, ok, *_ = child(preload=True)
    assert (st, used, ok) == ("0", "0", "1")  # refused, then read buffered


def test_registered_attention_backend_takes_part_in_auto(monkeypatch):
    """Every registered attention backend is open to ``auto``, in registration order after the
    ``cuda`` kernels: on a CPU device a CPU backend the caller registered is the one chosen."""
    from kvssd_b200.backends import BackendAvailability, registry

    table = registry.FactoryTable("attention")
    for name, (factory, auto) in registry._table._entries.items():
        table.add(name, factory, auto=auto)
    monkeypatch.setattr(registry, "_table", table)

    class CpuOnly:
        name = "cpu-only"

        def probe(self, device):
            ok = torch.device(device).type == "cpu"
            return BackendAvailability(self.name, ok, False, False, "test double",
                                       torch.device(device).type)

        def run(self, query, batch, sm_scale):
            raise AssertionError

    register_attention_backend("cpu-only", CpuOnly)
    assert isinstance(resolve_attention_backend("auto", "cpu"), CpuOnly)
    assert [a.name for a in available_attention_backends("cpu")] == ["cuda", "cpu-only"]
    with pytest.raises(ValueError, match="choose one of: auto, cuda, cpu-only"):
        resolve_attention_backend("triton", "cpu")
