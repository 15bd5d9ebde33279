"""On-GPU record decode (kvssd_b200_decode_records): raw kvssd records -> PackedBatch tensors
with header checks and the payload CRC-32 computed on the device, against the CPU
decode_record of the records the reference itself wrote (tests/golden/store_small), against
records encoded for a matrix of geometries (zlib CRC on the CPU), and with corruptions planted
in the input bytes on the CPU."""

from __future__ import annotations

import shutil

import pytest
import torch
from conftest import GOLDEN

from kvssd_b200 import CacheSpec, DeviceBlockPool, KVCacheStore, ops
from kvssd_b200.format import HEADER, PackedKVBlock, decode_record, encode_record
from kvssd_b200.quant import quantize_tensor

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _raw_layer(store, layer):
    ids = store.blocks_for_layer(layer)
    raw = torch.empty((len(ids), store.spec.record_bytes), dtype=torch.uint8)
    for i, b in enumerate(ids):
        store.read_into(store.entry(layer, b), raw[i])
    return ids, raw


def _check_against_cpu(raw, spec, dev_out):
    kp, vp, ks, vs, valid, status = [t.cpu() for t in dev_out]
    for i in range(raw.shape[0]):
        blk = decode_record(raw[i].clone(), spec)
        assert torch.equal(kp[i], blk.key.packed) and torch.equal(vp[i], blk.value.packed)
        assert torch.equal(ks[i].view(torch.int16), blk.key.scales.view(torch.int16))
        assert torch.equal(vs[i].view(torch.int16), blk.value.scales.view(torch.int16))
        assert int(valid[i]) == blk.valid_tokens
    assert torch.count_nonzero(status) == 0


def test_reference_written_records_decode_bit_exact():
    store = KVCacheStore.open(GOLDEN / "store_small")
    for layer in range(store.spec.layers):
        ids, raw = _raw_layer(store, layer)
        out = ops.decode_records(raw.to(DEV), store.spec, layer, torch.tensor(ids))
        torch.cuda.synchronize()
        _check_against_cpu(raw, store.spec, out)


@pytest.mark.parametrize("bits,bt,kvh,d,group", [
    (4, 128, 8, 128, 32), (2, 128, 8, 128, 32), (4, 40, 4, 128, 16), (2, 16, 1, 64, 32),
    (4, 1, 1, 32, 32), (4, 128, 2, 256, 128), (2, 7, 3, 96, 32)])
def test_encoded_records_of_many_geometries(bits, bt, kvh, d, group):
    spec = CacheSpec(layers=1, kv_heads=kvh, head_dim=d, block_tokens=bt, bits=bits,
                     group_size=group)
    gen = torch.Generator().manual_seed(bits * 1000 + bt * 10 + kvh)
    records = []
    for b in range(3):
        x = torch.randn(2, bt, kvh, d, generator=gen).half()
        kq, vq = quantize_tensor(x[0], bits, group), quantize_tensor(x[1], bits, group)
        rec, _ = encode_record(PackedKVBlock(0, b, max(1, bt - b), kq, vq), spec)
        records.append(torch.frombuffer(bytearray(rec), dtype=torch.uint8))
    raw = torch.stack(records)
    out = ops.decode_records(raw.to(DEV), spec, 0, torch.arange(3))
    torch.cuda.synchronize()
    _check_against_cpu(raw, spec, out)


def test_planted_corruptions_are_reported_per_record():
    store = KVCacheStore.open(GOLDEN / "store_small")
    ids0, raw0 = _raw_layer(store, 0)
    ids1, raw1 = _raw_layer(store, 1)
    ids, raw = ids0 + ids1, torch.cat([raw0, raw1])
    assert raw.shape[0] >= 4
    bad = raw.clone()
    bad[0, HEADER.size + 100] ^= 0x40          # payload bit flip -> CRC
    bad[1, 0] = ord("X")                        # magic
    bad[2, 16:20] = torch.tensor([9, 0, 0, 0], dtype=torch.uint8)  # block id field
    out = ops.decode_records(bad.to(DEV), store.spec, None, torch.tensor(ids))
    status = out[5].cpu().tolist()
    assert status[0] == ops.RECORD_BAD_CRC
    assert status[1] & ops.RECORD_BAD_HEADER
    assert status[2] & ops.RECORD_BAD_ID
    assert all(s == 0 for s in status[3:])
    # geometry that does not match the records
    other = CacheSpec(layers=store.spec.layers, kv_heads=store.spec.kv_heads,
                      head_dim=store.spec.head_dim, block_tokens=store.spec.block_tokens,
                      bits=6 - store.spec.bits, group_size=store.spec.group_size)
    raw_other = raw[:, : other.record_bytes] if other.record_bytes <= raw.shape[1] else None
    if raw_other is not None:
        st = ops.decode_records(raw_other.contiguous().to(DEV), other, 0)[5].cpu()
        assert torch.all(st & (ops.RECORD_BAD_GEOMETRY | ops.RECORD_BAD_LENGTH) != 0)


def test_pool_from_store_checks_crc_on_device(tmp_path):
    shutil.copytree(GOLDEN / "store_small", tmp_path / "s")
    store = KVCacheStore.open(tmp_path / "s")
    pool = DeviceBlockPool.from_store(store, 0, DEV)
    ids = store.blocks_for_layer(0)
    ref = [store.read(0, b) for b in ids]
    assert torch.equal(pool.packed_k.cpu(), torch.stack([r.key.packed for r in ref]))
    entry = store.entry(0, ids[1])
    store.close()
    path = tmp_path / "s" / "blocks.kvssd"
    data = bytearray(path.read_bytes())
    data[entry.offset + HEADER.size + 7] ^= 0x01
    path.write_bytes(bytes(data))
    store = KVCacheStore.open(tmp_path / "s")
    with pytest.raises(IOError, match="CRC mismatch"):
        DeviceBlockPool.from_store(store, 0, DEV)
    DeviceBlockPool.from_store(store, 0, DEV, verify_crc=False)


def _encoded(spec, n, seed):
    gen = torch.Generator().manual_seed(seed)
    shape = (spec.block_tokens, spec.kv_heads, spec.head_dim)
    records = []
    for b in range(n):
        x = torch.randn(2, *shape, generator=gen).half()
        kq = quantize_tensor(x[0], spec.bits, spec.group_size)
        vq = quantize_tensor(x[1], spec.bits, spec.group_size)
        rec, _ = encode_record(PackedKVBlock(0, b, spec.block_tokens - b % 5, kq, vq), spec)
        records.append(torch.frombuffer(bytearray(rec), dtype=torch.uint8))
    return torch.stack(records)


@pytest.mark.parametrize("n", [1, 2, 37])
def test_streaming_decode_runs_across_records(n):
    """The c2 record geometry (289 rows of 512 bytes per record, 3 rows per chunk): one record
    is split over many warps, 37 records give runs that end mid-record and cross records."""
    spec = CacheSpec(layers=1, kv_heads=8, head_dim=128, block_tokens=128, bits=4, group_size=32)
    raw = _encoded(spec, n, 100 + n)
    out = ops.decode_records(raw.to(DEV), spec, 0, torch.arange(n))
    torch.cuda.synchronize()
    _check_against_cpu(raw, spec, out)


def test_streaming_decode_flags_corruption_at_the_payload_edges():
    spec = CacheSpec(layers=1, kv_heads=8, head_dim=128, block_tokens=128, bits=4, group_size=32)
    raw = _encoded(spec, 9, 7)
    scales, codes = 128 * 8 * 4 * 2, 128 * 8 * 64       # bytes per section
    end = HEADER.size + 2 * scales + 2 * codes            # header + payload
    bad = raw.clone()
    bad[0, HEADER.size] ^= 0x01             # first payload byte
    bad[1, end - 1] ^= 0x80                 # last payload byte
    bad[2, end] ^= 0xFF                     # padding after the payload: outside the CRC
    bad[3, HEADER.size + 2 * scales] ^= 0x10  # first byte of the K codes
    bad[4, 0] = ord("Y")                    # magic: not copied, valid 0
    bad[5, 48] ^= 0x01                      # the stored CRC itself
    bad[6, 16] ^= 0x01                      # block id
    out = [t.cpu() for t in ops.decode_records(bad.to(DEV), spec, 0, torch.arange(9))]
    status = out[5].tolist()
    crc, hdr, bid = ops.RECORD_BAD_CRC, ops.RECORD_BAD_HEADER, ops.RECORD_BAD_ID
    assert status[:4] == [crc, crc, 0, crc]
    assert status[4] & hdr and int(out[4][4]) == 0
    assert status[5:] == [crc, bid, 0, 0]
    for i in (0, 1, 2, 3, 5, 6, 7, 8):  # copied whatever the CRC says
        blk = decode_record(bad[i].clone(), spec, verify_crc=False)
        assert torch.equal(out[0][i], blk.key.packed) and torch.equal(out[1][i], blk.value.packed)
        assert torch.equal(out[2][i].view(torch.int16), blk.key.scales.view(torch.int16))
        assert torch.equal(out[3][i].view(torch.int16), blk.value.scales.view(torch.int16))
        assert int(out[4][i]) == blk.valid_tokens


def test_unaligned_records_take_the_per_record_kernel_with_the_same_result():
    spec = CacheSpec(layers=1, kv_heads=8, head_dim=128, block_tokens=128, bits=4, group_size=32)
    raw = _encoded(spec, 5, 11)
    aligned = ops.decode_records(raw.to(DEV), spec, 0)
    flat = torch.zeros(raw.numel() + 4, dtype=torch.uint8, device=DEV)
    flat[4:] = raw.reshape(-1).to(DEV)
    shifted = ops.decode_records(flat[4:], spec, 0)    # 4-byte aligned, not 16
    torch.cuda.synchronize()
    for a, b in zip(aligned, shifted):
        assert torch.equal(a, b)
    _check_against_cpu(raw, spec, shifted)
