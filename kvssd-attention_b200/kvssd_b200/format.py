"""kvssd's on-disk record format: cache geometry, 4 KiB-aligned records and the manifest.

Byte-compatible with src/kvssd/format.py:16-177 so stores written by either implementation
read in the other: a 52-byte little-endian header ``<8sIIIIIIIIIII`` (magic ``KVSSD001``,
version 1, layer, block, valid_tokens, bits, block_tokens, kv_heads, head_dim, group_size,
payload_len, crc32 of the payload), then the payload -- K scales, V scales (FP16
[block_tokens, kv_heads, head_dim/group_size]), K codes, V codes (uint8
[block_tokens, kv_heads, head_dim*bits/8]) -- zero-padded to a multiple of 4096 bytes.
"""

from __future__ import annotations

import json
import struct
import zlib
from dataclasses import asdict, dataclass
from pathlib import Path

import torch

from .quant import QuantizedTensor

ALIGNMENT = 4096
MAGIC = b"KVSSD001"
HEADER = struct.Struct("<8sIIIIIIIIIII")


def align_up(value: int, alignment: int = ALIGNMENT) -> int:
    return -(-value // alignment) * alignment


@dataclass(frozen=True)
class CacheSpec:
    layers: int
    kv_heads: int
    head_dim: int
    block_tokens: int = 128
    bits: int = 4
    group_size: int = 32

    def validate(self) -> None:
        if min(self.layers, self.kv_heads, self.head_dim, self.block_tokens) <= 0:
            raise ValueError("all cache dimensions must be positive")
        if self.bits not in (2, 4):
            raise ValueError("bits must be 2 or 4")
        if self.head_dim % self.group_size:
            raise ValueError("head_dim must be divisible by group_size")

    @property
    def packed_dim(self) -> int:
        """Bytes of packed codes per (token, KV head)."""
        return self.head_dim * self.bits // 8

    @property
    def groups(self) -> int:
        return self.head_dim // self.group_size

    @property
    def scale_count(self) -> int:
        return self.block_tokens * self.kv_heads * self.groups

    @property
    def packed_count(self) -> int:
        return self.block_tokens * self.kv_heads * self.packed_dim

    @property
    def payload_bytes(self) -> int:
        return 2 * (self.scale_count * 2) + 2 * self.packed_count

    @property
    def record_bytes(self) -> int:
        return align_up(HEADER.size + self.payload_bytes)

    @property
    def packed_kv_bytes_per_block(self) -> int:
        """Bytes the decode kernel must read per block: K+V codes and K+V scales."""
        return self.payload_bytes


@dataclass(frozen=True)
class BlockEntry:
    layer: int
    block: int
    offset: int
    length: int
    valid_tokens: int
    crc32: int


@dataclass
class Manifest:
    spec: CacheSpec
    entries: list[BlockEntry]
    version: int = 1

    def save(self, path: Path) -> None:
        body = {
            "version": self.version,
            "spec": asdict(self.spec),
            "entries": [asdict(e) for e in self.entries],
        }
        path.write_text(json.dumps(body, indent=2) + "\n", encoding="utf-8")

    @classmethod
    def load(cls, path: Path) -> "Manifest":
        body = json.loads(path.read_text(encoding="utf-8"))
        return cls(
            spec=CacheSpec(**body["spec"]),
            entries=[BlockEntry(**e) for e in body["entries"]],
            version=body["version"],
        )


@dataclass(frozen=True)
class PackedKVBlock:
    layer: int
    block: int
    valid_tokens: int
    key: QuantizedTensor
    value: QuantizedTensor


def _payload_layout(spec: CacheSpec) -> list[tuple[str, int]]:
    scale_bytes = spec.scale_count * 2
    return [("ks", scale_bytes), ("vs", scale_bytes), ("kp", spec.packed_count),
            ("vp", spec.packed_count)]


def encode_record(block: PackedKVBlock, spec: CacheSpec) -> tuple[bytes, int]:
    """Serialises one padded block; returns (record bytes, payload crc32)."""
    expected = (spec.block_tokens, spec.kv_heads, spec.head_dim)
    if block.key.original_shape != expected or block.value.original_shape != expected:
        raise ValueError(f"padded KV block must have shape {expected}")

    def raw(t: torch.Tensor) -> bytes:
        return t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()

    payload = b"".join(
        (raw(block.key.scales), raw(block.value.scales), raw(block.key.packed),
         raw(block.value.packed))
    )
    crc = zlib.crc32(payload)
    header = HEADER.pack(MAGIC, 1, block.layer, block.block, block.valid_tokens, spec.bits,
                         spec.block_tokens, spec.kv_heads, spec.head_dim, spec.group_size,
                         len(payload), crc)
    body = header + payload
    return body + bytes(spec.record_bytes - len(body)), crc


def parse_header(raw: bytes | memoryview) -> tuple:
    return HEADER.unpack(bytes(raw[: HEADER.size]))


def decode_record(raw: torch.Tensor, spec: CacheSpec, verify_crc: bool = True) -> PackedKVBlock:
    """Views a CPU record as a PackedKVBlock (payload tensors alias ``raw``)."""
    if raw.dtype != torch.uint8 or raw.device.type != "cpu" or not raw.is_contiguous():
        raise TypeError("raw record must be a contiguous CPU uint8 tensor")
    view = memoryview(raw.numpy())
    magic, version, layer, block, valid, bits, bt, heads, dim, group, payload_len, crc = (
        parse_header(view)
    )
    if magic != MAGIC or version != 1:
        raise ValueError("invalid KVSSD record header")
    if (bits, bt, heads, dim, group) != (spec.bits, spec.block_tokens, spec.kv_heads,
                                         spec.head_dim, spec.group_size):
        raise ValueError("record layout does not match manifest")
    payload = view[HEADER.size : HEADER.size + payload_len]
    if verify_crc and zlib.crc32(payload) != crc:
        raise IOError(f"CRC mismatch for layer={layer}, block={block}")
    return _views(raw, spec, layer, block, valid)


def _views(raw: torch.Tensor, spec: CacheSpec, layer: int, block: int, valid: int) -> PackedKVBlock:
    scale_shape = (spec.block_tokens, spec.kv_heads, spec.groups)
    packed_shape = (spec.block_tokens, spec.kv_heads, spec.packed_dim)
    parts = {}
    cursor = HEADER.size
    for name, size in _payload_layout(spec):
        parts[name] = raw[cursor : cursor + size]
        cursor += size
    shape = (spec.block_tokens, spec.kv_heads, spec.head_dim)
    key = QuantizedTensor(parts["kp"].reshape(packed_shape),
                          parts["ks"].view(torch.float16).reshape(scale_shape), shape, spec.bits,
                          spec.group_size)
    value = QuantizedTensor(parts["vp"].reshape(packed_shape),
                            parts["vs"].view(torch.float16).reshape(scale_shape), shape,
                            spec.bits, spec.group_size)
    return PackedKVBlock(layer, block, valid, key, value)


def record_views(raw: torch.Tensor, spec: CacheSpec, entry: BlockEntry) -> PackedKVBlock:
    """Payload views of a record buffer on any device, trusting the manifest entry."""
    return _views(raw, spec, entry.layer, entry.block, entry.valid_tokens)
