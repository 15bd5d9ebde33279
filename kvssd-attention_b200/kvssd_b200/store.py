"""KVCacheStore: append-only fixed-record KV cache file plus manifest.

API-compatible with src/kvssd/store.py:20-113 (create / open / entry / blocks_for_layer /
read_into / read / close) and byte-compatible on disk. Host reads are positioned reads (pread)
of whole 4 KiB-aligned records, batched through the native O_DIRECT reader by read_records;
with the ``gds`` storage backend (storage.py) read_records and read_into also take CUDA
destinations, filled by cuFile straight from the file, and with ``mapped`` (the file mapped and
page-locked) by DMA copies from the page cache. The default (None) is ``buffered``
(the native batch reader still tries O_DIRECT); ``auto`` follows kvssd's order (gds, direct,
buffered).
"""

from __future__ import annotations

import os
import threading
from pathlib import Path

import torch

from .format import BlockEntry, CacheSpec, Manifest, PackedKVBlock, decode_record, encode_record
from .quant import QuantizedTensor, quantize_tensor

DATA_FILE = "blocks.kvssd"
MANIFEST_FILE = "manifest.json"


def _quantized_blocks(keys: torch.Tensor, values: torch.Tensor, spec: CacheSpec):
    """Yields the PackedKVBlocks of every (layer, block) in store order, one layer of keys and
    values quantized at a time."""
    layers, tokens = keys.shape[0], keys.shape[1]
    bt = spec.block_tokens
    n_blocks = -(-tokens // bt)
    block_shape = (bt, spec.kv_heads, spec.head_dim)

    def whole_blocks(x: torch.Tensor) -> QuantizedTensor:
        padded = torch.zeros((n_blocks * bt, spec.kv_heads, spec.head_dim), dtype=x.dtype)
        padded[:tokens].copy_(x.cpu())
        return quantize_tensor(padded.view(n_blocks, *block_shape), spec.bits, spec.group_size)

    def part(q: QuantizedTensor, b: int) -> QuantizedTensor:
        return QuantizedTensor(q.packed[b], q.scales[b], block_shape, spec.bits, spec.group_size)

    for layer in range(layers):
        kq, vq = whole_blocks(keys[layer]), whole_blocks(values[layer])
        for b in range(n_blocks):
            valid = min(bt, tokens - b * bt)
            yield PackedKVBlock(layer, b, valid, part(kq, b), part(vq, b))


class _PreadFile:
    """One lazily opened read-only descriptor shared by reader threads."""

    def __init__(self, path: Path):
        self.path = path
        self._fd: int | None = None
        self._lock = threading.Lock()

    def fd(self) -> int:
        with self._lock:
            if self._fd is None:
                self._fd = os.open(self.path, os.O_RDONLY)
            return self._fd

    def read_into(self, entry: BlockEntry, destination: torch.Tensor) -> None:
        if destination.device.type != "cpu":
            raise ValueError("record reads require a CPU destination tensor")
        if destination.dtype != torch.uint8 or destination.numel() < entry.length:
            raise ValueError("destination must be a sufficiently large uint8 tensor")
        target = memoryview(destination[: entry.length].numpy())
        got = os.preadv(self.fd(), [target], entry.offset)
        if got != entry.length:
            raise EOFError(
                f"short read for layer={entry.layer}, block={entry.block}: "
                f"expected {entry.length}, got {got}"
            )

    def close(self) -> None:
        with self._lock:
            if self._fd is not None:
                os.close(self._fd)
                self._fd = None


class KVCacheStore:
    """Append-only fixed-record KV cache store designed for large sequential reads."""

    def __init__(self, root: str | Path, manifest: Manifest, storage_backend=None):
        from .storage import resolve_storage_backend

        self.root = Path(root)
        # None: positioned reads, batched by read_records through the native reader (which
        # uses O_DIRECT where the file system allows it)
        self.storage_backend = resolve_storage_backend(
            "buffered" if storage_backend is None else storage_backend, self.root / DATA_FILE)
        self.manifest = manifest
        self.spec = manifest.spec
        self._entries = {(e.layer, e.block): e for e in manifest.entries}
        self._layer_blocks: dict[int, list[int]] = {}
        for e in manifest.entries:
            self._layer_blocks.setdefault(e.layer, []).append(e.block)
        for blocks in self._layer_blocks.values():
            blocks.sort()
        self._file = _PreadFile(self.root / DATA_FILE)

    @classmethod
    def create(
        cls,
        root: str | Path,
        keys: torch.Tensor,
        values: torch.Tensor,
        spec: CacheSpec,
        storage_backend: str | None = None,
    ) -> "KVCacheStore":
        """Creates a store from [layers, tokens, kv_heads, head_dim] tensors.

        Tokens are cut into blocks of ``block_tokens``; the last block of a layer is
        zero-padded and records its valid row count (the contract of src/kvssd/store.py:27-67).
        Each layer is quantized in one call: its token axis is zero-padded to whole blocks and
        viewed as [blocks, block_tokens, kv_heads, head_dim]; the quantization groups lie along
        head_dim, so this equals quantizing block by block. Records are then encoded from
        per-block views of the result and written by ``from_blocks``.
        """
        spec.validate()
        if keys.shape != values.shape or keys.ndim != 4:
            raise ValueError("keys and values must share [layers,tokens,kv_heads,head_dim]")
        if keys.shape[0] != spec.layers or tuple(keys.shape[2:]) != (spec.kv_heads, spec.head_dim):
            raise ValueError("input tensors do not match CacheSpec")
        return cls.from_blocks(root, spec, _quantized_blocks(keys, values, spec),
                               storage_backend)

    @classmethod
    def from_blocks(cls, root: str | Path, spec: CacheSpec, blocks,
                    storage_backend: str | None = None) -> "KVCacheStore":
        """Writes already-quantized PackedKVBlocks (any order of (layer, block)) as a store in
        the same byte format as ``create``."""
        spec.validate()
        root = Path(root)
        root.mkdir(parents=True, exist_ok=True)
        entries: list[BlockEntry] = []
        with (root / DATA_FILE).open("wb") as out:
            for block in blocks:
                record, crc = encode_record(block, spec)
                offset = out.tell()
                out.write(record)
                entries.append(BlockEntry(block.layer, block.block, offset, len(record),
                                          block.valid_tokens, crc))
        manifest = Manifest(spec=spec, entries=entries)
        manifest.save(root / MANIFEST_FILE)
        return cls(root, manifest, storage_backend)

    @classmethod
    def open(cls, root: str | Path, storage_backend: str | None = None) -> "KVCacheStore":
        root = Path(root)
        manifest = Manifest.load(root / MANIFEST_FILE)
        manifest.spec.validate()
        return cls(root, manifest, storage_backend)

    def entry(self, layer: int, block: int) -> BlockEntry:
        try:
            return self._entries[(layer, block)]
        except KeyError as exc:
            raise KeyError(f"no KV block layer={layer}, block={block}") from exc

    def blocks_for_layer(self, layer: int) -> list[int]:
        """Sorted block ids of a layer (precomputed; the reference scans all entries)."""
        return list(self._layer_blocks.get(layer, []))

    @property
    def reads_to_device(self) -> bool:
        """True when read_records can fill CUDA destinations directly: cuFile (gds, synchronous)
        or DMA from the page-locked mapping (mapped, enqueued on the current stream)."""
        return getattr(self.storage_backend, "name", "") in ("gds", "mapped")

    def read_into(self, entry: BlockEntry, destination: torch.Tensor) -> None:
        if destination.device.type == "cuda":
            if not self.reads_to_device:
                raise ValueError("CUDA destinations need the 'gds' or 'mapped' storage backend")
            self.storage_backend.read_into(entry, destination)
            return
        self._file.read_into(entry, destination)

    def read_records(self, layer: int, block_ids, destination: torch.Tensor | None = None,
                     threads: int = 8, direct: bool = True) -> torch.Tensor:
        """Raw records of ``block_ids`` in one call of the native reader (O_DIRECT where the file
        system allows it, a pool of reader threads). Returns uint8 [n, record_bytes] (pinned
        when CUDA is available, or ``destination``), ready for one host-to-device copy and
        ops.decode_records on the GPU. A CUDA ``destination`` (4096-byte aligned) is filled by
        cuFile with the gds backend, with no host copy."""
        import ctypes

        from . import _native

        ids = list(block_ids)
        rb = self.spec.record_bytes
        if destination is not None and destination.device.type == "cuda":
            if not self.reads_to_device:
                raise ValueError("CUDA destinations need the 'gds' or 'mapped' storage backend")
            offsets = []
            for b in ids:
                entry = self.entry(layer, b)
                if entry.length != rb:
                    raise ValueError("records of one store all have the spec's record_bytes")
                offsets.append(entry.offset)
            flat = destination.view(-1)
            self.storage_backend.read_records(offsets, rb, flat, threads)
            self.last_read_direct = bool(self.storage_backend.direct)
            return flat[: len(ids) * rb].view(len(ids), rb)
        if destination is None:
            destination = torch.empty((len(ids), rb), dtype=torch.uint8,
                                      pin_memory=torch.cuda.is_available())
        if destination.dtype != torch.uint8 or destination.device.type != "cpu" or \
                not destination.is_contiguous() or destination.numel() < len(ids) * rb:
            raise ValueError("destination must be a contiguous CPU uint8 tensor of n records")
        if not ids:
            return destination[:0]
        offsets = (ctypes.c_longlong * len(ids))()
        for i, b in enumerate(ids):
            entry = self.entry(layer, b)
            if entry.length != rb:
                raise ValueError("records of one store all have the spec's record_bytes")
            offsets[i] = entry.offset
        used = ctypes.c_int()
        lib = _native.library()
        status = lib.kvssd_b200_read_records(str(self._file.path).encode(), offsets, len(ids), rb,
                                             destination.data_ptr(), threads, int(direct),
                                             ctypes.byref(used))
        if status != _native.OK:
            raise OSError(f"record read failed: {lib.kvssd_b200_io_last_error().decode()}")
        self.last_read_direct = bool(used.value)
        return destination[: len(ids)].view(len(ids), rb)

    def read(self, layer: int, block: int, verify_crc: bool = True) -> PackedKVBlock:
        entry = self.entry(layer, block)
        raw = torch.empty(entry.length, dtype=torch.uint8)
        self.read_into(entry, raw)
        return decode_record(raw, self.spec, verify_crc)

    def close(self) -> None:
        self._file.close()
        self.storage_backend.close()

    def __enter__(self) -> "KVCacheStore":
        return self

    def __exit__(self, *_: object) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass
