"""Record storage backends of KVCacheStore with kvssd's storage API
(src/kvssd/storage/base.py:12-39, registry.py:15-68): ``buffered`` positioned reads into host
memory, ``direct`` the same through the native O_DIRECT reader, and ``gds``, cuFile reads of
whole records straight into device memory (src/kvssd/storage/gds.py:13-94) through
libkvssd_b200's kvssd_b200_gds_* calls. ``auto`` takes gds where its probe succeeds, else
direct, else buffered, the reference's order.
"""

from __future__ import annotations

import ctypes
import os
import sys
import threading
from dataclasses import dataclass
from pathlib import Path
from typing import Protocol, runtime_checkable

import torch

from ._registry import FactoryTable
from .format import BlockEntry

ALIGNMENT = 4096


@dataclass(frozen=True)
class StorageAvailability:
    name: str
    available: bool
    direct: bool
    asynchronous: bool
    reason: str


@runtime_checkable
class StorageBackend(Protocol):
    """What KVCacheStore asks of a storage backend, kvssd's interface
    (src/kvssd/storage/base.py:21-39): a probe, aligned buffers, single-record reads and
    close. The backends here also offer ``read_records`` for batches of records."""

    name: str

    def probe(self) -> StorageAvailability: ...

    def allocate_buffer(self, size: int, *, pinned: bool = False,
                        device: torch.device | None = None) -> torch.Tensor: ...

    def read_into(self, entry: BlockEntry, destination: torch.Tensor) -> None: ...

    def close(self) -> None: ...


def _aligned(size: int, device: torch.device | str | None = None, pinned: bool = False):
    """A uint8 view of ``size`` bytes whose address is a multiple of 4096."""
    device = torch.device(device) if device is not None else torch.device("cpu")
    pin = pinned and device.type == "cpu" and torch.cuda.is_available()
    owner = torch.empty(size + ALIGNMENT - 1, dtype=torch.uint8, device=device, pin_memory=pin)
    shift = (-owner.data_ptr()) % ALIGNMENT
    return owner[shift:shift + size]


class BufferedStorageBackend:
    """Positioned reads (pread) into host tensors through one shared descriptor."""

    name = "buffered"
    direct = False

    def __init__(self, path: str | Path):
        self.path = Path(path)
        self._fd: int | None = None
        self._lock = threading.Lock()

    def probe(self) -> StorageAvailability:
        ok = self.path.is_file()
        return StorageAvailability(self.name, ok, False, False,
                                   "positioned reads" if ok else f"no data file: {self.path}")

    def allocate_buffer(self, size: int, *, pinned: bool = False,
                        device: torch.device | None = None) -> torch.Tensor:
        del device
        return _aligned(size, pinned=pinned)

    def _descriptor(self) -> int:
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
        got = os.preadv(self._descriptor(), [target], entry.offset)
        if got != entry.length:
            raise EOFError(f"short read for layer={entry.layer}, block={entry.block}: "
                           f"expected {entry.length}, got {got}")

    def close(self) -> None:
        with self._lock:
            if self._fd is not None:
                os.close(self._fd)
                self._fd = None


class DirectStorageBackend(BufferedStorageBackend):
    """The same reads, batched through the native reader with O_DIRECT (KVCacheStore.read_records
    asks for it; single-record reads stay positioned reads)."""

    name = "direct"
    direct = True

    def probe(self) -> StorageAvailability:
        if sys.platform != "linux" or not hasattr(os, "O_DIRECT"):
            return StorageAvailability(self.name, False, True, True, "O_DIRECT requires Linux")
        if not self.path.is_file():
            return StorageAvailability(self.name, False, True, True, f"no data file: {self.path}")
        try:
            os.close(os.open(self.path, os.O_RDONLY | os.O_DIRECT))
        except OSError as exc:
            return StorageAvailability(self.name, False, True, True, f"O_DIRECT open failed: {exc}")
        return StorageAvailability(self.name, True, True, True, "O_DIRECT reads, native threads")


_CUFILE_PROBE_SECONDS = 30
_cufile_probed: dict[str, str] = {}  # file -> "" (usable) or why not; "" key: a hung driver
_cufile_lock = threading.Lock()


def _cufile_opens(path: Path) -> str:
    """Opens and closes ``path`` through kvssd_b200_gds_open in a child process first, so that a
    cuFile driver that does not return (seen in containers without the GDS kernel module)
    cannot block the caller: a child that has not answered after 30 s is killed and the file is
    reported unavailable. Returns "" when the open succeeded, else the reason; cached per file."""
    import subprocess

    from . import _native

    key = str(path.resolve())
    with _cufile_lock:
        if key in _cufile_probed:
            return _cufile_probed[key]
        if "" in _cufile_probed:  # an earlier probe's driver open did not return: nor will this
            return _cufile_probed[""]
    code = ("import ctypes, sys\n"
            "lib = ctypes.CDLL(sys.argv[1])\n"
            "h = ctypes.c_void_p()\n"
            "lib.kvssd_b200_gds_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]\n"
            "lib.kvssd_b200_gds_last_error.restype = ctypes.c_char_p\n"
            "st = lib.kvssd_b200_gds_open(sys.argv[2].encode(), ctypes.byref(h))\n"
            "print(lib.kvssd_b200_gds_last_error().decode() if st else 'ok')\n"
            "if not st: lib.kvssd_b200_gds_close(h)\n")
    try:
        done = subprocess.run([sys.executable, "-c", code, str(_native.LIB_PATH), key],
                              capture_output=True, text=True, timeout=_CUFILE_PROBE_SECONDS)
        lines = done.stdout.strip().splitlines()
        answer = lines[-1] if lines else f"probe exited with {done.returncode}"
        reason = "" if answer == "ok" and done.returncode == 0 else answer
    except subprocess.TimeoutExpired:
        reason = f"cuFile open did not return within {_CUFILE_PROBE_SECONDS} s"
        with _cufile_lock:
            _cufile_probed[""] = reason
    with _cufile_lock:
        _cufile_probed[key] = reason
    return reason


class GDSStorageBackend:
    """cuFile reads of whole 4 KiB-aligned records into 4 KiB-aligned CUDA buffers."""

    name = "gds"
    direct = True

    def __init__(self, path: str | Path):
        self.path = Path(path)
        self._file: int | None = None
        self._lock = threading.Lock()

    def _lib(self):
        from . import _native

        return _native.library()

    def _handle(self) -> int:
        with self._lock:
            if self._file is None:
                handle = ctypes.c_void_p()
                lib = self._lib()
                if lib.kvssd_b200_gds_open(str(self.path).encode(), ctypes.byref(handle)) != 0:
                    raise OSError(lib.kvssd_b200_gds_last_error().decode())
                self._file = handle.value
            return self._file

    def probe(self) -> StorageAvailability:
        def no(reason: str) -> StorageAvailability:
            return StorageAvailability(self.name, False, True, True, reason)

        if sys.platform != "linux":
            return no("cuFile requires Linux")
        if not self.path.is_file():
            return no(f"data file does not exist: {self.path}")
        if not torch.cuda.is_available():
            return no("cuFile requires an NVIDIA CUDA device")
        reason = _cufile_opens(self.path)
        if reason:
            return no(f"cuFile probe failed: {reason}")
        try:
            self._handle()
        except Exception as exc:  # library missing, driver or O_DIRECT refused
            return no(f"cuFile probe failed: {exc}")
        return StorageAvailability(self.name, True, True, True,
                                   "cuFile direct reads into aligned CUDA buffers")

    def allocate_buffer(self, size: int, *, pinned: bool = False,
                        device: torch.device | None = None) -> torch.Tensor:
        del pinned
        return _aligned(size, device or torch.device("cuda"))

    def read_records(self, offsets: list[int], record_bytes: int, destination: torch.Tensor,
                     threads: int = 8) -> None:
        """Records at ``offsets`` into destination[i * record_bytes:] (a CUDA uint8 tensor,
        4096-byte aligned); returns when the bytes are in device memory."""
        if destination.device.type != "cuda" or destination.dtype != torch.uint8:
            raise ValueError("GDS backend requires a CUDA uint8 destination")
        if not destination.is_contiguous() or destination.numel() < len(offsets) * record_bytes:
            raise ValueError("GDS destination must be contiguous and large enough")
        if destination.data_ptr() % ALIGNMENT:
            raise ValueError(f"GDS destination address must be {ALIGNMENT}-byte aligned; "
                             f"got address=0x{destination.data_ptr():x}")
        if not offsets:
            return
        arr = (ctypes.c_longlong * len(offsets))(*offsets)
        lib = self._lib()
        with torch.cuda.device(destination.device):
            st = lib.kvssd_b200_gds_read_records(self._handle(), arr, len(offsets), record_bytes,
                                                 destination.data_ptr(), threads)
        if st != 0:
            raise OSError(f"cuFile read failed: {lib.kvssd_b200_gds_last_error().decode()}")

    def read_into(self, entry: BlockEntry, destination: torch.Tensor) -> None:
        if entry.offset % ALIGNMENT or entry.length % ALIGNMENT:
            raise ValueError(f"unaligned GDS read for layer={entry.layer}, block={entry.block}: "
                             f"offset={entry.offset}, length={entry.length}, "
                             f"alignment={ALIGNMENT}")
        try:
            self.read_records([entry.offset], entry.length, destination)
        except OSError as exc:
            raise OSError(f"cuFile read failed for layer={entry.layer}, block={entry.block}, "
                          f"offset={entry.offset}, bytes={entry.length}: {exc}") from exc

    def close(self) -> None:
        with self._lock:
            if self._file is not None:
                self._lib().kvssd_b200_gds_close(self._file)
                self._file = None


class MappedStorageBackend:
    """The store file mapped (mmap) and page-locked with the CUDA driver: reads into
    CUDA destinations are asynchronous DMA copies from the page cache on the current stream
    (kvssd_b200_copy_records_h2d: one copy per run of consecutive records), with no reader
    threads and no staging buffer; host reads are plain slices of the mapping. The whole file
    stays pinned while the backend is open, so this is for stores that fit in host memory, and
    one mapped backend per file at a time (the driver refuses to register the same pages
    twice). Not in kvssd; opt-in by name (``auto`` does not pick it)."""

    name = "mapped"
    direct = False
    device_reads_async = True

    def __init__(self, path: str | Path):
        self.path = Path(path)
        self._map = None
        self._view = None
        self._registered = 0
        self._devices: set[int] = set()  # devices with copies from the mapping enqueued
        self._lock = threading.Lock()

    def _lib(self):
        from . import _native

        return _native.library()

    def _mapping(self):
        """(numpy view of the whole file, its address), mapping and registering on first use."""
        import mmap

        import numpy as np

        with self._lock:
            if self._view is None:
                size = self.path.stat().st_size
                if size == 0:
                    raise OSError(f"empty data file: {self.path}")
                lib = self._lib()
                reasons = []
                # A shared read-only mapping registered read-only pins the page cache itself;
                # where the driver refuses that, a private mapping registered for writing
                # pins private copies of the pages (made once, at registration).
                for flags, prot, read_only in ((mmap.MAP_SHARED, mmap.PROT_READ, 1),
                                               (mmap.MAP_PRIVATE,
                                                mmap.PROT_READ | mmap.PROT_WRITE, 0)):
                    with open(self.path, "rb") as f:
                        mm = mmap.mmap(f.fileno(), size, flags=flags, prot=prot)
                    view = np.frombuffer(mm, dtype=np.uint8)
                    addr = view.ctypes.data
                    if lib.kvssd_b200_host_register(addr, size, read_only) == 0:
                        self._map, self._view, self._registered = mm, view, addr
                        break
                    reasons.append(lib.kvssd_b200_host_last_error().decode())
                    del view
                    mm.close()
                else:
                    raise OSError("; ".join(reasons))
            return self._view, self._registered

    def probe(self) -> StorageAvailability:
        def no(reason: str) -> StorageAvailability:
            return StorageAvailability(self.name, False, False, True, reason)

        if not self.path.is_file():
            return no(f"data file does not exist: {self.path}")
        if not torch.cuda.is_available():
            return no("page-locking a mapped file requires a CUDA device")
        # Map, register and let go again: the driver refuses a second registration of the same
        # pages, so a probe (available_storage_backends probes and drops every backend) must not
        # keep them; the first read maps the file anew.
        was_open = self._view is not None
        try:
            self._mapping()
        except Exception as exc:  # mmap refused, or the driver would not register the range
            return no(f"mapping failed: {exc}")
        finally:
            if not was_open:
                self.close()
        return StorageAvailability(self.name, True, False, True,
                                   "page-locked file mapping; DMA copies to the device")

    def allocate_buffer(self, size: int, *, pinned: bool = False,
                        device: torch.device | None = None) -> torch.Tensor:
        del pinned
        return _aligned(size, device or torch.device("cuda"))

    def read_records(self, offsets: list[int], record_bytes: int, destination: torch.Tensor,
                     threads: int = 8) -> None:
        """Records at ``offsets`` into destination[i * record_bytes:] (a CUDA uint8 tensor),
        enqueued on the current stream of the destination's device."""
        del threads
        if destination.device.type != "cuda" or destination.dtype != torch.uint8:
            raise ValueError("mapped reads into the device need a CUDA uint8 destination")
        if not destination.is_contiguous() or destination.numel() < len(offsets) * record_bytes:
            raise ValueError("destination must be contiguous and large enough")
        if not offsets:
            return
        view, addr = self._mapping()
        arr = (ctypes.c_longlong * len(offsets))(*offsets)
        lib = self._lib()
        stream = torch.cuda.current_stream(destination.device).cuda_stream
        with self._lock:
            self._devices.add(destination.device.index)
        with torch.cuda.device(destination.device):
            st = lib.kvssd_b200_copy_records_h2d(addr, view.size, arr, len(offsets), record_bytes,
                                                 destination.data_ptr(), stream)
        if st != 0:
            raise OSError(f"mapped record copy failed: {lib.kvssd_b200_host_last_error().decode()}")

    def read_into(self, entry: BlockEntry, destination: torch.Tensor) -> None:
        if destination.device.type == "cuda":
            self.read_records([entry.offset], entry.length, destination)
            return
        if destination.dtype != torch.uint8 or destination.numel() < entry.length:
            raise ValueError("destination must be a sufficiently large uint8 tensor")
        view, _ = self._mapping()
        if entry.offset + entry.length > view.size:
            raise EOFError(f"short read for layer={entry.layer}, block={entry.block}")
        destination[: entry.length].copy_(
            torch.from_numpy(view[entry.offset:entry.offset + entry.length].copy()))

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def close(self) -> None:
        with self._lock:
            if self._view is not None:
                # no copy from the mapping may still be in flight, on any device it fed
                for device in sorted(self._devices):
                    try:
                        torch.cuda.synchronize(device)
                    except Exception:
                        pass
                self._devices.clear()
                self._lib().kvssd_b200_host_unregister(self._registered)
                self._view = None
                self._map.close()
                self._map = None
                self._registered = 0


# kvssd's three backends, in the order ``auto`` tries them, then ``mapped``, which ``auto``
# never picks (it pins the whole file in host memory)
_table = FactoryTable("storage")
for _name, _factory in (("gds", GDSStorageBackend), ("direct", DirectStorageBackend),
                        ("buffered", BufferedStorageBackend)):
    _table.add(_name, _factory, auto=True)
_table.add("mapped", MappedStorageBackend, auto=False)


def register_storage_backend(name: str, factory) -> None:
    """Adds (or replaces) a backend under ``name`` (case-insensitive, not 'auto'). As in
    kvssd, ``auto`` only considers the names gds, direct and buffered, so a factory registered
    under one of those replaces that step of ``auto``; other names are chosen explicitly."""
    _table.add(name, factory)


def _close(backend) -> None:
    close = getattr(backend, "close", None)
    if close is not None:
        close()


def available_storage_backends(path: str | Path) -> list[StorageAvailability]:
    """The probe result of every registered backend for ``path``; each probed instance is closed
    again (a gds probe opens a cuFile handle and an O_DIRECT descriptor)."""
    states = []
    for key in _table.names():
        backend = _table.factory(key)(Path(path))
        try:
            states.append(backend.probe())
        finally:
            _close(backend)
    return states


def resolve_storage_backend(requested, path: str | Path):
    """An instance (probed), a registered name, or ``auto``/None: gds, direct, buffered in that
    order of preference. Unavailable explicit choices raise RuntimeError; unknown names
    ValueError (kvssd's messages). Probed instances that are not returned are closed."""
    path = Path(path)
    return _table.resolve(requested, lambda factory: factory(path),
                          lambda backend: backend.probe(), path, release=_close)
