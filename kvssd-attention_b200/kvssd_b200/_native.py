"""ctypes binding of libkvssd_b200.so (declarations: include/kvssd_b200.h).

This is the only place Python touches the native library. Loading never falls back to
anything: if the library is missing or does not export the full ABI, ``library()`` raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libkvssd_b200.so"

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_DEVICE_STATUS = 5

Q_F32, Q_F16, Q_BF16, Q_F64 = 0, 1, 2, 3
IPC_HANDLE_BYTES = 64
DEV_BAD_BLOCK, DEV_BAD_VALID, DEV_COMBINE_TIMEOUT, DEV_EXCHANGE_TIMEOUT = 1, 2, 4, 8
DEV_BAD_PROBLEM, DEV_STREAM_TIMEOUT = 16, 32
PATH_AUTO, PATH_TENSOR_CORE, PATH_GENERIC, PATH_TENSOR_CORE_REGS = 0, 1, 2, 3
PATH_TENSOR_CORE_CPASYNC = 4

_c_int = ctypes.c_int
_c_ll = ctypes.c_longlong
_c_float = ctypes.c_float
_c_size = ctypes.c_size_t
_c_void = ctypes.c_void_p
_c_uint_p = ctypes.POINTER(ctypes.c_uint)

# name -> (restype, argtypes); must match include/kvssd_b200.h exactly.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "kvssd_b200_version": (_c_int, []),
    "kvssd_b200_status_string": (ctypes.c_char_p, [_c_int]),
    "kvssd_b200_last_error": (ctypes.c_char_p, []),
    "kvssd_b200_decode_workspace_size": (
        _c_int,
        [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_size)],
    ),
    "kvssd_b200_decode": (
        _c_int,
        [
            _c_void, _c_int,  # query, dtype
            _c_void, _c_void, _c_void, _c_void,  # packed_k, packed_v, scales_k, scales_v
            _c_void, _c_void,  # valid_tokens, block_table
            _c_int, _c_int, _c_int,  # n_pool, n_sel, block_tokens
            _c_int, _c_int, _c_int, _c_int, _c_int,  # qh, kvh, d, bits, group
            _c_float, _c_void, _c_void,  # sm_scale, out, lse
            _c_void, _c_size, _c_void,  # workspace, bytes, stream
        ],
    ),
    "kvssd_b200_decode_static": (
        _c_int,
        [
            _c_void, _c_int, _c_void, _c_void, _c_void, _c_void, _c_void, _c_void,
            _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
            _c_float, _c_void, _c_void, ctypes.POINTER(_c_void), _c_void,
        ],
    ),
    "kvssd_b200_decode_split": (
        _c_int,
        [
            _c_void, _c_int, _c_void, _c_void, _c_void, _c_void, _c_void, _c_void,
            _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
            _c_float, _c_void, _c_size, ctypes.POINTER(_c_int), _c_void,
        ],
    ),
    "kvssd_b200_decode_combine": (_c_int, [_c_void, _c_int, _c_int, _c_int, _c_void, _c_void, _c_void]),
    "kvssd_b200_decode_path": (_c_int, [_c_int, _c_int, _c_int, ctypes.POINTER(_c_int)]),
    "kvssd_b200_decode_plan": (
        _c_int, [_c_int] * 7 + [ctypes.POINTER(_c_int)] * 3
    ),
    "kvssd_b200_set_path_override": (_c_int, [_c_int]),
    "kvssd_b200_read_status": (_c_int, [_c_void, _c_int, _c_uint_p, _c_void]),
    "kvssd_b200_decode_batched_workspace_size": (
        _c_int, [_c_int] * 7 + [ctypes.POINTER(_c_size)]
    ),
    "kvssd_b200_decode_batched": (
        _c_int,
        [_c_void, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float,
         _c_void, _c_size, _c_void],
    ),
    "kvssd_b200_decode_records": (
        _c_int,
        [_c_void, _c_size, _c_int, _c_int, _c_void, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_void, _c_void, _c_void, _c_void, _c_void, _c_void, _c_void],
    ),
    "kvssd_b200_read_records": (
        _c_int,
        [ctypes.c_char_p, _c_void, _c_int, _c_size, _c_void, _c_int, _c_int,
         ctypes.POINTER(_c_int)],
    ),
    "kvssd_b200_io_last_error": (ctypes.c_char_p, []),
    "kvssd_b200_host_register": (_c_int, [_c_void, _c_size, _c_int]),
    "kvssd_b200_host_unregister": (_c_int, [_c_void]),
    "kvssd_b200_copy_records_h2d": (_c_int, [_c_void, _c_size, _c_void, _c_int, _c_size, _c_void,
                                             _c_void]),
    "kvssd_b200_host_last_error": (ctypes.c_char_p, []),
    "kvssd_b200_gds_open": (_c_int, [ctypes.c_char_p, ctypes.POINTER(_c_void)]),
    "kvssd_b200_gds_read_records": (_c_int, [_c_void, _c_void, _c_int, _c_size, _c_void, _c_int]),
    "kvssd_b200_gds_close": (_c_int, [_c_void]),
    "kvssd_b200_gds_last_error": (ctypes.c_char_p, []),
    "kvssd_b200_exchange_bytes": (_c_int, [_c_int, _c_int, _c_int, ctypes.POINTER(_c_size)]),
    "kvssd_b200_exchange_alloc": (_c_int, [_c_size, ctypes.POINTER(_c_void)]),
    "kvssd_b200_exchange_clear": (_c_int, [_c_void, _c_size]),
    "kvssd_b200_exchange_free": (_c_int, [_c_void]),
    "kvssd_b200_ipc_handle": (_c_int, [_c_void, _c_void]),
    "kvssd_b200_ipc_open": (_c_int, [_c_void, ctypes.POINTER(_c_void)]),
    "kvssd_b200_ipc_close": (_c_int, [_c_void]),
    "kvssd_b200_decode_exchange": (
        _c_int,
        [
            _c_void, _c_int, _c_void, _c_void, _c_void, _c_void, _c_void, _c_void,
            _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
            _c_float, _c_int, _c_int, ctypes.POINTER(_c_void),
            _c_void, _c_void, _c_void, _c_size, _c_void,
        ],
    ),
    "kvssd_b200_merge_chunks": (
        _c_int, [_c_void, _c_void, _c_int, _c_int, _c_int, _c_void, _c_void, _c_void]
    ),
    "kvssd_b200_merge_pair": (
        _c_int,
        [_c_void, _c_void, _c_void, _c_void, _c_int, _c_int, _c_void, _c_void, _c_void],
    ),
    "kvssd_b200_dequantize": (
        _c_int,
        [_c_void, _c_void, _c_ll, _c_int, _c_int, _c_int, _c_int, _c_void, _c_void, _c_void],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeError(RuntimeError):
    """A nonzero status returned by libkvssd_b200."""

    def __init__(self, status: int, where: str, detail: str):
        self.status = status
        super().__init__(f"{where} failed: {detail or status_string(status)} (status {status})")


def library() -> ctypes.CDLL:
    """Loads the native library once; raises RuntimeError if it is absent or incomplete."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"kvssd_b200 native library not built ({LIB_PATH}); run "
                    "`python -m kvssd_b200._build`"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)  # AttributeError = incomplete ABI: fail loudly
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
        return _lib


def available() -> bool:
    try:
        library()
        return True
    except (OSError, RuntimeError, AttributeError):
        return False


def status_string(status: int) -> str:
    return library().kvssd_b200_status_string(status).decode()


def check(status: int, where: str) -> None:
    if status != OK:
        detail = library().kvssd_b200_last_error().decode()
        if status == ERR_INVALID_ARGUMENT:
            raise ValueError(f"{where}: {detail}")
        raise NativeError(status, where, detail)
