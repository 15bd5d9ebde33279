"""Torch-tensor wrappers over the C ABI (include/kvssd_b200.h).

Every function here launches CUDA kernels from libkvssd_b200 on the current CUDA stream of
the tensors' device; none has a CPU path. Tensors are passed by data pointer, so callers must
pass contiguous CUDA tensors (the wrappers check and raise otherwise).
"""

from __future__ import annotations

import ctypes
import math
import threading

import torch

from . import _native

_QUERY_DTYPES = {
    torch.float32: _native.Q_F32,
    torch.float16: _native.Q_F16,
    torch.bfloat16: _native.Q_BF16,
    torch.float64: _native.Q_F64,
}

_WORKSPACE_HEADER = 2048


class _Workspaces:
    """Per-(device, stream) decode workspaces, grown on demand and reused across calls.

    Reuse is safe because calls that share a workspace are ordered on one stream. A workspace
    is zeroed once at allocation: the header's device status word (it accumulates until read),
    the fused combine's epoch and the part words, whose epoch tags must not match a future call.
    """

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._buffers: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> torch.Tensor:
        key = (device.index, stream.cuda_stream)
        with self._lock:
            buf = self._buffers.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 20)
                if buf is not None:
                    size = max(size, 2 * buf.numel())
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
                self._buffers[key] = buf
            return buf


_workspaces = _Workspaces()


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(name: str, t: torch.Tensor, device: torch.device, dtype: torch.dtype) -> None:
    if t.device != device:
        raise ValueError(f"{name} must be on {device}, got {t.device}")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _decode_args(query, packed_k, packed_v, scales_k, scales_v, valid_tokens, bits, group_size,
                 block_table):
    """Validates decode tensors; returns (query, geometry tuple, n_sel)."""
    device = query.device
    if device.type != "cuda":
        raise RuntimeError(f"kvssd_b200 decode requires a CUDA device, got {device}")
    if query.ndim != 2:
        raise ValueError("query must be [query_heads, head_dim]")
    if query.dtype not in _QUERY_DTYPES:
        raise ValueError(f"unsupported query dtype {query.dtype}")
    if not query.is_contiguous():
        query = query.contiguous()
    if packed_k.ndim != 4 or packed_k.shape != packed_v.shape:
        raise ValueError("packed KV must match [blocks,tokens,kv_heads,packed_dim]")
    if scales_k.ndim != 4 or scales_k.shape != scales_v.shape:
        raise ValueError("KV scales must match [blocks,tokens,kv_heads,groups]")
    for name, t, dt in (("packed_k", packed_k, torch.uint8), ("packed_v", packed_v, torch.uint8),
                        ("scales_k", scales_k, torch.float16), ("scales_v", scales_v, torch.float16),
                        ("valid_tokens", valid_tokens, torch.int32)):
        _require_cuda(name, t, device, dt)
    n_pool, bt, kvh, pd = packed_k.shape
    qh, d = query.shape
    if tuple(scales_k.shape[:3]) != (n_pool, bt, kvh) or scales_k.shape[3] * group_size != d:
        raise ValueError("scale dimension mismatch")
    if valid_tokens.shape != (n_pool,):
        raise ValueError("valid_tokens must contain one count per block")
    if pd * 8 != d * bits:
        raise ValueError("packed dimension does not match query head dimension")
    if block_table is not None:
        _require_cuda("block_table", block_table, device, torch.int32)
        if block_table.ndim != 1:
            raise ValueError("block_table must be 1-D")
        n_sel = block_table.shape[0]
    else:
        n_sel = n_pool
    return query, (n_pool, n_sel, bt, qh, kvh, d, bits, group_size)


def _workspace_for(device, geometry) -> tuple[torch.Tensor, torch.cuda.Stream]:
    n_pool, n_sel, bt, qh, kvh, d, bits, group_size = geometry
    need = ctypes.c_size_t()
    _native.check(
        _native.library().kvssd_b200_decode_workspace_size(n_sel, bt, qh, kvh, d, bits,
                                                           group_size, ctypes.byref(need)),
        "kvssd_b200_decode_workspace_size",
    )
    stream = torch.cuda.current_stream(device)
    return _workspaces.get(device, stream, need.value), stream


def decode(
    query: torch.Tensor,
    packed_k: torch.Tensor,
    packed_v: torch.Tensor,
    scales_k: torch.Tensor,
    scales_v: torch.Tensor,
    valid_tokens: torch.Tensor,
    bits: int,
    group_size: int,
    sm_scale: float,
    block_table: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    lse: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused dequantize + decode attention; returns (out fp32 [QH, D], lse fp32 [QH]).

    ``packed_*``/``scales_*``/``valid_tokens`` form a block pool; ``block_table`` (int32
    [n_sel]) selects and orders pool blocks (None = all pool blocks in order).
    """
    query, geom = _decode_args(query, packed_k, packed_v, scales_k, scales_v, valid_tokens, bits,
                               group_size, block_table)
    device = query.device
    n_pool, n_sel, bt, qh, kvh, d, _, _ = geom
    with torch.cuda.device(device):
        ws, stream = _workspace_for(device, geom)
        if out is None:
            out = torch.empty((qh, d), dtype=torch.float32, device=device)
        if lse is None:
            lse = torch.empty((qh,), dtype=torch.float32, device=device)
        _require_cuda("out", out, device, torch.float32)
        _require_cuda("lse", lse, device, torch.float32)
        status = _native.library().kvssd_b200_decode(
            _ptr(query), _QUERY_DTYPES[query.dtype],
            _ptr(packed_k), _ptr(packed_v), _ptr(scales_k), _ptr(scales_v),
            _ptr(valid_tokens), _ptr(block_table),
            n_pool, n_sel, bt, qh, kvh, d, bits, group_size,
            float(sm_scale), _ptr(out), _ptr(lse),
            _ptr(ws), ws.numel(), stream.cuda_stream,
        )
        _native.check(status, "kvssd_b200_decode")
    return out, lse


def decode_exchange(query, packed_k, packed_v, scales_k, scales_v, valid_tokens, bits: int,
                    group_size: int, sm_scale: float, rank: int, world: int,
                    buffers: list[int], block_table=None, out=None, lse=None,
                    workspace: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """This rank's share of a multi-GPU decode (token-block-range shards) with the cross-rank
    merge fused into the kernel (kvssd_b200_decode_exchange); returns the whole context's
    (out, lse), identical on every rank. ``buffers`` are the ranks' exchange buffers as device
    addresses valid in this process (see sharding.PeerExchange)."""
    query, geom = _decode_args(query, packed_k, packed_v, scales_k, scales_v, valid_tokens, bits,
                               group_size, block_table)
    device = query.device
    n_pool, n_sel, bt, qh, kvh, d, _, _ = geom
    with torch.cuda.device(device):
        if workspace is None:
            workspace, stream = _workspace_for(device, geom)
        else:
            stream = torch.cuda.current_stream(device)
        if out is None:
            out = torch.empty((qh, d), dtype=torch.float32, device=device)
        if lse is None:
            lse = torch.empty((qh,), dtype=torch.float32, device=device)
        _require_cuda("out", out, device, torch.float32)
        _require_cuda("lse", lse, device, torch.float32)
        ptrs = (ctypes.c_void_p * len(buffers))(*buffers)
        status = _native.library().kvssd_b200_decode_exchange(
            _ptr(query), _QUERY_DTYPES[query.dtype],
            _ptr(packed_k), _ptr(packed_v), _ptr(scales_k), _ptr(scales_v),
            _ptr(valid_tokens), _ptr(block_table),
            n_pool, n_sel, bt, qh, kvh, d, bits, group_size, float(sm_scale),
            rank, world, ptrs, _ptr(out), _ptr(lse),
            _ptr(workspace), workspace.numel(), stream.cuda_stream,
        )
        _native.check(status, "kvssd_b200_decode_exchange")
    return out, lse


class BatchedDecode:
    """Several independent decodes in ONE launch (kvssd_b200_decode_batched).

    ``problems``: sequence of (query, packed_k, packed_v, scales_k, scales_v, valid_tokens,
    block_table or None) sharing the geometry (INT4, head_dim 128, group 32/64). The device
    descriptor table, the outputs and the workspace are built once, so ``run()`` is a single
    launch with no host-to-device copy: it can be captured in a CUDA graph and replayed (the
    tensors the descriptors point to may be refilled in place between replays).
    """

    def __init__(self, problems, bits: int, group_size: int, sm_scale: float,
                 out: torch.Tensor | None = None, lse: torch.Tensor | None = None):
        """``out`` fp32 [L, QH, D] / ``lse`` fp32 [L, QH] (optional): contiguous buffers the
        L problems write into (e.g. one buffer to all-gather across ranks); allocated per
        problem when absent."""
        problems = list(problems)
        if not problems:
            raise ValueError("at least one problem is required")
        self.bits, self.group_size, self.sm_scale = bits, group_size, float(sm_scale)
        checked = []
        geom0 = None
        for prob in problems:
            query, kp, vp, ks, vs, valid, table = prob
            query, geom = _decode_args(query, kp, vp, ks, vs, valid, bits, group_size, table)
            n_pool, n_sel, bt, qh, kvh, d, _, _ = geom
            if geom0 is None:
                geom0 = (bt, qh, kvh, d, query.dtype, query.device)
            elif (bt, qh, kvh, d, query.dtype, query.device) != geom0:
                raise ValueError("batched problems must share geometry, query dtype and device")
            checked.append((query, kp, vp, ks, vs, valid, table, n_pool, n_sel))
        self.geometry = geom0
        bt, qh, kvh, d, qdtype, device = geom0
        self.device = device
        self._keep = checked  # the tensors the descriptors point to
        n = len(checked)
        if (out is None) != (lse is None):
            raise ValueError("pass both out and lse, or neither")
        if out is None:
            self.outs = [(torch.empty((qh, d), dtype=torch.float32, device=device),
                          torch.empty((qh,), dtype=torch.float32, device=device))
                         for _ in checked]
        else:
            if tuple(out.shape) != (n, qh, d) or tuple(lse.shape) != (n, qh):
                raise ValueError(f"out/lse must be [{n}, {qh}, {d}] and [{n}, {qh}]")
            _require_cuda("out", out, device, torch.float32)
            _require_cuda("lse", lse, device, torch.float32)
            self.outs = [(out[i], lse[i]) for i in range(n)]
        desc = torch.empty((len(checked), 10), dtype=torch.int64, pin_memory=True)
        for i, ((query, kp, vp, ks, vs, valid, table, n_pool, n_sel), (out, lse)) in enumerate(
                zip(checked, self.outs)):
            desc[i] = torch.tensor([_ptr(query), _ptr(kp), _ptr(vp), _ptr(ks), _ptr(vs),
                                    _ptr(valid), _ptr(table) or 0, _ptr(out), _ptr(lse),
                                    (n_pool & 0xFFFFFFFF) | (n_sel << 32)], dtype=torch.int64)
        self.descriptors = desc.to(device)
        need = ctypes.c_size_t()
        with torch.cuda.device(device):
            _native.check(_native.library().kvssd_b200_decode_batched_workspace_size(
                len(checked), bt, qh, kvh, d, bits, group_size, ctypes.byref(need)),
                "kvssd_b200_decode_batched_workspace_size")
        self.workspace = torch.zeros(need.value, dtype=torch.uint8, device=device)
        torch.cuda.synchronize(device)

    def run(self) -> list[tuple[torch.Tensor, torch.Tensor]]:
        bt, qh, kvh, d, qdtype, device = self.geometry
        with torch.cuda.device(device):
            _native.check(_native.library().kvssd_b200_decode_batched(
                _ptr(self.descriptors), len(self.outs), _QUERY_DTYPES[qdtype], bt, qh, kvh, d,
                self.bits, self.group_size, self.sm_scale, _ptr(self.workspace),
                self.workspace.numel(), _stream_handle(device)),
                "kvssd_b200_decode_batched")
        return self.outs

    def read_status(self, clear: bool = True) -> int:
        """The sticky device status word of this batch's workspace (bit 16: a refused
        descriptor; see read_device_status for the others)."""
        value = ctypes.c_uint()
        with torch.cuda.device(self.device):
            status = _native.library().kvssd_b200_read_status(
                _ptr(self.workspace), 1 if clear else 0, ctypes.byref(value),
                _stream_handle(self.device))
        if status not in (_native.OK, _native.ERR_DEVICE_STATUS):
            _native.check(status, "kvssd_b200_read_status")
        return int(value.value)


def decode_batched(problems, bits: int, group_size: int, sm_scale: float):
    """One-shot BatchedDecode: builds the descriptors and launches; returns [(out, lse), ...]."""
    return BatchedDecode(problems, bits, group_size, sm_scale).run()


RECORD_BAD_HEADER, RECORD_BAD_GEOMETRY, RECORD_BAD_LENGTH, RECORD_BAD_CRC = 1, 2, 4, 8
RECORD_BAD_ID, RECORD_BAD_VALID = 16, 32


def decode_records(records: torch.Tensor, spec, layer: int | None = None,
                   block_ids: torch.Tensor | None = None):
    """Raw kvssd records on a CUDA device -> PackedBatch tensors, CRC-32 checked on the device.

    ``records`` is uint8 [n, record_bytes] (or flat, n * record_bytes), as read from the store.
    Returns (packed_k, packed_v, scales_k, scales_v, valid_tokens, status) where status is
    int32 [n] with the RECORD_BAD_* bits of each record (0 = good); see
    kvssd_b200_decode_records. Asynchronous on the current stream.
    """
    device = records.device
    if device.type != "cuda":
        raise RuntimeError(f"decode_records requires a CUDA tensor, got {device}")
    if records.dtype != torch.uint8 or not records.is_contiguous():
        raise ValueError("records must be a contiguous uint8 tensor")
    stride = spec.record_bytes
    if records.numel() % stride:
        raise ValueError(f"records must be whole records of {stride} bytes")
    n = records.numel() // stride
    bt, kvh = spec.block_tokens, spec.kv_heads
    packed_k = torch.empty((n, bt, kvh, spec.packed_dim), dtype=torch.uint8, device=device)
    packed_v = torch.empty_like(packed_k)
    scales_k = torch.empty((n, bt, kvh, spec.groups), dtype=torch.float16, device=device)
    scales_v = torch.empty_like(scales_k)
    valid = torch.empty((n,), dtype=torch.int32, device=device)
    status = torch.empty((n,), dtype=torch.int32, device=device)
    if block_ids is not None:
        block_ids = block_ids.to(device=device, dtype=torch.int32).contiguous()
        if block_ids.shape != (n,):
            raise ValueError("block_ids must name one block per record")
    with torch.cuda.device(device):
        _native.check(
            _native.library().kvssd_b200_decode_records(
                _ptr(records), stride, n, -1 if layer is None else int(layer), _ptr(block_ids),
                spec.bits, bt, kvh, spec.head_dim, spec.group_size, _ptr(packed_k),
                _ptr(packed_v), _ptr(scales_k), _ptr(scales_v), _ptr(valid), _ptr(status),
                _stream_handle(device)),
            "kvssd_b200_decode_records",
        )
    return packed_k, packed_v, scales_k, scales_v, valid, status


def decode_split(query, packed_k, packed_v, scales_k, scales_v, valid_tokens, bits: int,
                 group_size: int, sm_scale: float, block_table=None) -> tuple[int, torch.Tensor]:
    """Runs only the streaming split-KV kernel; returns (n_parts, workspace).

    The parts stay in the returned workspace until the next decode on this stream;
    decode_combine folds them into (out, lse).
    """
    query, geom = _decode_args(query, packed_k, packed_v, scales_k, scales_v, valid_tokens, bits,
                               group_size, block_table)
    device = query.device
    n_pool, n_sel, bt, qh, kvh, d, _, _ = geom
    n_parts = ctypes.c_int()
    with torch.cuda.device(device):
        ws, stream = _workspace_for(device, geom)
        status = _native.library().kvssd_b200_decode_split(
            _ptr(query), _QUERY_DTYPES[query.dtype],
            _ptr(packed_k), _ptr(packed_v), _ptr(scales_k), _ptr(scales_v),
            _ptr(valid_tokens), _ptr(block_table),
            n_pool, n_sel, bt, qh, kvh, d, bits, group_size, float(sm_scale),
            _ptr(ws), ws.numel(), ctypes.byref(n_parts), stream.cuda_stream,
        )
        _native.check(status, "kvssd_b200_decode_split")
    return n_parts.value, ws


def decode_combine(workspace: torch.Tensor, n_parts: int, query_heads: int, head_dim: int,
                   out: torch.Tensor | None = None, lse: torch.Tensor | None = None):
    device = workspace.device
    if out is None:
        out = torch.empty((query_heads, head_dim), dtype=torch.float32, device=device)
    if lse is None:
        lse = torch.empty((query_heads,), dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        _native.check(
            _native.library().kvssd_b200_decode_combine(
                _ptr(workspace), n_parts, query_heads, head_dim, _ptr(out), _ptr(lse),
                _stream_handle(device)),
            "kvssd_b200_decode_combine",
        )
    return out, lse


def read_device_status(device: torch.device | str | None = None, clear: bool = True,
                       stream: torch.cuda.Stream | None = None) -> int:
    """Synchronously reads the sticky device status word of the current (or given) stream's
    workspace; ``clear`` zeroes the word (and the fused combine's test hook) when it is nonzero.

    Bit 1: a block-table entry was outside the pool; bit 2: a valid_tokens entry was outside
    [0, block_tokens] (such entries are skipped/clamped by the kernels, never dereferenced);
    bit 4: a fused combine, bit 8: a cross-GPU exchange, bit 32: a TMA-fed kernel's copy
    wait gave up (about a second) -- the out/lse of that call, and of later calls until the
    word is cleared, are NaN; bit 16: a batched problem descriptor was refused.
    """
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    stream = stream or torch.cuda.current_stream(device)
    ws = _workspaces.get(device, stream, _WORKSPACE_HEADER)
    value = ctypes.c_uint()
    with torch.cuda.device(device):
        status = _native.library().kvssd_b200_read_status(
            _ptr(ws), 1 if clear else 0, ctypes.byref(value), stream.cuda_stream
        )
    if status not in (_native.OK, _native.ERR_DEVICE_STATUS):
        _native.check(status, "kvssd_b200_read_status")
    return int(value.value)


def read_device_status_all(device: torch.device | str | None = None, clear: bool = True) -> int:
    """OR of the status words of every decode workspace on ``device`` (one per stream that has
    decoded, graph-capture streams included), read after synchronising the device."""
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    torch.cuda.synchronize(device)
    with _workspaces._lock:
        buffers = [buf for (dev, _), buf in _workspaces._buffers.items() if dev == device.index]
    total = 0
    stream = torch.cuda.current_stream(device)
    with torch.cuda.device(device):
        for ws in buffers:
            value = ctypes.c_uint()
            status = _native.library().kvssd_b200_read_status(
                _ptr(ws), 1 if clear else 0, ctypes.byref(value), stream.cuda_stream)
            if status not in (_native.OK, _native.ERR_DEVICE_STATUS):
                _native.check(status, "kvssd_b200_read_status")
            total |= int(value.value)
    return total


# Status bits that make a call's result invalid (the kernels then write NaN into out/lse) or
# that mean the caller passed entries the kernels had to refuse. Bit 2 (a valid_tokens entry
# outside [0, block_tokens], clamped like kvssd's CPU path clamps it by slicing) is not one.
FAILURE_BITS = (_native.DEV_BAD_BLOCK | _native.DEV_COMBINE_TIMEOUT |
                _native.DEV_EXCHANGE_TIMEOUT | _native.DEV_BAD_PROBLEM |
                _native.DEV_STREAM_TIMEOUT)

_STATUS_TEXT = {
    _native.DEV_BAD_BLOCK: "a block-table entry outside the pool",
    _native.DEV_BAD_VALID: "a valid_tokens entry outside [0, block_tokens]",
    _native.DEV_COMBINE_TIMEOUT: "the fused split-KV combine gave up waiting for parts",
    _native.DEV_EXCHANGE_TIMEOUT: "the cross-GPU exchange gave up waiting for another rank",
    _native.DEV_BAD_PROBLEM: "a batched problem descriptor was refused",
    _native.DEV_STREAM_TIMEOUT: "a TMA-fed kernel gave up waiting for its copies",
}


def describe_status(value: int) -> str:
    """Human-readable list of the conditions in a device status word."""
    parts = [text for bit, text in _STATUS_TEXT.items() if value & bit]
    return "; ".join(parts) or "none"


# Bits after which the kernels write NaN into out/lse (a wait gave up).
NAN_BITS = _native.DEV_COMBINE_TIMEOUT | _native.DEV_EXCHANGE_TIMEOUT | _native.DEV_STREAM_TIMEOUT


class DeviceFailure(RuntimeError):
    """A decode kernel flagged a failure in its workspace status word (see FAILURE_BITS)."""

    def __init__(self, status: int, where: str):
        self.status = status
        tail = ("; the out/lse of the failed call are NaN" if status & NAN_BITS else
                "; the offending entries were skipped, never dereferenced")
        super().__init__(f"{where}: device status {status:#x} ({describe_status(status)}){tail}")


class _StatusWatch:
    """Asynchronous reads of one (device, stream) workspace's status word.

    ``arm()`` enqueues, after a call's kernels, a 4-byte copy of the status word into a slot of
    pinned host memory and records an event; ``poll()`` looks at the slots whose event has
    completed (no synchronisation) and ``check()`` waits for all of them. A failure is raised
    once, as DeviceFailure, after the word has been read and cleared on the device (which
    makes the workspace usable again).
    """

    SLOTS = 4

    def __init__(self, device: torch.device, stream: torch.cuda.Stream):
        self.device, self.stream = device, stream
        self._host = torch.zeros(self.SLOTS, dtype=torch.int32, pin_memory=True)
        self._events: list[torch.cuda.Event | None] = [None] * self.SLOTS
        self._next = 0

    def _take(self, i: int, block: bool) -> int:
        ev = self._events[i]
        if ev is None:
            return 0
        if not block and not ev.query():
            return 0
        ev.synchronize()
        self._events[i] = None
        return int(self._host[i])

    def _raise(self, value: int, where: str) -> None:
        if value & FAILURE_BITS:
            read_device_status(self.device, clear=True, stream=self.stream)
            for i in range(self.SLOTS):  # older slots hold the same sticky bits
                self._events[i] = None
            raise DeviceFailure(value, where)

    def arm(self, where: str) -> None:
        if torch.cuda.is_current_stream_capturing():
            return  # inside a graph capture the caller checks after replay (check())
        i = self._next % self.SLOTS
        self._raise(self._take(i, block=True), where)  # the slot's earlier read, long done
        ws = _workspaces.get(self.device, self.stream, _WORKSPACE_HEADER)
        with torch.cuda.stream(self.stream):
            self._host[i:i + 1].copy_(ws[:4].view(torch.int32), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(self.stream)
        self._events[i] = ev
        self._next += 1

    def poll(self, where: str) -> None:
        value = 0
        for i in range(self.SLOTS):
            value |= self._take(i, block=False)
        self._raise(value, where)

    def check(self, where: str) -> None:
        value = 0
        for i in range(self.SLOTS):
            value |= self._take(i, block=True)
        self._raise(value, where)

    def discard(self) -> None:
        """Waits for the outstanding reads and drops them (the caller reads the word itself)."""
        for i in range(self.SLOTS):
            self._take(i, block=True)


_watch_lock = threading.Lock()
_watches: dict[tuple[int, int], _StatusWatch] = {}


def status_watch(device: torch.device, stream: torch.cuda.Stream | None = None) -> _StatusWatch:
    """The status watch of ``device``'s current (or given) stream workspace."""
    stream = stream or torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    with _watch_lock:
        w = _watches.get(key)
        if w is None:
            w = _watches[key] = _StatusWatch(device, stream)
        return w


def decode_path(head_dim: int, bits: int, group_size: int) -> int:
    path = ctypes.c_int()
    _native.check(
        _native.library().kvssd_b200_decode_path(head_dim, bits, group_size, ctypes.byref(path)),
        "kvssd_b200_decode_path",
    )
    return path.value


# decode_plan kernel names of the two streaming kernels (split-KV with the fused combine)
STREAMING_KERNELS = ("tensor_core_tma", "tensor_core_stream")


def decode_plan(n_sel: int, block_tokens: int, query_heads: int, kv_heads: int, head_dim: int,
                bits: int, group_size: int) -> dict:
    """Kernel choice and split count for a geometry on the current CUDA device."""
    kernel, splits, parts = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _native.check(
        _native.library().kvssd_b200_decode_plan(
            n_sel, block_tokens, query_heads, kv_heads, head_dim, bits, group_size,
            ctypes.byref(kernel), ctypes.byref(splits), ctypes.byref(parts)),
        "kvssd_b200_decode_plan",
    )
    names = {_native.PATH_TENSOR_CORE: "tensor_core_tma",
             _native.PATH_TENSOR_CORE_CPASYNC: "tensor_core_stream",
             _native.PATH_TENSOR_CORE_REGS: "tensor_core_regs", _native.PATH_GENERIC: "generic"}
    return {"kernel": names[kernel.value], "path": kernel.value, "n_splits": splits.value,
            "n_parts": parts.value}


def set_path_override(path: int) -> None:
    _native.check(_native.library().kvssd_b200_set_path_override(path), "set_path_override")


def merge_chunks(outs: torch.Tensor, lses: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact N-way merge of normalised chunks: outs [N, QH, D] fp32, lses [N, QH] fp32."""
    device = outs.device
    if device.type != "cuda":
        raise RuntimeError(f"merge_chunks requires CUDA tensors, got {device}")
    if outs.ndim != 3 or lses.shape != outs.shape[:2]:
        raise ValueError("expected outs [N, QH, D] and lses [N, QH]")
    _require_cuda("outs", outs, device, torch.float32)
    _require_cuda("lses", lses, device, torch.float32)
    n, qh, d = outs.shape
    out = torch.empty((qh, d), dtype=torch.float32, device=device)
    lse = torch.empty((qh,), dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        _native.check(
            _native.library().kvssd_b200_merge_chunks(
                _ptr(outs), _ptr(lses), n, qh, d, _ptr(out), _ptr(lse), _stream_handle(device)
            ),
            "kvssd_b200_merge_chunks",
        )
    return out, lse


def merge_pair(
    left_output: torch.Tensor, left_lse: torch.Tensor, right_output: torch.Tensor,
    right_lse: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    device = left_output.device
    if device.type != "cuda":
        raise RuntimeError(f"merge_attention_chunks requires CUDA tensors, got {device}")
    if left_output.ndim != 2 or right_output.shape != left_output.shape:
        raise ValueError("chunk outputs must both be [QH, D]")
    qh, d = left_output.shape
    if left_lse.shape != (qh,) or right_lse.shape != (qh,):
        raise ValueError("chunk LSEs must be [QH]")
    tensors = [t.contiguous().float() for t in (left_output, left_lse, right_output, right_lse)]
    for name, t in zip(("left_output", "left_lse", "right_output", "right_lse"), tensors):
        _require_cuda(name, t, device, torch.float32)
    out = torch.empty((qh, d), dtype=torch.float32, device=device)
    lse = torch.empty((qh,), dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        _native.check(
            _native.library().kvssd_b200_merge_pair(
                *map(_ptr, tensors), qh, d, _ptr(out), _ptr(lse), _stream_handle(device)
            ),
            "kvssd_b200_merge_pair",
        )
    return out, lse


def dequantize_packed(
    packed: torch.Tensor, scales: torch.Tensor, bits: int, group_size: int, mode: int = 0
) -> tuple[torch.Tensor, torch.Tensor]:
    """Runs the decode kernels' register unpacker over [rows, packed_dim] codes.

    Returns (codes uint8 [rows, D], values fp16 [rows, D]); used to prove bit-exactness
    against kvssd's unpack_codes / dequantize_tensor(q, torch.float16).
    """
    device = packed.device
    if device.type != "cuda":
        raise RuntimeError(f"dequantize_packed requires CUDA tensors, got {device}")
    pd = packed.shape[-1]
    d = pd * 8 // bits
    rows = packed.numel() // pd
    p2 = packed.reshape(rows, pd).contiguous()
    s2 = scales.reshape(rows, -1).contiguous()
    _require_cuda("packed", p2, device, torch.uint8)
    _require_cuda("scales", s2, device, torch.float16)
    values = torch.empty((rows, d), dtype=torch.float16, device=device)
    codes = torch.empty((rows, d), dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        _native.check(
            _native.library().kvssd_b200_dequantize(
                _ptr(p2), _ptr(s2), rows, d, bits, group_size, mode, _ptr(values), _ptr(codes),
                _stream_handle(device),
            ),
            "kvssd_b200_dequantize",
        )
    shape = (*packed.shape[:-1], d)
    return codes.reshape(shape), values.reshape(shape)


def default_sm_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
