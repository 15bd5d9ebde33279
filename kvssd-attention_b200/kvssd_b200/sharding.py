"""Multi-GPU decode: one process per GPU, the packed KV of a layer sharded two ways.

* Token-block ranges (long contexts): rank r owns a contiguous, balanced range of the
  selected blocks, decodes it into a normalised (out, lse) pair for every query head, and
  the ranks exchange those pairs with one all-gather of ``query_heads * (head_dim + 1)``
  FP32 values each; every rank then folds the N pairs with the exact N-way merge (the algebra
  of kvssd's merge_attention_chunks, src/kvssd/attention.py:91-102, generalised to N).
* KV-head groups (many layers, moderate contexts): rank r owns KV heads
  ``[r*KVH/N, (r+1)*KVH/N)`` and the query heads mapped to them by kvssd's GQA rule
  ``kv = h // (QH/KVH)`` (csrc/fused_decode.cu:34, backends/reference.py:41). No softmax
  merge is needed: the ranks all-gather their output rows and LSEs and concatenate them in
  rank order. kvssd records interleave heads per token (src/kvssd/format.py:165), so a
  head shard is re-laid head-contiguous (``shard_batch_by_heads``) when it is staged.

Transports. For token shards on CUDA with the streaming kernel's shapes, ``transport="auto"``
(or ``"peer"``) runs the whole step as ONE kernel per rank (kvssd_b200_decode_exchange): each
rank's combined slices are pushed with peer stores over NVLink into every rank's exchange
buffer (mapped through CUDA IPC, see PeerExchange) and merged there, so no collective library
call and no extra kernel is on the path. Otherwise (``"nccl"``, head shards, other shapes) the
exchange is an all-gather of the caller's process group (NCCL over NVLink for CUDA tensors)
and the merge libkvssd_b200's N-way merge kernel; a ``decode_fn`` / ``merge_fn`` with the
backend ``run`` / merge signatures can be injected instead (the host logic is the same).
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import replace

import torch
import torch.distributed as dist

from .backends.base import PackedBatch

DecodeFn = Callable[[torch.Tensor, PackedBatch, float], tuple[torch.Tensor, torch.Tensor]]
MergeFn = Callable[[torch.Tensor, torch.Tensor], tuple[torch.Tensor, torch.Tensor]]

MODES = ("tokens", "heads")
TRANSPORTS = ("auto", "nccl", "peer")


def block_range(n_blocks: int, rank: int, world: int) -> tuple[int, int]:
    """Balanced contiguous block range [lo, hi) of ``rank`` (sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_blocks < 0:
        raise ValueError("n_blocks must be non-negative")
    base, extra = divmod(n_blocks, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def head_shard(kv_heads: int, query_heads: int, rank: int, world: int) -> tuple[int, int, int, int]:
    """(kv_lo, kv_hi, q_lo, q_hi) owned by ``rank``; KV heads must divide evenly over ranks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads do not divide over {world} ranks")
    if query_heads % kv_heads:
        raise ValueError("query heads must be divisible by KV heads")
    per = kv_heads // world
    gqa = query_heads // kv_heads
    return rank * per, (rank + 1) * per, rank * per * gqa, (rank + 1) * per * gqa


def shard_batch_by_blocks(batch: PackedBatch, rank: int, world: int) -> PackedBatch:
    """The block-range shard of a stacked batch (views; no copy)."""
    lo, hi = block_range(batch.packed_k.shape[0], rank, world)
    return replace(batch, packed_k=batch.packed_k[lo:hi], packed_v=batch.packed_v[lo:hi],
                   scales_k=batch.scales_k[lo:hi], scales_v=batch.scales_v[lo:hi],
                   valid_tokens=batch.valid_tokens[lo:hi])


def shard_batch_by_heads(batch: PackedBatch, rank: int, world: int,
                         query_heads: int) -> PackedBatch:
    """The KV-head shard of a stacked batch, re-laid head-contiguous (a copy)."""
    kv_lo, kv_hi, _, _ = head_shard(batch.packed_k.shape[2], query_heads, rank, world)
    cut = lambda t: t[:, :, kv_lo:kv_hi].contiguous()  # noqa: E731
    return replace(batch, packed_k=cut(batch.packed_k), packed_v=cut(batch.packed_v),
                   scales_k=cut(batch.scales_k), scales_v=cut(batch.scales_v))


def _default_merge() -> MergeFn:
    from . import ops

    return ops.merge_chunks


class PeerExchange:
    """Exchange buffers of a process group, mapped into every rank over CUDA IPC.

    Each rank allocates one buffer (kvssd_b200_exchange_bytes for the group size and query
    geometry) on its GPU, exports an IPC handle, and opens every peer's handle; ``buffers``
    lists all ranks' buffers as device addresses valid in this process, in rank order.
    Collective: every rank of ``group`` constructs it (and closes it) at the same point.
    """

    def __init__(self, group: dist.ProcessGroup | None, device: torch.device, query_heads: int,
                 head_dim: int):
        import ctypes

        from . import _native

        lib = _native.library()
        self.group = group
        self.device = device
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.query_heads, self.head_dim = query_heads, head_dim
        nbytes = ctypes.c_size_t()
        _native.check(lib.kvssd_b200_exchange_bytes(self.world, query_heads, head_dim,
                                                    ctypes.byref(nbytes)), "exchange_bytes")
        self.nbytes = nbytes.value
        local = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(_native.IPC_HANDLE_BYTES)
        with torch.cuda.device(device):
            _native.check(lib.kvssd_b200_exchange_alloc(self.nbytes, ctypes.byref(local)),
                          "exchange_alloc")
            _native.check(lib.kvssd_b200_ipc_handle(local, handle), "ipc_handle")
        self._local = local.value
        handles: list[bytes | None] = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.buffers: list[int] = []
        self._opened: list[int] = []
        with torch.cuda.device(device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.buffers.append(self._local)
                    continue
                peer = ctypes.c_void_p()
                _native.check(lib.kvssd_b200_ipc_open(h, ctypes.byref(peer)), "ipc_open")
                self.buffers.append(peer.value)
                self._opened.append(peer.value)

    def reset(self) -> None:
        """Re-zeroes every rank's buffer (call numbers and flags) after an exchange timeout
        left the ranks' call numbers apart. Collective; no exchange may be in flight."""
        from . import _native

        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            _native.check(_native.library().kvssd_b200_exchange_clear(self._local, self.nbytes),
                          "exchange_clear")
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (collective, after all use)."""
        from . import _native

        if self._local is None:
            return
        lib = _native.library()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                _native.check(lib.kvssd_b200_ipc_close(p), "ipc_close")
            self._opened.clear()
            dist.barrier(group=self.group)
            _native.check(lib.kvssd_b200_exchange_free(self._local), "exchange_free")
        self._local = None


class ShardedDecoder:
    """Decodes this rank's shard and returns the full (out fp32 [QH, D], lse fp32 [QH]) on
    every rank of ``group``.

    ``mode="tokens"``: ``local`` is this rank's block-range shard (it may hold no blocks,
    which contributes an empty chunk: out 0, lse -inf). ``mode="heads"``: ``local`` is this
    rank's KV-head shard and ``query`` the full query; the rank decodes its query heads.
    All ranks take the same collective steps in the same order, whatever their shard holds.
    """

    def __init__(self, mode: str = "tokens", group: dist.ProcessGroup | None = None,
                 decode_fn: DecodeFn | None = None, merge_fn: MergeFn | None = None,
                 transport: str = "auto"):
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}")
        if transport not in TRANSPORTS:
            raise ValueError(f"transport must be one of {TRANSPORTS}")
        if transport == "peer" and (mode != "tokens" or decode_fn is not None):
            raise ValueError("the peer transport serves token shards with the native decode")
        self.mode = mode
        self.group = group
        self.decode_fn = decode_fn
        self.merge_fn = merge_fn
        self.transport = transport
        self._send: torch.Tensor | None = None
        self._recv: torch.Tensor | None = None
        self._peer: PeerExchange | None = None
        self._peer_out: tuple[torch.Tensor, torch.Tensor] | None = None
        self._device: torch.device | None = None  # the device of the last run
        self._stand_in: tuple | None = None  # (shape key, one-block empty batch) for empty shards

    def _use_peer(self, query: torch.Tensor, local: PackedBatch) -> bool:
        """Token shards on CUDA with a native streaming kernel (INT4 or INT2, head_dim 128, group
        32/64) and more than one rank: one fused kernel per rank.

        Decided from what every rank shares -- the geometry, not the number of blocks, their
        alignment or whether this rank holds any -- so that all ranks take the same transport:
        a rank that chose the all-gather while the others ran the exchange kernel would leave
        both sides waiting for a partner. The kernel choice depends on the geometry alone."""
        if self.transport == "nccl" or self.mode != "tokens" or self.decode_fn is not None:
            return False
        if self.world == 1 or query.device.type != "cuda":
            return False
        from . import ops

        _, block_tokens, kv_heads, _ = local.packed_k.shape
        plan = ops.decode_plan(1, block_tokens, query.shape[0], kv_heads, query.shape[1],
                               local.bits, local.group_size)
        ok = plan["kernel"] in ops.STREAMING_KERNELS
        if self.transport == "peer" and not ok:
            raise RuntimeError("peer transport needs the streaming kernel's shapes")
        return ok

    def _peer_operands(self, local: PackedBatch) -> PackedBatch:
        """The shard as the exchange kernel takes it. An empty shard joins the exchange as a
        one-block stand-in with no valid tokens, for which the kernel returns out 0 and lse -inf
        (no weight in the ranks' merge); operands that are not contiguous and 16-byte aligned
        are copied. The stand-in is kept for later calls of the same shape."""
        if local.packed_k.shape[0] == 0:
            _, block_tokens, kv_heads, packed_dim = local.packed_k.shape
            groups = local.scales_k.shape[3]
            key = (block_tokens, kv_heads, packed_dim, groups, local.scales_k.dtype,
                   local.packed_k.device, local.bits, local.group_size)
            if self._stand_in is None or self._stand_in[0] != key:
                dev = local.packed_k.device
                codes = torch.zeros((1, block_tokens, kv_heads, packed_dim), dtype=torch.uint8,
                                    device=dev)
                scales = torch.zeros((1, block_tokens, kv_heads, groups),
                                     dtype=local.scales_k.dtype, device=dev)
                self._stand_in = (key, replace(local, packed_k=codes, packed_v=codes,
                                               scales_k=scales, scales_v=scales,
                                               valid_tokens=torch.zeros(1, dtype=torch.int32,
                                                                        device=dev)))
            return self._stand_in[1]

        def ready(t: torch.Tensor) -> torch.Tensor:
            if t.is_contiguous() and t.data_ptr() % 16 == 0:
                return t
            return t.clone(memory_format=torch.contiguous_format)

        return replace(local, packed_k=ready(local.packed_k), packed_v=ready(local.packed_v),
                       scales_k=ready(local.scales_k), scales_v=ready(local.scales_v),
                       valid_tokens=local.valid_tokens.to(torch.int32).contiguous())

    def check(self) -> None:
        """Collective failure check: every rank of the group calls it at the same point.

        Each rank waits for its decodes, reads and clears the status words of its device's
        decode workspaces (graph-capture streams included), and the ranks all-gather them. If any rank flagged a failure (a wait that gave up: the
        exchange, the fused combine or a TMA copy; or a refused block-table entry), every rank
        re-zeroes the peer-exchange buffers (after a rank missed a call the ranks' call numbers
        differ, so later calls could never meet) and raises ops.DeviceFailure with the OR of
        the words. A failed step has already returned NaN on every rank that ran it (the
        exchange spreads a NaN slice to all ranks); ``run`` itself never raises on a device
        failure, since a rank that stopped alone would leave the others' next exchange
        without a partner.
        """
        from . import ops

        device = self._device
        value = 0
        if device is not None and device.type == "cuda":
            ops.status_watch(device).discard()
            value = ops.read_device_status_all(device, clear=True)
        words = [0] * self.world
        if self.world > 1:
            dist.all_gather_object(words, value, group=self.group)
        else:
            words = [value]
        total = 0
        for w in words:
            total |= int(w)
        if total & ops.FAILURE_BITS:
            if self._peer is not None:
                self._peer.reset()
            bad = [r for r, w in enumerate(words) if int(w) & ops.FAILURE_BITS]
            raise ops.DeviceFailure(total, f"ShardedDecoder (ranks {bad} flagged)")

    def close(self) -> None:
        """Checks the group for device failures (``check``) and releases the peer-exchange
        buffers; collective. The buffers are released even when the check raises."""
        try:
            self.check()
        finally:
            if self._peer is not None:
                self._peer.close()
                self._peer = None

    @property
    def world(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    @property
    def rank(self) -> int:
        return dist.get_rank(self.group) if dist.is_initialized() else 0

    def _send_buffer(self, n: int, device: torch.device) -> torch.Tensor:
        if self._send is None or self._send.numel() != n or self._send.device != device:
            self._send = torch.empty(n, dtype=torch.float32, device=device)
        return self._send

    def _local(self, query: torch.Tensor, local: PackedBatch, sm_scale: float) -> torch.Tensor:
        """Decodes ``query`` over ``local`` into the flat send row [out (QH*D) | lse (QH)]."""
        qh, d = query.shape
        send = self._send_buffer(qh * d + qh, query.device)
        out_v, lse_v = send[: qh * d].view(qh, d), send[qh * d :]
        if local.packed_k.shape[0] == 0:  # an empty shard: no weight in the merge
            out_v.zero_()
            lse_v.fill_(float("-inf"))
        elif self.decode_fn is None:
            from . import ops

            PackedBatch.validate(local, query)
            ops.decode(query, local.packed_k.contiguous(), local.packed_v.contiguous(),
                       local.scales_k.contiguous(), local.scales_v.contiguous(),
                       local.valid_tokens.to(torch.int32).contiguous(), local.bits,
                       local.group_size, sm_scale, out=out_v, lse=lse_v)
        else:
            out, lse = self.decode_fn(query, local, sm_scale)
            out_v.copy_(out)
            lse_v.copy_(lse)
        return send

    def _gather(self, send: torch.Tensor) -> torch.Tensor:
        world = self.world
        n = send.numel()
        if self._recv is None or self._recv.numel() != world * n or \
                self._recv.device != send.device:
            self._recv = torch.empty(world * n, dtype=send.dtype, device=send.device)
        if world == 1:
            self._recv.copy_(send)
        else:
            dist.all_gather_into_tensor(self._recv, send, group=self.group)
        return self._recv.view(world, n)

    def run(self, query: torch.Tensor, local: PackedBatch,
            sm_scale: float) -> tuple[torch.Tensor, torch.Tensor]:
        qh, d = query.shape
        self._device = query.device
        if self.mode == "heads":
            kvh_local = local.packed_k.shape[2]
            world = self.world
            if kvh_local * world * (qh // (kvh_local * world)) != qh:
                raise ValueError("query heads must be divisible by the sharded KV heads")
            _, _, q_lo, q_hi = head_shard(kvh_local * world, qh, self.rank, world)
            rows = q_hi - q_lo
            recv = self._gather(self._local(query[q_lo:q_hi].contiguous(), local, sm_scale))
            out_all = recv[:, : rows * d].reshape(world * rows, d)
            lse_all = recv[:, rows * d :].reshape(world * rows)
            return out_all.clone(), lse_all.clone()

        if self._use_peer(query, local):
            return self._run_peer(query, local, sm_scale)
        recv = self._gather(self._local(query, local, sm_scale))
        outs = recv[:, : qh * d].reshape(-1, qh, d).contiguous()
        lses = recv[:, qh * d :].contiguous()
        merge = self.merge_fn or _default_merge()
        return merge(outs, lses)

    def _run_peer(self, query: torch.Tensor, local: PackedBatch,
                  sm_scale: float) -> tuple[torch.Tensor, torch.Tensor]:
        from . import ops

        qh, d = query.shape
        if self._peer is None or (self._peer.query_heads, self._peer.head_dim) != (qh, d):
            if self._peer is not None:
                self._peer.close()
            self._peer = PeerExchange(self.group, query.device, qh, d)
        if self._peer_out is None or self._peer_out[0].shape != (qh, d):
            self._peer_out = (torch.empty((qh, d), dtype=torch.float32, device=query.device),
                              torch.empty((qh,), dtype=torch.float32, device=query.device))
        PackedBatch.validate(local, query)
        local = self._peer_operands(local)
        out, lse = self._peer_out
        return ops.decode_exchange(
            query, local.packed_k, local.packed_v, local.scales_k, local.scales_v,
            local.valid_tokens, local.bits, local.group_size,
            sm_scale, self._peer.rank, self._peer.world, self._peer.buffers, out=out, lse=lse)
