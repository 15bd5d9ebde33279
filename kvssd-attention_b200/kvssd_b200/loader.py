"""Bounded asynchronous record reader (API of src/kvssd/loader.py:22-137).

``depth`` reader threads pread whole records into ``depth`` reusable (optionally pinned)
host slots; a slot is handed back to the pool only after the consumer is done with it, so
memory stays bounded and a recycled slot can never alias a block still in use.
"""

from __future__ import annotations

from collections.abc import Iterator
from concurrent.futures import Future, ThreadPoolExecutor
from queue import Queue

import torch

from .format import PackedKVBlock, decode_record
from .quant import QuantizedTensor


class AsyncBlockLoader:
    def __init__(self, store, depth: int = 2, pinned: bool = True, device: torch.device | None = None):
        if depth < 1:
            raise ValueError("depth must be positive")
        del device  # slots are host buffers; staging to the device is the pipeline's job
        self.store = store
        self.depth = depth
        self.executor = ThreadPoolExecutor(max_workers=depth, thread_name_prefix="kvssd-io")
        self.free: Queue[torch.Tensor] = Queue()
        pin = pinned and torch.cuda.is_available()
        for _ in range(depth):
            self.free.put(torch.empty(store.spec.record_bytes, dtype=torch.uint8, pin_memory=pin))

    def iter_records(self, layer: int, block_ids: list[int],
                     verify_crc: bool = True) -> Iterator[PackedKVBlock]:
        """Yields blocks whose payloads VIEW a slot; valid until the next iteration step."""
        pending: list[tuple[torch.Tensor, Future[None]]] = []
        source = iter(block_ids)

        def submit(block_id: int) -> None:
            slot = self.free.get()
            entry = self.store.entry(layer, block_id)
            pending.append((slot, self.executor.submit(self.store.read_into, entry, slot)))

        for block_id in source:
            submit(block_id)
            if len(pending) == self.depth:
                break
        try:
            while pending:
                slot, future = pending[0]
                future.result()
                block = decode_record(slot, self.store.spec, verify_crc)
                yield block
                pending.pop(0)
                self.free.put(slot)
                nxt = next(source, None)
                if nxt is not None:
                    submit(nxt)
        finally:
            for slot, future in pending:  # consumer stopped early: drain and recycle
                try:
                    future.result()
                finally:
                    self.free.put(slot)

    def iter_blocks(self, layer: int, block_ids: list[int]) -> Iterator[PackedKVBlock]:
        """Yields blocks with payloads copied out of the slot (safe to keep)."""
        for b in self.iter_records(layer, block_ids):
            yield PackedKVBlock(
                b.layer, b.block, b.valid_tokens,
                QuantizedTensor(b.key.packed.clone(), b.key.scales.clone(),
                                b.key.original_shape, b.key.bits, b.key.group_size),
                QuantizedTensor(b.value.packed.clone(), b.value.scales.clone(),
                                b.value.original_shape, b.value.bits, b.value.group_size),
            )

    def close(self) -> None:
        self.executor.shutdown(wait=True, cancel_futures=False)

    def __enter__(self) -> "AsyncBlockLoader":
        return self

    def __exit__(self, *_: object) -> None:
        self.close()
