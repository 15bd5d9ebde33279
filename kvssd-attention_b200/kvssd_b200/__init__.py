"""kvssd_b200: B200-native fused dequantize + decode attention behind kvssd's Python API.

Mirrors the public surface of kvssd (src/kvssd/__init__.py) for the decode path: CacheSpec and
the KVCacheStore record format, AllBlocks / RecentSinkBlocks selectors, the attention backend
contract with a ``cuda`` backend, packed_attention, merge_attention_chunks and
KVSSDPipeline.decode(query, layer, selector). All attention math runs in libkvssd_b200
(hand-written sm_100a CUDA, C ABI in include/kvssd_b200.h); there is no CPU attention path.
"""

from .attention import (
    fused_attention_tensors,
    merge_attention_chunks,
    merge_attention_chunks_n,
    packed_attention,
    stack_blocks,
)
from .backends import (
    B200AttentionBackend,
    PackedBatch,
    available_attention_backends,
    register_attention_backend,
    resolve_attention_backend,
)
from .format import CacheSpec
from .pipeline import KVSSDPipeline
from .pool import DeviceBlockPool
from .quant import dequantize_tensor, quantize_tensor
from .selectors import AllBlocks, RecentSinkBlocks
from .storage import (
    GDSStorageBackend,
    StorageAvailability,
    StorageBackend,
    available_storage_backends,
    register_storage_backend,
    resolve_storage_backend,
)
from .store import KVCacheStore

__all__ = [
    "AllBlocks",
    "B200AttentionBackend",
    "CacheSpec",
    "DeviceBlockPool",
    "GDSStorageBackend",
    "KVCacheStore",
    "KVSSDPipeline",
    "PackedBatch",
    "RecentSinkBlocks",
    "StorageAvailability",
    "StorageBackend",
    "available_storage_backends",
    "available_attention_backends",
    "dequantize_tensor",
    "fused_attention_tensors",
    "merge_attention_chunks",
    "merge_attention_chunks_n",
    "packed_attention",
    "quantize_tensor",
    "register_attention_backend",
    "register_storage_backend",
    "resolve_attention_backend",
    "resolve_storage_backend",
    "stack_blocks",
]
