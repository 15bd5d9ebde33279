"""Attention backend contract and the B200 ``cuda`` backend."""

from .base import AttentionBackend, BackendAvailability, PackedBatch
from .cuda import B200AttentionBackend
from .registry import (
    available_attention_backends,
    register_attention_backend,
    resolve_attention_backend,
)

__all__ = [
    "AttentionBackend",
    "B200AttentionBackend",
    "BackendAvailability",
    "PackedBatch",
    "available_attention_backends",
    "register_attention_backend",
    "resolve_attention_backend",
]
