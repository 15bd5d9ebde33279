"""Attention-backend lookup with kvssd's registry API (src/kvssd/backends/registry.py:23-68).

This package ships exactly one implementation, the B200 kernels under kvssd's name ``cuda``;
it has no CPU or portable attention path. The lookup is therefore a small table of factories
in registration order with ``cuda`` first:

* ``auto`` takes the first registered backend whose probe reports it available on the
  device, and fails closed (RuntimeError) when none is -- on a CPU device that is always the
  case unless the caller registered a CPU backend of their own;
* an explicit name returns that backend or raises RuntimeError with its probe's reason;
* an unknown name raises ValueError listing the names that exist;
* a backend instance is probed and returned as is.

The error types and messages are kvssd's, so callers catch the same exceptions.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from .base import AttentionBackend, BackendAvailability
from .cuda import B200AttentionBackend

BackendFactory = Callable[[], AttentionBackend]


class _BackendTable:
    """Name -> factory, in registration order (``cuda`` is registered at import)."""

    def __init__(self) -> None:
        self._factories: dict[str, BackendFactory] = {}

    @staticmethod
    def key(name: str) -> str:
        return name.strip().lower()

    def add(self, name: str, factory: BackendFactory) -> None:
        key = self.key(name)
        if key in ("", "auto"):
            raise ValueError("backend name must be non-empty and cannot be 'auto'")
        self._factories[key] = factory

    def names(self) -> list[str]:
        return list(self._factories)

    def make(self, key: str) -> AttentionBackend:
        factory = self._factories.get(key)
        if factory is None:
            listed = ", ".join(["auto", *self._factories])
            raise ValueError(f"unknown attention backend '{key}'; choose one of: {listed}")
        return factory()

    def first_available(self, device: torch.device) -> AttentionBackend:
        for key in self._factories:
            candidate = self._factories[key]()
            if candidate.probe(device).available:
                return candidate
        raise RuntimeError(f"no attention backend is available for {device}")


_table = _BackendTable()
_table.add("cuda", B200AttentionBackend)


def _usable(backend: AttentionBackend, device: torch.device, name: str | None = None):
    state = backend.probe(device)
    if not state.available:
        raise RuntimeError(f"attention backend '{name or state.name}' unavailable: {state.reason}")
    return backend


def register_attention_backend(name: str, factory: BackendFactory) -> None:
    """Adds (or replaces) a backend under ``name`` (case-insensitive, not 'auto')."""
    _table.add(name, factory)


def available_attention_backends(device: str | torch.device) -> list[BackendAvailability]:
    """The probe result of every registered backend on ``device``."""
    device = torch.device(device)
    return [_table.make(key).probe(device) for key in _table.names()]


def resolve_attention_backend(
    requested: str | AttentionBackend | None,
    device: str | torch.device,
) -> AttentionBackend:
    """The backend to run on ``device``: an instance, a registered name, or ``auto``/None."""
    device = torch.device(device)
    if requested is not None and not isinstance(requested, str):
        return _usable(requested, device)
    key = _table.key(requested or "auto")
    if key == "auto":
        return _table.first_available(device)
    return _usable(_table.make(key), device, key)
