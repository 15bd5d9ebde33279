"""Attention-backend lookup with kvssd's registry API (src/kvssd/backends/registry.py:23-68).

This package ships exactly one implementation, the B200 kernels under kvssd's name ``cuda``;
it has no CPU or portable attention path. The lookup is a name table (kvssd_b200._registry)
in registration order with ``cuda`` first, every entry open to ``auto``:

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

from .._registry import FactoryTable
from .base import AttentionBackend, BackendAvailability
from .cuda import B200AttentionBackend

BackendFactory = Callable[[], AttentionBackend]

_table = FactoryTable("attention")
_table.add("cuda", B200AttentionBackend, auto=True)


def register_attention_backend(name: str, factory: BackendFactory) -> None:
    """Adds (or replaces) a backend under ``name`` (case-insensitive, not 'auto'); ``auto``
    considers it after the backends registered before it."""
    _table.add(name, factory, auto=True)


def available_attention_backends(device: str | torch.device) -> list[BackendAvailability]:
    """The probe result of every registered backend on ``device``."""
    device = torch.device(device)
    return [_table.factory(key)().probe(device) for key in _table.names()]


def resolve_attention_backend(
    requested: str | AttentionBackend | None,
    device: str | torch.device,
) -> AttentionBackend:
    """The backend to run on ``device``: an instance, a registered name, or ``auto``/None."""
    device = torch.device(device)
    return _table.resolve(requested, lambda factory: factory(),
                          lambda backend: backend.probe(device), device)
