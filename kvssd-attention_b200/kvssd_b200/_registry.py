"""The name table behind both plug-in registries of this package: attention backends
(backends/registry.py, with the API of kvssd's src/kvssd/backends/registry.py:23-68) and record
storage backends (storage.py, with the API of src/kvssd/storage/registry.py:15-68).

A table holds factories under case-insensitive names, in registration order, each marked
whether ``auto`` may pick it. The caller says how to build an instance from a factory and how
to probe it (an attention backend probes a device, a storage backend its file), so one lookup
serves both kinds. The exception types and messages are kvssd's, so code written against kvssd
catches the same errors.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any


class FactoryTable:
    """Backend factories of one kind ("attention" or "storage", as the messages name it)."""

    def __init__(self, kind: str) -> None:
        self.kind = kind
        self._entries: dict[str, tuple[Callable[..., Any], bool]] = {}  # key -> (factory, auto)

    @staticmethod
    def key(name: str) -> str:
        return name.strip().lower()

    def add(self, name: str, factory: Callable[..., Any], auto: bool | None = None) -> None:
        """Registers ``factory`` under ``name``. A name registered again keeps its place in the
        order and, unless ``auto`` is given, whether ``auto`` picks it; a new name is not
        picked by ``auto`` unless ``auto`` is true."""
        key = self.key(name)
        if key in ("", "auto"):
            raise ValueError("backend name must be non-empty and cannot be 'auto'")
        if auto is None:
            auto = self._entries.get(key, (factory, False))[1]
        self._entries[key] = (factory, auto)

    def names(self) -> list[str]:
        return list(self._entries)

    def factory(self, key: str) -> Callable[..., Any]:
        entry = self._entries.get(key)
        if entry is None:
            listed = ", ".join(["auto", *self._entries])
            raise ValueError(f"unknown {self.kind} backend '{key}'; choose one of: {listed}")
        return entry[0]

    def resolve(self, requested: Any, make: Callable[[Callable[..., Any]], Any],
                probe: Callable[[Any], Any], where: object,
                release: Callable[[Any], None] | None = None) -> Any:
        """The backend for ``requested``:

        * an instance is probed and returned as it is;
        * a registered name is built and probed;
        * ``auto`` (or None) builds the ``auto`` entries in registration order and returns the
          first whose probe reports it available.

        An unavailable choice raises RuntimeError with its probe's reason (``where``, the
        device or file, names the target when no ``auto`` entry is available); an unknown name
        raises ValueError. Instances built here and not returned are passed to ``release``.
        """
        if requested is not None and not isinstance(requested, str):
            return self._usable(requested, probe(requested), None, None)
        key = self.key(requested or "auto")
        if key != "auto":
            backend = make(self.factory(key))
            return self._usable(backend, probe(backend), key, release)
        for factory, auto in self._entries.values():
            if not auto:
                continue
            backend = make(factory)
            if probe(backend).available:
                return backend
            if release is not None:
                release(backend)
        raise RuntimeError(f"no {self.kind} backend is available for {where}")

    def _usable(self, backend: Any, state: Any, key: str | None,
                release: Callable[[Any], None] | None) -> Any:
        if state.available:
            return backend
        if release is not None:
            release(backend)
        raise RuntimeError(f"{self.kind} backend '{key or state.name}' unavailable: "
                           f"{state.reason}")
