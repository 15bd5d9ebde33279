"""Block-selection policies (API of src/kvssd/selectors.py:7-28).

A selector maps the sorted block ids of a layer to the ids that enter attention, in order.
The selected ids become the block table of the decode kernel.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol


class BlockSelector(Protocol):
    def select(self, available: list[int]) -> list[int]: ...


@dataclass(frozen=True)
class AllBlocks:
    def select(self, available: list[int]) -> list[int]:
        return list(available)


@dataclass(frozen=True)
class RecentSinkBlocks:
    """The first ``sink`` blocks plus the last ``recent`` blocks, order kept, no repeats."""

    sink: int = 1
    recent: int = 8

    def select(self, available: list[int]) -> list[int]:
        if self.sink < 0 or self.recent < 0:
            raise ValueError("sink and recent counts must be non-negative")
        head = list(available[: self.sink])
        tail = list(available[len(available) - self.recent :]) if self.recent else []
        if self.recent > len(available):
            tail = list(available)
        seen: set[int] = set()
        chosen = []
        for block in head + tail:
            if block not in seen:
                seen.add(block)
                chosen.append(block)
        return chosen
