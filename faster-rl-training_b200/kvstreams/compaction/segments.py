"""Segments: contiguous stream ranges the compaction policies reason about (segments.py:10-43)."""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Optional


@dataclass
class Segment:
    """``[start, end)`` of the stream: the prompt (protected), a turn, or a summary turn.

    ``evicted_at`` is the stream length at the compaction that removed the whole
    segment (None while any of it is live).
    """

    index: int
    kind: str
    start: int
    end: int
    protected: bool = False
    evicted_at: Optional[int] = None
    partially_evicted: bool = False

    @property
    def length(self) -> int:
        return self.end - self.start

    @property
    def alive(self) -> bool:
        return self.evicted_at is None

    @property
    def span(self) -> tuple[int, int]:
        return (self.start, self.end)

    def to_dict(self) -> dict:
        return asdict(self)
