"""Compaction policies: decide which stream spans to forget (policies.py:1-183).

A policy only chooses *what* to evict (whole turns by default, boundary tags
included); the engine decides *how* (KV-streams evicts in place).
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from typing import Optional

from ..utils.spans import Span, merge_spans
from .segments import Segment


@dataclass
class CompactionPlan:
    spans: list[Span]
    segments: list[int] = field(default_factory=list)
    summary_request: Optional[str] = None
    reason: str = ""

    @property
    def empty(self) -> bool:
        return not self.spans and self.summary_request is None


def _evictable(segments: list[Segment], keep_last: int) -> list[Segment]:
    """Live, unprotected, fully-alive segments other than the ``keep_last`` newest live ones
    (policies.py:34-38)."""
    live = [s for s in segments if s.alive and not s.partially_evicted]
    newest = {s.index for s in live[-keep_last:]} if keep_last > 0 else set()
    return [s for s in live if not s.protected and s.index not in newest]


class CompactionPolicy(ABC):
    name = "base"
    granularity = "turn"

    @abstractmethod
    def plan(self, segments: list[Segment], live_tokens: int, budget: int, required: int) -> CompactionPlan:
        """Spans to evict given the segments so far, the live KV entries, the soft budget and
        the entries the next turn needs (live + incoming + reserve)."""

    def __repr__(self) -> str:
        return f"{type(self).__name__}()"


class KeepRecentTurns(CompactionPolicy):
    """Drop the oldest evictable turns until the overflow is covered (policies.py:62-88)."""

    name = "keep_recent"

    def __init__(self, keep_last: int = 2) -> None:
        if keep_last < 1:
            raise ValueError("keep_last must be >= 1 (the latest turn must stay live)")
        self.keep_last = keep_last

    def plan(self, segments, live_tokens, budget, required) -> CompactionPlan:
        overflow = required - budget
        picked: list[Segment] = []
        freed = 0
        for seg in _evictable(segments, self.keep_last):
            if freed >= overflow:
                break
            picked.append(seg)
            freed += seg.length
        return CompactionPlan(
            spans=merge_spans(s.span for s in picked),
            segments=[s.index for s in picked],
            reason=f"overflow={overflow}",
        )

    def __repr__(self) -> str:
        return f"KeepRecentTurns(keep_last={self.keep_last})"


class MarkovianPolicy(CompactionPolicy):
    """Keep the prompt and only the last ``keep_last`` turns (policies.py:91-113)."""

    name = "markovian"

    def __init__(self, keep_last: int = 1) -> None:
        if keep_last < 1:
            raise ValueError("keep_last must be >= 1")
        self.keep_last = keep_last

    def plan(self, segments, live_tokens, budget, required) -> CompactionPlan:
        picked = _evictable(segments, self.keep_last)
        return CompactionPlan(
            spans=merge_spans(s.span for s in picked),
            segments=[s.index for s in picked],
            reason="markovian reset",
        )

    def __repr__(self) -> str:
        return f"MarkovianPolicy(keep_last={self.keep_last})"


class SummaryPolicy(CompactionPolicy):
    """Request a summary turn, then drop all older evictable turns (policies.py:116-137)."""

    name = "summary"

    def __init__(self, keep_last: int = 1, request: str = "summarize what matters") -> None:
        if keep_last < 1:
            raise ValueError("keep_last must be >= 1")
        self.keep_last = keep_last
        self.request = request

    def plan(self, segments, live_tokens, budget, required) -> CompactionPlan:
        picked = _evictable(segments, self.keep_last)
        return CompactionPlan(
            spans=merge_spans(s.span for s in picked),
            segments=[s.index for s in picked],
            summary_request=self.request,
            reason="summarize then evict",
        )

    def __repr__(self) -> str:
        return f"SummaryPolicy(keep_last={self.keep_last})"


class TokenSlidingWindow(CompactionPolicy):
    """Token-level window: keep the prompt and the newest ``window`` tokens, never cutting into
    the latest turn (policies.py:140-167)."""

    name = "token_window"
    granularity = "token"

    def __init__(self, window: int = 128) -> None:
        self.window = window

    def plan(self, segments, live_tokens, budget, required) -> CompactionPlan:
        if not segments:
            return CompactionPlan(spans=[])
        prompt_end = max((s.end for s in segments if s.protected), default=0)
        cut = min(segments[-1].end - self.window, segments[-1].start)
        if cut <= prompt_end:
            return CompactionPlan(spans=[])
        touched = [s.index for s in segments if s.alive and s.start < cut and s.end > prompt_end]
        return CompactionPlan(spans=[(prompt_end, cut)], segments=touched, reason="sliding window")

    def __repr__(self) -> str:
        return f"TokenSlidingWindow(window={self.window})"


POLICIES = {
    "keep_recent": KeepRecentTurns,
    "markovian": MarkovianPolicy,
    "summary": SummaryPolicy,
    "token_window": TokenSlidingWindow,
}


def build_policy(name: str, **kwargs) -> CompactionPolicy:
    if name not in POLICIES:
        raise ValueError(f"unknown policy {name!r}; choose from {sorted(POLICIES)}")
    return POLICIES[name](**kwargs)
