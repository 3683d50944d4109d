"""Compaction policies: which parts of a rollout stream to forget when the next turn would
overflow the context budget.

Each policy is one rule applied in a single pass over the rollout's segment table, in stream
order -- the same pass `compact_plan_kernel` (csrc/kvs_compact.cu) makes on the device for a
whole batch of rollouts, so a host decision and a device decision are the same function of the
table.  The rules are the reference's (compaction/policies.py:34-170): they decide which tokens a
rollout keeps, so token streams and compaction logs depend on them.

* turn rules (keep-recent, Markovian, summary): candidates are the segments that are alive,
  whole (not partially evicted) and unprotected, minus the ``keep_last`` most recent alive whole
  segments; keep-recent stops as soon as the overflow is freed, the others take every candidate;
* token window: one span from the end of the protected prompt to
  ``min(stream end - window, start of the last segment)``.

Spans arrive in stream order, so merging them (utils/spans.py:10-18) is a running merge.
A policy only decides *what* to evict; the engine decides *how* (KV-streams evicts in place).
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from typing import Optional, Sequence

from ..utils.spans import Span
from .segments import Segment


@dataclass
class CompactionPlan:
    """Spans to evict (merged, stream order), the segments they came from, and for the summary
    policy the request of the summary turn to run first."""

    spans: list[Span]
    segments: list[int] = field(default_factory=list)
    summary_request: Optional[str] = None
    reason: str = ""

    @property
    def empty(self) -> bool:
        return not self.spans and self.summary_request is None


def _append_merged(spans: list[Span], start: int, end: int) -> None:
    """Add ``[start, end)`` to spans built in stream order, joining it to the last one when they
    touch or overlap; empty ranges are dropped."""
    if end <= start:
        return
    if spans and start <= spans[-1][1]:
        if end > spans[-1][1]:
            spans[-1] = (spans[-1][0], end)
    else:
        spans.append((start, end))


def select_turns(segments: Sequence[Segment], keep_last: int,
                 overflow: Optional[int] = None) -> tuple[list[Span], list[int]]:
    """The turn rule in one pass: every alive, whole, unprotected segment older than the
    ``keep_last`` most recent alive whole segments, oldest first; with ``overflow`` the pass
    stops once that many tokens are chosen.  Returns (merged spans, segment indices)."""
    whole = sum(1 for seg in segments if seg.alive and not seg.partially_evicted)
    last_old = whole - keep_last  # ranks 1 .. last_old are older than the kept tail
    spans: list[Span] = []
    chosen: list[int] = []
    freed = 0
    rank = 0
    for seg in segments:
        if not seg.alive or seg.partially_evicted:
            continue
        rank += 1
        if rank > last_old or seg.protected:
            continue
        if overflow is not None and freed >= overflow:
            break
        chosen.append(seg.index)
        freed += seg.length
        _append_merged(spans, seg.start, seg.end)
    return spans, chosen


def select_window(segments: Sequence[Segment], window: int) -> tuple[list[Span], list[int]]:
    """The token-window rule: forget ``[prompt end, cut)`` with ``cut`` the smaller of
    ``stream end - window`` and the start of the last segment (so the latest turn stays whole);
    nothing when the cut does not pass the prompt.  Returns (spans, alive segments touched)."""
    if not segments:
        return [], []
    prompt_end = 0
    for seg in segments:
        if seg.protected and seg.end > prompt_end:
            prompt_end = seg.end
    last = segments[-1]
    cut = min(last.end - window, last.start)
    if cut <= prompt_end:
        return [], []
    touched = [seg.index for seg in segments if seg.alive and seg.start < cut and seg.end > prompt_end]
    return [(prompt_end, cut)], touched


class CompactionPolicy(ABC):
    """A rule choosing what to evict.  ``device_code`` / ``device_param`` name the same rule for
    the device plan kernel (None when it has no device form)."""

    name = "base"
    granularity = "turn"
    device_code: Optional[int] = None

    @abstractmethod
    def plan(self, segments: list[Segment], live_tokens: int, budget: int, required: int) -> CompactionPlan:
        """Spans to evict given the segments so far, the live KV entries, the soft budget and
        the entries the next turn needs (live + incoming + reserve)."""

    @property
    def device_param(self) -> int:
        raise ValueError(f"policy {self.name!r} has no device implementation")

    def __repr__(self) -> str:
        return f"{type(self).__name__}()"


class _TurnRule(CompactionPolicy):
    """Turn-granular rules: parameterised by how many recent segments always stay."""

    stop_at_overflow = False
    default_keep = 1

    def __init__(self, keep_last: Optional[int] = None) -> None:
        keep_last = self.default_keep if keep_last is None else int(keep_last)
        if keep_last < 1:
            raise ValueError("keep_last must be >= 1: the latest turn always stays live")
        self.keep_last = keep_last

    @property
    def device_param(self) -> int:
        return self.keep_last

    def _summary(self) -> Optional[str]:
        return None

    def plan(self, segments, live_tokens, budget, required) -> CompactionPlan:
        overflow = required - budget
        spans, chosen = select_turns(segments, self.keep_last, overflow if self.stop_at_overflow else None)
        why = f"{self.name}: overflow {overflow}, keep {self.keep_last}"
        return CompactionPlan(spans=spans, segments=chosen, summary_request=self._summary(), reason=why)

    def __repr__(self) -> str:
        return f"{type(self).__name__}(keep_last={self.keep_last})"


class KeepRecentTurns(_TurnRule):
    """Forget the oldest evictable turns, only as many as the overflow needs."""

    name = "keep_recent"
    device_code = 0
    stop_at_overflow = True
    default_keep = 2


class MarkovianPolicy(_TurnRule):
    """Keep the prompt and the ``keep_last`` latest turns; forget everything else at once."""

    name = "markovian"
    device_code = 1


class SummaryPolicy(_TurnRule):
    """Ask for a summary turn first, then forget every evictable turn before the kept tail."""

    name = "summary"
    device_code = 2

    def __init__(self, keep_last: int = 1, request: str = "summarize what matters") -> None:
        super().__init__(keep_last)
        self.request = request

    def _summary(self) -> Optional[str]:
        return self.request


class TokenSlidingWindow(CompactionPolicy):
    """Token-granular window: the prompt and the newest ``window`` tokens stay, never cutting
    into the latest turn."""

    name = "token_window"
    granularity = "token"
    device_code = 3

    def __init__(self, window: int = 128) -> None:
        self.window = int(window)

    @property
    def device_param(self) -> int:
        return self.window

    def plan(self, segments, live_tokens, budget, required) -> CompactionPlan:
        spans, touched = select_window(segments, self.window)
        return CompactionPlan(spans=spans, segments=touched, reason=f"token_window: window {self.window}")

    def __repr__(self) -> str:
        return f"TokenSlidingWindow(window={self.window})"


POLICIES = {cls.name: cls for cls in (KeepRecentTurns, MarkovianPolicy, SummaryPolicy, TokenSlidingWindow)}


def build_policy(name: str, **kwargs) -> CompactionPolicy:
    """A policy by its reference name (``keep_recent``, ``markovian``, ``summary``,
    ``token_window``) with its keyword arguments."""
    try:
        cls = POLICIES[name]
    except KeyError:
        raise ValueError(f"unknown policy {name!r}; choose from {sorted(POLICIES)}") from None
    return cls(**kwargs)
