"""Half-open integer spans [start, end) over the rollout stream (utils/spans.py:1-31)."""

from __future__ import annotations

from typing import Iterable

Span = tuple[int, int]


def merge_spans(spans: Iterable[Span]) -> list[Span]:
    """Sorted union of the non-empty spans; touching spans are joined (spans.py:10-18)."""
    cleaned = sorted((int(a), int(b)) for a, b in spans if b > a)
    merged: list[Span] = []
    for a, b in cleaned:
        if merged and a <= merged[-1][1]:
            if b > merged[-1][1]:
                merged[-1] = (merged[-1][0], b)
        else:
            merged.append((a, b))
    return merged


def positions_to_spans(positions: Iterable[int]) -> list[Span]:
    """Runs of consecutive integers as spans (spans.py:21-23)."""
    return merge_spans((int(p), int(p) + 1) for p in positions)


def span_length(spans: Iterable[Span]) -> int:
    return sum(b - a for a, b in spans)


def in_spans(position: int, spans: Iterable[Span]) -> bool:
    return any(a <= position < b for a, b in spans)
