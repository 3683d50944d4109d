"""Half-open integer spans [start, end) over the rollout stream (utils/spans.py:1-31)."""

from __future__ import annotations

from bisect import bisect_right
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


def split_by_spans(positions: Iterable[int], spans: Iterable[Span]) -> tuple[list[int], list[int]]:
    """(positions in none of the spans, positions in one), each in the given order: a binary
    search per position over the merged spans instead of a scan of every span."""
    merged = merge_spans(spans)
    starts = [a for a, _ in merged]
    outside: list[int] = []
    inside: list[int] = []
    for p in positions:
        j = bisect_right(starts, p) - 1
        (inside if j >= 0 and p < merged[j][1] else outside).append(p)
    return outside, inside
