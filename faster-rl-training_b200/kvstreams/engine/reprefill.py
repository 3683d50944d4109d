"""Re-prefill baseline (engine/reprefill.py:1-35): after a compaction the sequence is
rebuilt from the retained tokens, renumbered from 0, and forwarded again."""

from __future__ import annotations

from ..utils.spans import Span, positions_to_spans
from .base import BaseEngine, _Run


class RePrefillEngine(BaseEngine):
    name = "reprefill"

    def _positions(self, run: _Run, idx: list[int]) -> list[int]:
        first = len(run.context)
        return list(range(first, first + len(idx)))

    def _evict(self, run: _Run, spans: list[Span]) -> list[Span]:
        current = run.context + run.pending
        dropped = [i for i in current if any(s <= i < e for s, e in spans)]
        if not dropped:
            return []
        gone = set(dropped)
        retained = [i for i in current if i not in gone]
        self.cache.free_sequence(run.seq_id)
        self.cache.add_sequence(run.seq_id)
        run.context, run.pending = [], []
        if retained:
            self._forward(run, retained, "reprefill")
        self._uncommit_tail(run)
        return positions_to_spans(dropped)
