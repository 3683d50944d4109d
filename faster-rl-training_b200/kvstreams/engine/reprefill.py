"""Re-prefill baseline (the comparison arm of the KV-streams paper, engine/reprefill.py:22-35 in
the reference): compaction drops the sequence's cache and forwards the retained tokens again,
renumbered from 0, so every compaction costs a prefill of the whole retained context."""

from __future__ import annotations

from ..utils.spans import Span, positions_to_spans, split_by_spans
from .base import BaseEngine, _Episode


class RePrefillEngine(BaseEngine):
    name = "reprefill"

    def _positions(self, ep: _Episode, idx: list[int]) -> list[int]:
        # the cache holds exactly ep.context, renumbered 0..len-1; new tokens follow it
        base = len(ep.context)
        return list(range(base, base + len(idx)))

    def _evict(self, ep: _Episode, spans: list[Span]):
        keep, gone = split_by_spans(ep.context + ep.pending, spans)
        if not gone:
            return [], None
        self.cache.free_sequence(ep.seq_id)
        self.cache.add_sequence(ep.seq_id)
        ep.context, ep.pending = [], []
        return positions_to_spans(gone), keep
