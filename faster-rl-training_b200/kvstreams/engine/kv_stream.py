"""KV-streams engine (engine/kv_stream.py:1-27): compaction in place on the live cache.

A token's RoPE position is its stream index, so retained keys keep their rotation
and new tokens continue the original counter; eviction drops whole blocks and joins
the block table on the device, and no retained token is ever forwarded twice.
"""

from __future__ import annotations

from ..utils.spans import Span, in_spans
from .base import BaseEngine, _Episode


class KVStreamEngine(BaseEngine):
    name = "kvstream"

    def _positions(self, ep: _Episode, idx: list[int]) -> list[int]:
        return list(idx)

    def _evict(self, ep: _Episode, spans: list[Span]):
        evicted = self.cache.evict_positions(ep.seq_id, spans)
        if evicted:
            ep.context = [i for i in ep.context if not in_spans(i, evicted)]
            self.cache.check_invariants(ep.seq_id)
        return evicted, None
