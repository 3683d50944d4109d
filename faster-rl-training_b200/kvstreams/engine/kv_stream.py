"""KV-streams engine (engine/kv_stream.py:1-27): compaction in place on the live cache.

A token's RoPE position is its stream index, so retained keys keep their rotation
and new tokens continue the original counter; eviction drops whole blocks and joins
the block table on the device, and no retained token is ever forwarded twice.
"""

from __future__ import annotations

from ..utils.spans import Span, split_by_spans
from .base import BaseEngine, _Episode


class KVStreamEngine(BaseEngine):
    name = "kvstream"

    def _positions(self, ep: _Episode, idx: list[int]) -> list[int]:
        return list(idx)

    def _evict(self, ep: _Episode, spans: list[Span]):
        # the eviction and the cache's invariant check come back in one device round trip
        evicted = self.cache.evict_positions(ep.seq_id, spans, check=True)
        if evicted:
            ep.context = split_by_spans(ep.context, evicted)[0]
        return evicted, None
