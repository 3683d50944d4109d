"""KV-streams engine (engine/kv_stream.py:1-27): compaction in place on the live cache.

A token's RoPE position is its stream index, so retained keys keep their rotation
and new tokens continue the original counter; eviction drops whole blocks and joins
the block table on the device, and no retained token is ever forwarded twice.
"""

from __future__ import annotations

from ..utils.spans import Span
from .base import BaseEngine, _Run


class KVStreamEngine(BaseEngine):
    name = "kvstream"

    def _positions(self, run: _Run, idx: list[int]) -> list[int]:
        return list(idx)

    def _evict(self, run: _Run, spans: list[Span]) -> list[Span]:
        evicted = self.cache.evict_positions(run.seq_id, spans)
        if evicted:
            run.context = [i for i in run.context if not any(s <= i < e for s, e in evicted)]
            self.cache.check_invariants(run.seq_id)
        return evicted
