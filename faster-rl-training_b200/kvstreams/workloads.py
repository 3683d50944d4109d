"""Seeded synthetic workloads with the shapes of the benchmark configurations.

* :func:`compaction_plan` -- many streams whose block tables are built from turns of
  geometric length padded to the block size, then 1-8 keep-recent compaction
  events per stream (prompt pinned, keep_last ~ U[1, 4]).
* :func:`decode_state` -- paged decode microbench state: per-stream live context
  ~U[lo, hi] tokens in blocks drawn from a random permutation of the pool, with
  1-6 evicted whole-block spans per stream so logical positions have gaps.
* :func:`replay_evicted_at` -- evicted_at rows of long streams from keep-recent
  eviction of geometric-length turns with 3-8 events.

Everything is host-side numpy; the caller moves what it needs to the device.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

NEVER = np.iinfo(np.int64).max


def _turn_lengths(rng, total: int, mean: float, bs: int, first: int = 0) -> list[int]:
    """Turn lengths ~Geometric(mean) rounded up to a multiple of ``bs`` until ``total``."""
    out = []
    acc = 0
    if first:
        out.append(first)
        acc = first
    while acc < total:
        n = int(rng.geometric(1.0 / mean))
        n = -(-n // bs) * bs
        n = min(n, total - acc) if total - acc >= bs else total - acc
        out.append(n)
        acc += n
    return out


@dataclass
class CompactionRound:
    """Work of one round: appends (then) one batched eviction over ``evict_seqs``."""

    append_seqs: list[int] = field(default_factory=list)
    append_positions: list[np.ndarray] = field(default_factory=list)
    evict_seqs: list[int] = field(default_factory=list)
    evict_spans: list[list[tuple[int, int]]] = field(default_factory=list)


def compaction_plan(num_streams: int = 256, blocks_per_stream: int = 512, block_size: int = 16,
                    num_events_range=(1, 8), mean_turn: float = 96.0, keep_last_range=(1, 4),
                    seed: int = 0) -> list[CompactionRound]:
    """Rounds of batched appends and evictions.  Round 0 fills every stream to
    ``blocks_per_stream`` blocks (streams interleaved turn by turn, so block ids
    are scattered over the pool); each later round evicts keep-recent turn spans in
    the streams that have an event left, then appends fresh turns to refill them."""
    rng = np.random.default_rng(seed)
    bs = block_size
    target = blocks_per_stream * bs
    turns: list[list[tuple[int, int]]] = [[] for _ in range(num_streams)]
    alive: list[list[bool]] = [[] for _ in range(num_streams)]
    next_pos = [0] * num_streams
    rounds: list[CompactionRound] = []
    # fill: interleave turn-sized appends across streams
    plans = [_turn_lengths(rng, target, mean_turn, bs, first=2 * bs) for _ in range(num_streams)]
    r0 = CompactionRound()
    depth = max(len(p) for p in plans)
    for k in range(depth):
        for s in range(num_streams):
            if k < len(plans[s]):
                n = plans[s][k]
                a = next_pos[s]
                r0.append_seqs.append(s)
                r0.append_positions.append(np.arange(a, a + n, dtype=np.int64))
                turns[s].append((a, a + n))
                alive[s].append(True)
                next_pos[s] = a + n
    rounds.append(r0)
    n_events = rng.integers(num_events_range[0], num_events_range[1] + 1, size=num_streams)
    for e in range(int(n_events.max())):
        rd = CompactionRound()
        for s in range(num_streams):
            if e >= n_events[s]:
                continue
            keep = int(rng.integers(keep_last_range[0], keep_last_range[1] + 1))
            live_idx = [i for i, a in enumerate(alive[s]) if a]
            evictable = [i for i in live_idx[:-keep] if i != 0]  # turn 0 = pinned prompt
            if not evictable:
                continue
            spans = [turns[s][i] for i in evictable]
            if rng.random() < 0.25:  # an unaligned request, shrunk to whole blocks by the cache
                a, b = spans[0]
                spans[0] = (a + int(rng.integers(1, bs)) if bs > 1 else a, b)
            for i in evictable:
                alive[s][i] = False
            rd.evict_seqs.append(s)
            rd.evict_spans.append(spans)
            # refill with new turns
            freed = sum(b - a for a, b in (turns[s][i] for i in evictable))
            for n in _turn_lengths(rng, freed, mean_turn, bs):
                a = next_pos[s]
                rd.append_seqs.append(s)
                rd.append_positions.append(np.arange(a, a + n, dtype=np.int64))
                turns[s].append((a, a + n))
                alive[s].append(True)
                next_pos[s] = a + n
        rounds.append(rd)
    return rounds


@dataclass
class DecodeState:
    block_size: int
    num_blocks: int
    tables: list[np.ndarray]  # per stream block ids
    positions: list[np.ndarray]  # per stream logical positions of live entries (strictly increasing)
    next_positions: np.ndarray  # [S] position of the token each stream decodes next
    free_list: np.ndarray  # remaining blocks, bottom to top

    @property
    def lengths(self) -> np.ndarray:
        return np.asarray([p.size for p in self.positions], dtype=np.int64)


def decode_state(num_streams: int = 64, ctx_range=(1024, 16384), block_size: int = 16, num_blocks: int = 131072,
                 evicted_spans_range=(1, 6), seed: int = 0) -> DecodeState:
    """Live context ~U[ctx_range] per stream; blocks from a random permutation of the pool;
    1-6 evicted whole-block spans per stream leave gaps in the logical positions."""
    rng = np.random.default_rng(seed)
    bs = block_size
    perm = rng.permutation(num_blocks).astype(np.int32)
    cursor = 0
    tables, positions = [], []
    nxt = np.zeros(num_streams, dtype=np.int64)
    for s in range(num_streams):
        ctx = int(rng.integers(ctx_range[0], ctx_range[1] + 1))
        nb = -(-ctx // bs)
        tables.append(perm[cursor:cursor + nb].copy())
        cursor += nb
        # logical positions: ctx live tokens with 1-6 evicted gaps of whole blocks
        n_gaps = int(rng.integers(evicted_spans_range[0], evicted_spans_range[1] + 1))
        full_blocks = ctx // bs
        cuts = np.sort(rng.choice(np.arange(1, max(full_blocks, 2)), size=min(n_gaps, max(full_blocks - 1, 1)),
                                  replace=False))
        gap_blocks = rng.integers(1, 9, size=cuts.size)
        pos = np.arange(ctx, dtype=np.int64)
        for c, g in zip(cuts, gap_blocks):
            pos[c * bs:] += int(g) * bs
        positions.append(pos)
        nxt[s] = pos[-1] + 1
    free_list = perm[cursor:][::-1].copy()
    return DecodeState(bs, num_blocks, tables, positions, nxt, free_list)


def replay_evicted_at(batch: int = 16, seq_len: int = 32768, events_range=(3, 8), mean_turn: float = 96.0,
                      keep_last_range=(1, 4), block_size: int = 16, seed: int = 0):
    """``[B, T]`` evicted_at and the (start, end, time) triples of every stream."""
    rng = np.random.default_rng(seed)
    T = seq_len
    out = np.full((batch, T), NEVER, dtype=np.int64)
    all_triples = []
    for b in range(batch):
        lens = _turn_lengths(rng, T, mean_turn, block_size, first=2 * block_size)
        bounds = np.cumsum([0] + lens)
        n_turns = len(lens)
        n_ev = int(rng.integers(events_range[0], events_range[1] + 1))
        ev_turns = np.sort(rng.choice(np.arange(2, n_turns), size=min(n_ev, n_turns - 2), replace=False))
        alive = [True] * n_turns
        triples = []
        for et in ev_turns:
            time = int(bounds[et])  # the event happens before turn et is forwarded
            keep = int(rng.integers(keep_last_range[0], keep_last_range[1] + 1))
            live = [i for i in range(et) if alive[i]]
            for i in [i for i in live[:-keep] if i != 0]:
                alive[i] = False
                triples.append((int(bounds[i]), int(bounds[i + 1]), time))
        for s, e, t in triples:
            out[b, s:e] = np.minimum(out[b, s:e], t)
        all_triples.append(np.asarray(triples, dtype=np.int64).reshape(-1, 3))
    return out, all_triples


def visible_pairs(evicted_at: np.ndarray, lengths=None) -> int:
    """nnz of the replay mask summed over streams: sum_s (min(evicted_at[s], L) - s)."""
    B, T = evicted_at.shape
    total = 0
    for b in range(B):
        L = T if lengths is None else int(lengths[b])
        e = np.minimum(evicted_at[b, :L], L)
        total += int((e - np.arange(L)).sum())
        total += T - L  # padded rows see themselves
    return total
