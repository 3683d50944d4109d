"""CPU oracle of the KV-streams paged-KV path -- TEST INFRASTRUCTURE ONLY.

A plain numpy / Python restatement of the reference algorithms
(thanhauco/faster-RL-training, package kvstreams 0.2.0).  Only the tests,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
this module, and only as the expected result (or the timed CPU baseline); the product
(the ``kvstreams`` package and libkvs_b200.so) never calls it.

Pinned against golden vectors produced by running the reference itself
(tests/golden/make_golden.py, fixtures in tests/golden/) -- see
tests/test_oracle_golden.py.

Sections:
  * OracleCache -- BlockAllocator + PagedKVCache metadata (paged_cache.py:32-273)
  * evicted_at -- CompactionLog.evicted_at (compaction/events.py:66-74)
  * merge_spans / positions_to_spans (utils/spans.py:10-23)
  * rope_* -- RotaryEmbedding + apply_rope (rope.py:21-46)
  * gqa_attention / replay_attention / replay_attention_rows -- Attention.forward math
    (model.py:50-75) with the KV-streams mask (training/replay.py:55-63, collate :132-149)
  * tinylm_forward -- TinyLM.forward (model.py:132-157) for small models
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

NEVER = np.iinfo(np.int64).max


# ---------------------------------------------------------------------- spans
def merge_spans(spans):
    """utils/spans.py:10-18 -- sorted union; touching spans join."""
    out = []
    for s, e in sorted((int(s), int(e)) for s, e in spans if e > s):
        if out and s <= out[-1][1]:
            out[-1][1] = max(out[-1][1], e)
        else:
            out.append([s, e])
    return [(s, e) for s, e in out]


def positions_to_spans(positions):
    """utils/spans.py:21-23."""
    return merge_spans((p, p + 1) for p in positions)


# ---------------------------------------------------------------------- cache
class OutOfBlocksError(RuntimeError):
    pass


@dataclass
class OracleStats:
    """paged_cache.py:70-78 (CacheStats)."""

    written_tokens: int = 0
    evicted_tokens: int = 0
    evicted_blocks: int = 0
    truncated_tokens: int = 0
    peak_blocks: int = 0
    eviction_calls: int = 0
    shrunk_tokens: int = 0

    def as_list(self):
        return [self.written_tokens, self.evicted_tokens, self.evicted_blocks, self.truncated_tokens,
                self.peak_blocks, self.eviction_calls, self.shrunk_tokens]


class OracleCache:
    """Metadata of PagedKVCache (paged_cache.py:81-273) without the K/V pool.

    ``free`` is the reference allocator's ``_free`` list (paged_cache.py:37): the
    next block handed out is ``free[-1]``; freed blocks are appended.
    """

    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.free = list(range(num_blocks - 1, -1, -1))  # paged_cache.py:37
        self.used: set[int] = set()
        self.slot_pos = np.full((num_blocks, block_size), -1, dtype=np.int64)  # :100-102
        self.tables: dict[int, list[int]] = {}
        self.lengths: dict[int, int] = {}
        self.stats = OracleStats()

    def load(self, tables, positions, free_list) -> None:
        """Install tables / live positions / free list directly (sequence ids 0..n-1)."""
        bs = self.block_size
        self.free = [int(b) for b in free_list]
        for sid, (tab, pos) in enumerate(zip(tables, positions)):
            self.tables[sid] = [int(b) for b in tab]
            self.lengths[sid] = len(pos)
            self.used.update(self.tables[sid])
            for i, p in enumerate(pos):
                self.slot_pos[self.tables[sid][i // bs], i % bs] = int(p)
        self.stats.peak_blocks = max(self.stats.peak_blocks, len(self.used))

    # allocator (paged_cache.py:40-51)
    def _allocate(self) -> int:
        if not self.free:
            raise OutOfBlocksError(f"all {self.num_blocks} KV blocks are in use")
        b = self.free.pop()
        self.used.add(b)
        return b

    def _release(self, b: int) -> None:
        if b not in self.used:
            raise ValueError(f"double free of block {b}")
        self.used.remove(b)
        self.free.append(b)

    # sequences (paged_cache.py:123-142)
    def add_sequence(self, sid: int) -> None:
        if sid in self.tables:
            raise ValueError(f"sequence {sid} already exists")
        self.tables[sid] = []
        self.lengths[sid] = 0

    def free_sequence(self, sid: int) -> None:
        for b in self.tables.pop(sid, []):
            self.slot_pos[b] = -1
            self._release(b)
        self.lengths.pop(sid, None)

    # append (paged_cache.py:145-165)
    def append_slots(self, sid: int, positions):
        table = self.tables[sid]
        n = self.lengths[sid]
        bs = self.block_size
        blocks, offsets = [], []
        for i in range(len(positions)):
            b, o = divmod(n + i, bs)
            if b == len(table):
                table.append(self._allocate())
            blocks.append(table[b])
            offsets.append(o)
        for b, o, p in zip(blocks, offsets, positions):
            self.slot_pos[b, o] = int(p)
        self.lengths[sid] = n + len(positions)
        self.stats.written_tokens += len(positions)
        self.stats.peak_blocks = max(self.stats.peak_blocks, len(self.used))
        return blocks, offsets

    def positions(self, sid: int) -> np.ndarray:
        """paged_cache.py:184-188."""
        n = self.lengths[sid]
        t = self.tables[sid]
        if not t:
            return np.zeros(0, dtype=np.int64)
        return self.slot_pos[np.asarray(t)].reshape(-1)[:n].copy()

    # eviction (paged_cache.py:190-240)
    def evict_blocks(self, sid: int, idxs) -> int:
        idxs = sorted(set(int(i) for i in idxs))
        if not idxs:
            return 0
        table = self.tables[sid]
        n = self.lengths[sid]
        n_full = n // self.block_size
        for i in idxs:
            if not 0 <= i < n_full:
                raise ValueError(f"block index {i} is not a full block (sequence has {n_full} full blocks)")
        drop = set(idxs)
        for i in idxs:
            self.slot_pos[table[i]] = -1
            self._release(table[i])
        self.tables[sid] = [b for j, b in enumerate(table) if j not in drop]
        removed = len(idxs) * self.block_size
        self.lengths[sid] = n - removed
        self.stats.evicted_blocks += len(idxs)
        self.stats.evicted_tokens += removed
        self.stats.eviction_calls += 1
        return removed

    def evict_positions(self, sid: int, spans):
        spans = list(spans)
        n = self.lengths[sid]
        if not spans or n == 0:
            return []
        pos = self.positions(sid)
        covered = np.zeros(n, dtype=bool)
        for s, e in spans:
            covered |= (pos >= s) & (pos < e)
        bs = self.block_size
        n_full = n // bs
        drop = [j for j in range(n_full) if covered[j * bs:(j + 1) * bs].all()]
        removed = [int(p) for j in drop for p in pos[j * bs:(j + 1) * bs]]
        self.stats.shrunk_tokens += int(covered.sum()) - len(removed)
        self.evict_blocks(sid, drop)
        return positions_to_spans(removed)

    # truncate (paged_cache.py:242-260)
    def truncate(self, sid: int, n_tokens: int) -> None:
        if n_tokens <= 0:
            return
        n = self.lengths[sid]
        if n_tokens > n:
            raise ValueError("cannot truncate more tokens than are live")
        new_len = n - n_tokens
        table = self.tables[sid]
        keep = -(-new_len // self.block_size)
        for i in range(new_len, n):
            b, o = divmod(i, self.block_size)
            self.slot_pos[table[b], o] = -1
        for b in table[keep:]:
            self._release(b)
        del table[keep:]
        self.lengths[sid] = new_len
        self.stats.truncated_tokens += n_tokens

    # invariants (paged_cache.py:262-273)
    def check_invariants(self, sid: int) -> str:
        """'' when fine, else the reference's AssertionError message."""
        table = self.tables[sid]
        n = self.lengths[sid]
        if len(set(table)) != len(table):
            return "block table references a block twice"
        if len(table) != -(-n // self.block_size):
            return "block table length does not match token count"
        pos = self.positions(sid)
        if (pos < 0).any():
            return "live slot without a logical position (hole in block table)"
        if pos.size > 1 and not (pos[1:] > pos[:-1]).all():
            return "logical positions are not strictly increasing"
        return ""


# ---------------------------------------------------------------------- evicted_at
def evicted_at(triples, length: int) -> np.ndarray:
    """compaction/events.py:66-74: triples = (start, end, time) of every evicted span."""
    out = np.full(length, NEVER, dtype=np.int64)
    for s, e, t in triples:
        e = min(int(e), length)
        if s < e:
            out[s:e] = np.minimum(out[s:e], int(t))
    return out


def kvstream_mask(ev: np.ndarray) -> np.ndarray:
    """training/replay.py:60-62: mask[t, s] = s <= t and t < evicted_at[s]."""
    T = ev.shape[0]
    idx = np.arange(T)
    return (idx[None, :] <= idx[:, None]) & (idx[:, None] < ev[None, :])


# ---------------------------------------------------------------------- rope
def rope_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """rope.py:26-28: computed in float64, stored as float32."""
    return (1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))).astype(np.float32)


def rope_apply(x: np.ndarray, positions: np.ndarray, theta: float, dtype=np.float32) -> np.ndarray:
    """rope.py:30-34,42-46 for x [..., T, H, D] and positions [..., T].

    float32: angle = float32(pos) * inv_freq in float32; float64: the float32 table
    widened to double (the reference module after ``.double()``)."""
    D = x.shape[-1]
    inv = rope_inv_freq(D, theta).astype(dtype)
    ang = positions.astype(dtype)[..., None] * inv  # [..., T, D/2]
    c = np.cos(ang).astype(dtype)[..., None, :]
    s = np.sin(ang).astype(dtype)[..., None, :]
    x = x.astype(dtype)
    a, b = x[..., : D // 2], x[..., D // 2:]
    return np.concatenate([a * c + (-b) * s, b * c + a * s], axis=-1).astype(dtype)


# ---------------------------------------------------------------------- attention
def gqa_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray, scale: float,
                  dtype=np.float64) -> np.ndarray:
    """model.py:67-74: q [T, Hq, D], k/v [S, Hkv, D], mask [T, S] -> [T, Hq, D]."""
    Hq, Hkv = q.shape[1], k.shape[1]
    rep = Hq // Hkv
    q = q.astype(dtype)
    k = np.repeat(k.astype(dtype), rep, axis=1)
    v = np.repeat(v.astype(dtype), rep, axis=1)
    s = np.einsum("qhd,khd->hqk", q, k) * dtype(scale)
    s = np.where(mask[None], s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.einsum("hqk,khd->qhd", p, v)


def replay_attention(q, k, v, ev, lengths, scale, dtype=np.float64):
    """Masked replay attention for a collated batch: q [B, T, Hq, D], k/v [B, T, Hkv, D],
    ev [B, T], lengths [B]; padded rows see only themselves (replay.py:221-222)."""
    B, T = q.shape[:2]
    out = np.zeros(q.shape, dtype=dtype)
    for b in range(B):
        m = np.eye(T, dtype=bool)
        n = int(lengths[b])
        m[:n, :n] = kvstream_mask(ev[b, :n])
        out[b] = gqa_attention(q[b], k[b], v[b], m, scale, dtype)
    return out


def replay_attention_rows(q, k, v, ev, rows, scale, dtype=np.float64):
    """Selected rows of the masked replay attention of one full-length stream, for sizes where
    the dense [T, T] mask does not fit: q [T, Hq, D], k/v [T, Hkv, D], ev [T]; row t attends to
    the keys s <= t with t < ev[s] (replay.py:55-63) with the math of model.py:67-74 (query
    head h reads KV head h // (Hq / Hkv), softmax of scaled scores, weighted values), computed
    per KV head as one small GEMM.  Returns [len(rows), Hq, D]."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    kh = np.ascontiguousarray(np.transpose(k, (1, 0, 2)).astype(dtype))  # [Hkv, T, D]
    vh = np.ascontiguousarray(np.transpose(v, (1, 0, 2)).astype(dtype))
    out = np.zeros((len(rows), Hq, D), dtype=dtype)
    for i, t in enumerate(np.asarray(rows, dtype=np.int64)):
        vis = ev[: t + 1] > t
        for g in range(Hkv):
            qs = q[t, g * rep:(g + 1) * rep].astype(dtype)              # [rep, D]
            sc = (qs @ kh[g, : t + 1].T) * dtype(scale)                  # [rep, t + 1]
            sc = np.where(vis[None], sc, -np.inf)
            sc -= sc.max(axis=-1, keepdims=True)
            pr = np.exp(sc)
            pr /= pr.sum(axis=-1, keepdims=True)
            out[i, g * rep:(g + 1) * rep] = pr @ vh[g, : t + 1]
    return out


# ---------------------------------------------------------------------- TinyLM
def _rms(x, w, eps):
    return x * (1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)) * w


def _silu(x):
    return x / (1.0 + np.exp(-x))


def tinylm_forward(params: dict, cfg: dict, tokens: np.ndarray, positions: np.ndarray, mask: np.ndarray,
                   dtype=np.float64) -> np.ndarray:
    """model.py:132-157 for one sequence: tokens/positions [T], mask [T, T] -> logits [T, V].

    ``params`` maps the reference state-dict names to arrays."""
    P = {k: np.asarray(v, dtype=dtype) for k, v in params.items()}
    H, Hkv = cfg["n_heads"], cfg["n_kv_heads"]
    D = cfg["d_model"] // H
    eps = cfg["norm_eps"]
    x = P["embed.weight"][tokens]
    for i in range(cfg["n_layers"]):
        p = f"layers.{i}."
        h = _rms(x, P[p + "attn_norm.weight"], eps)
        T = h.shape[0]
        q = (h @ P[p + "attn.q_proj.weight"].T).reshape(T, H, D)
        k = (h @ P[p + "attn.k_proj.weight"].T).reshape(T, Hkv, D)
        v = (h @ P[p + "attn.v_proj.weight"].T).reshape(T, Hkv, D)
        q = rope_apply(q, positions, cfg["rope_theta"], dtype)
        k = rope_apply(k, positions, cfg["rope_theta"], dtype)
        a = gqa_attention(q, k, v, mask, D ** -0.5, dtype).reshape(T, H * D)
        x = x + a @ P[p + "attn.o_proj.weight"].T
        h = _rms(x, P[p + "mlp_norm.weight"], eps)
        x = x + (_silu(h @ P[p + "mlp.gate.weight"].T) * (h @ P[p + "mlp.up.weight"].T)) @ P[p + "mlp.down.weight"].T
    return _rms(x, P["norm.weight"], eps) @ P["lm_head.weight"].T


def log_softmax(x: np.ndarray) -> np.ndarray:
    m = x.max(-1, keepdims=True)
    return x - m - np.log(np.exp(x - m).sum(-1, keepdims=True))


@dataclass
class OracleTrace:
    """A recorded sequence of cache operations (the op-trace format of the golden files)."""

    ops: list = field(default_factory=list)


def replay_trace(ops, num_blocks: int, block_size: int):
    """Run an op trace on OracleCache; returns the list of per-op observations
    (the same record tests/golden/make_golden.py takes from the reference)."""
    c = OracleCache(num_blocks, block_size)
    obs = []
    for op in ops:
        kind = op[0]
        res = None
        try:
            if kind == "add":
                c.add_sequence(op[1])
            elif kind == "append":
                c.append_slots(op[1], op[2])
            elif kind == "evict_positions":
                res = [list(s) for s in c.evict_positions(op[1], [tuple(s) for s in op[2]])]
            elif kind == "evict_blocks":
                res = c.evict_blocks(op[1], op[2])
            elif kind == "truncate":
                c.truncate(op[1], op[2])
            elif kind == "free":
                c.free_sequence(op[1])
            err = None
        except (ValueError, OutOfBlocksError) as exc:
            err = type(exc).__name__
        obs.append(snapshot(c, res, err))
    return c, obs


def snapshot(c: OracleCache, res, err):
    return {
        "result": res,
        "error": err,
        "tables": {str(k): list(v) for k, v in sorted(c.tables.items())},
        "lengths": {str(k): int(v) for k, v in sorted(c.lengths.items())},
        "free": list(c.free),
        "stats": c.stats.as_list(),
        "slot_pos_hash": slot_pos_digest(c.slot_pos),
    }


def slot_pos_digest(slot_pos: np.ndarray) -> str:
    import hashlib

    return hashlib.sha256(np.ascontiguousarray(slot_pos, dtype=np.int64).tobytes()).hexdigest()[:24]
