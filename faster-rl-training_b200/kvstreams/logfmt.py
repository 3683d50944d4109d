"""Binary rollout batches: the compaction logs in compact columnar form for the trainer handoff.

The reference hands rollouts to the trainer as JSON (``Rollout.to_dict``, engine/rollout.py:66-80;
``CompactionLog.to_json``, compaction/events.py:79-84): every token, loss flag and log-prob as a
JSON number, and every compaction event as a dict.  This format stores the same content as
little-endian arrays, one section per field over the whole batch, so that the trainer reads a
batch with a handful of ``numpy.frombuffer`` calls and builds ``evicted_at`` on the device
from the stored (start, end, time) spans (the ``kvs_evicted_at`` kernel), never materialising
per-token Python objects:

    header   magic ``KVSROLL1``, then u32 version, u32 n_rollouts, u32 flags (bit 0: log-probs
             as f64, else f32), u32 reserved, u64 n_tokens, u64 n_events, u64 n_spans,
             u64 n_requested, u64 meta_bytes                                      (64 bytes)
    tok_off  u64[n_rollouts + 1]     token offset of each rollout
    tokens   i32[n_tokens]
    loss     u8[ceil(n_tokens / 8)]  loss mask, one bit per token (little bit order)
    logp     f32 or f64[n_tokens]    inference log-probs
    ev_off   u64[n_rollouts + 1]     event offset of each rollout
    ev_time  i64[n_events]           stream length at each compaction
    ev_live  i64[n_events][2]        live entries before / after
    sp_off   u64[n_events + 1]       evicted-span offset of each event
    spans    i64[n_spans][2]         evicted (start, end)
    rq_off   u64[n_events + 1]       requested-span offset of each event
    rq_spans i64[n_requested][2]     requested (start, end)
    meta     UTF-8 JSON: per rollout engine, segments, stats, reward, completions, block size,
             temperature, env seed; per event policy name and segment indices

Every section starts on an 8-byte boundary.  ``read_rollouts`` restores the rollouts exactly
(with ``f64`` log-probs); ``read_replay_batch`` returns the trainer's ``Batch`` for the
KV-streams replay (replay.py:55-63 + collate :132-149) of every rollout in the file.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import Optional, Sequence

import numpy as np
import torch

from .compaction.events import CompactionEvent, CompactionLog
from .compaction.segments import Segment
from .engine.rollout import Rollout, RolloutStats

MAGIC = b"KVSROLL1"
VERSION = 1
_HEADER = struct.Struct("<8sIIIIQQQQQ")
_HEADER_BYTES = _HEADER.size  # 64


def _pad8(n: int) -> int:
    return -n % 8


def write_rollouts(path, rollouts: Sequence[Rollout], logprob_dtype=np.float32) -> int:
    """Write ``rollouts`` to ``path``; returns the file size in bytes."""
    lp_dtype = np.dtype(logprob_dtype)
    if lp_dtype not in (np.dtype(np.float32), np.dtype(np.float64)):
        raise ValueError("log-probs are stored as float32 or float64")
    n = len(rollouts)
    lengths = np.asarray([len(r.tokens) for r in rollouts], dtype=np.uint64)
    tok_off = np.zeros(n + 1, dtype=np.uint64)
    np.cumsum(lengths, out=tok_off[1:])
    tokens = np.concatenate([np.asarray(r.tokens, dtype=np.int32) for r in rollouts]) if n else np.zeros(0, np.int32)
    loss = np.concatenate([np.asarray(r.loss_mask, dtype=bool) for r in rollouts]) if n else np.zeros(0, bool)
    logp = (np.concatenate([np.asarray(r.inf_logprobs, dtype=np.float64) for r in rollouts]) if n
            else np.zeros(0)).astype(lp_dtype)
    events = [e for r in rollouts for e in r.log]
    ev_off = np.zeros(n + 1, dtype=np.uint64)
    np.cumsum([len(r.log) for r in rollouts], out=ev_off[1:])
    ev_time = np.asarray([e.time for e in events], dtype=np.int64)
    ev_live = np.asarray([(e.live_before, e.live_after) for e in events], dtype=np.int64).reshape(-1, 2)
    sp_off = np.zeros(len(events) + 1, dtype=np.uint64)
    np.cumsum([len(e.evicted) for e in events], out=sp_off[1:])
    spans = np.asarray([s for e in events for s in e.evicted], dtype=np.int64).reshape(-1, 2)
    rq_off = np.zeros(len(events) + 1, dtype=np.uint64)
    np.cumsum([len(e.requested) for e in events], out=rq_off[1:])
    rq = np.asarray([s for e in events for s in e.requested], dtype=np.int64).reshape(-1, 2)
    meta = json.dumps({
        "rollouts": [{
            "engine": r.engine, "segments": [s.to_dict() for s in r.segments], "stats": r.stats.to_dict(),
            "reward": r.reward, "completions": r.completions, "block_size": r.block_size,
            "temperature": r.temperature, "env_seed": r.env_seed,
        } for r in rollouts],
        "events": [{"policy": e.policy, "segments": list(e.segments)} for e in events],
    }).encode()
    flags = 1 if lp_dtype == np.float64 else 0
    header = _HEADER.pack(MAGIC, VERSION, n, flags, 0, int(tokens.size), len(events), int(spans.shape[0]),
                          int(rq.shape[0]), len(meta))
    parts = [header]
    for arr in (tok_off, tokens, np.packbits(loss, bitorder="little"), logp, ev_off, ev_time, ev_live, sp_off,
                spans, rq_off, rq):
        b = np.ascontiguousarray(arr).astype(arr.dtype.newbyteorder("<"), copy=False).tobytes()
        parts.append(b + b"\0" * _pad8(len(b)))
    parts.append(meta)
    data = b"".join(parts)
    Path(path).write_bytes(data)
    return len(data)


class _Sections:
    def __init__(self, data: bytes) -> None:
        if len(data) < _HEADER_BYTES or data[:8] != MAGIC:
            raise ValueError("not a KV-streams rollout file")
        (_, version, n, flags, _, n_tok, n_ev, n_sp, n_rq, meta_bytes) = _HEADER.unpack_from(data, 0)
        if version != VERSION:
            raise ValueError(f"unsupported rollout file version {version}")
        self.n, self.n_tok, self.n_ev = n, n_tok, n_ev
        off = _HEADER_BYTES

        def take(dtype, count, shape=None):
            nonlocal off
            dt = np.dtype(dtype).newbyteorder("<")
            nbytes = dt.itemsize * count
            arr = np.frombuffer(data, dtype=dt, count=count, offset=off)
            off += nbytes + _pad8(nbytes)
            return arr.reshape(shape) if shape is not None else arr

        self.tok_off = take(np.uint64, n + 1).astype(np.int64)
        self.tokens = take(np.int32, n_tok)
        self.loss = np.unpackbits(take(np.uint8, (n_tok + 7) // 8), bitorder="little", count=n_tok).astype(bool)
        self.logp = take(np.float64 if flags & 1 else np.float32, n_tok)
        self.ev_off = take(np.uint64, n + 1).astype(np.int64)
        self.ev_time = take(np.int64, n_ev)
        self.ev_live = take(np.int64, 2 * n_ev, (n_ev, 2))
        self.sp_off = take(np.uint64, n_ev + 1).astype(np.int64)
        self.spans = take(np.int64, 2 * n_sp, (n_sp, 2))
        self.rq_off = take(np.uint64, n_ev + 1).astype(np.int64)
        self.rq = take(np.int64, 2 * n_rq, (n_rq, 2))
        self.meta = json.loads(data[off:off + meta_bytes].decode()) if meta_bytes else None


def read_rollouts(path) -> list[Rollout]:
    """The rollouts of a file, as the engines produced them."""
    s = _Sections(Path(path).read_bytes())
    out = []
    for i in range(s.n):
        a, b = s.tok_off[i], s.tok_off[i + 1]
        m = s.meta["rollouts"][i]
        events = []
        for e in range(s.ev_off[i], s.ev_off[i + 1]):
            em = s.meta["events"][e]
            events.append(CompactionEvent(
                time=int(s.ev_time[e]),
                evicted=[(int(x), int(y)) for x, y in s.spans[s.sp_off[e]:s.sp_off[e + 1]]],
                requested=[(int(x), int(y)) for x, y in s.rq[s.rq_off[e]:s.rq_off[e + 1]]],
                live_before=int(s.ev_live[e, 0]), live_after=int(s.ev_live[e, 1]),
                policy=em["policy"], segments=list(em["segments"])))
        out.append(Rollout(
            engine=m["engine"], tokens=s.tokens[a:b].astype(np.int64).tolist(), loss_mask=s.loss[a:b].tolist(),
            inf_logprobs=s.logp[a:b].astype(np.float64).tolist(),
            segments=[Segment(**d) for d in m["segments"]], log=CompactionLog(events),
            stats=RolloutStats(**m["stats"]), reward=m["reward"], completions=list(m["completions"]),
            block_size=m["block_size"], temperature=m["temperature"], env_seed=m["env_seed"]))
    return out


def read_replay_batch(path, device=None, pad_id: int = 0, rows: Optional[Sequence[int]] = None):
    """The trainer's :class:`~kvstreams.training.replay.Batch` for the KV-streams replay of the
    rollouts in ``path`` (all, or the given ``rows``): whole streams at their original
    positions, padded to the longest, ``evicted_at`` built on the device from the spans."""
    from .ops import evicted_at_from_spans
    from .training.replay import Batch

    s = _Sections(Path(path).read_bytes())
    rows = list(range(s.n)) if rows is None else list(rows)
    lens = np.asarray([s.tok_off[i + 1] - s.tok_off[i] for i in rows], dtype=np.int64)
    B, T = len(rows), int(lens.max()) if len(rows) else 0
    tokens = np.full((B, T), pad_id, dtype=np.int64)
    loss = np.zeros((B, T), dtype=bool)
    inf = np.zeros((B, T), dtype=np.float64)
    triples, cu = [], np.zeros(B + 1, dtype=np.int32)
    for j, i in enumerate(rows):
        a, b = s.tok_off[i], s.tok_off[i + 1]
        tokens[j, :b - a] = s.tokens[a:b]
        loss[j, :b - a] = s.loss[a:b]
        inf[j, :b - a] = s.logp[a:b]
        e0, e1 = s.ev_off[i], s.ev_off[i + 1]
        ev_of_span = np.repeat(np.arange(e0, e1), np.diff(s.sp_off[e0:e1 + 1]))
        sp = s.spans[s.sp_off[e0]:s.sp_off[e1]]
        triples.append(np.concatenate([sp, s.ev_time[ev_of_span, None]], axis=1))
        cu[j + 1] = cu[j] + sp.shape[0]
    flat = np.concatenate(triples) if cu[-1] else np.zeros((1, 3), dtype=np.int64)
    dev = torch.device(device) if device is not None else torch.device("cuda")
    ev = evicted_at_from_spans(cu, flat, lens.tolist(), dev, T)
    # original positions (stream indices); padding at 0, as collate leaves it
    ar = torch.arange(T, dtype=torch.long)[None, :].expand(B, T)
    positions = torch.where(ar < torch.from_numpy(lens)[:, None], ar, torch.zeros_like(ar))
    return Batch(torch.from_numpy(tokens), positions, ev, torch.from_numpy(loss), torch.from_numpy(inf),
                 torch.from_numpy(lens))
