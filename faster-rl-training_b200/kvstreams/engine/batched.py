"""Many KV-streams rollouts advanced together on one GPU.

The reference plays one episode at a time (engine/base.py:85-308): prompt prefill, then per
turn a compaction check (``_maybe_compact``, :260-285), the user-turn prefill, token-by-token
decoding and block padding.  :class:`BatchedKVStreams` runs the same per-rollout sequence for a
whole batch of rollouts sharing one :class:`~kvstreams.paged_cache.PagedKVCache`:

* every loop iteration forwards one token for each rollout that is generating (the fused paged
  decode kernel, one launch per layer for the whole batch), and in one batched prefill call
  (the tensor-core paged prefill) the chunks of the rollouts that start a turn (the
  observation; for the first turn the padded prompt too) or end a reply (its last token with
  the turn's block padding, so that the padding is in the cache before the next compaction
  check, as in the reference);
* compaction decisions are the reference policies' (``policy.plan`` on the rollout's segments,
  same ``required = live + incoming + reserve`` test), executed for all rollouts that need one
  in a single batched in-place eviction (``evict_positions_batch``, one device round trip for
  its result); with ``device_policy=True`` the decision, the eviction and the bookkeeping all
  run on the device (:class:`~kvstreams.compaction.device.DeviceCompaction`, no round trip)
  and segments, compaction log and stats are read back once, when the rollouts end;
* sampling, sampled tokens and their log-probs stay on the device; the host only tracks
  lengths, positions and segments, so a step needs no device round trip.

Episodes are synthetic token streams (``SyntheticEpisode``): a prompt, then per turn an
observation chunk and a reply of a given length, sampled from the model (or teacher-forced).
Positions are stream indices, as in ``KVStreamEngine._positions`` (engine/kv_stream.py:19-21).
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np
import torch

from .. import _native as N
from ..compaction.events import CompactionEvent, CompactionLog
from ..compaction.policies import CompactionPolicy
from ..compaction.segments import Segment
from .rollout import Rollout, RolloutStats


@dataclass
class SyntheticEpisode:
    """Token-level episode: ``prompt`` ids, then per turn ``observations[i]`` ids followed by a
    reply of ``reply_lens[i]`` generated tokens (``replies[i]`` when teacher-forced)."""

    prompt: np.ndarray
    observations: list[np.ndarray]
    reply_lens: list[int]
    replies: Optional[list[np.ndarray]] = None

    @property
    def turns(self) -> int:
        return len(self.observations)


def synthetic_episodes(n: int, turns: int = 24, turn_range=(64, 512), prompt_len: int = 64, vocab: int = 128256,
                       forced: bool = False, seed: int = 0) -> list[SyntheticEpisode]:
    """Seeded episodes with uniform random ids: observation and reply lengths ~U[turn_range]."""
    rng = np.random.default_rng(seed)
    lo, hi = turn_range
    out = []
    for _ in range(n):
        prompt = rng.integers(1, vocab, size=prompt_len, dtype=np.int64)
        obs = [rng.integers(1, vocab, size=int(rng.integers(lo, hi + 1)), dtype=np.int64) for _ in range(turns)]
        rl = [int(rng.integers(lo, hi + 1)) for _ in range(turns)]
        reps = [rng.integers(1, vocab, size=r, dtype=np.int64) for r in rl] if forced else None
        out.append(SyntheticEpisode(prompt, obs, rl, reps))
    return out


# rollout phases
_PREFILL, _DECODE, _DONE = 0, 1, 2


@dataclass
class _Run:
    idx: int
    ep: SyntheticEpisode
    seq_id: int
    n_tokens: int = 0             # stream length (tokens appended so far, forwarded or pending)
    turn: int = -1                # current turn (-1: prompt not yet forwarded)
    phase: int = _PREFILL
    step: int = 0                 # reply tokens forwarded in the current turn
    pending: list = field(default_factory=list)  # the padded prompt until the first chunk
    segments: list = field(default_factory=list)
    log: CompactionLog = field(default_factory=CompactionLog)
    stats: RolloutStats = field(default_factory=RolloutStats)
    turn_start: int = 0
    live: int = 0                 # cache entries (forwarded and not evicted)
    # stream-index ranges of generated tokens: (stream start, device buffer offset, length)
    gen_ranges: list = field(default_factory=list)
    host_spans: list = field(default_factory=list)  # (start, tokens) appended from the host


class BatchedKVStreams:
    """Batched KV-streams rollouts (see the module docstring)."""

    name = "kvstream"

    def __init__(self, model, cache, policy: CompactionPolicy, context_budget: int = 8192, pad_to_block: bool = True,
                 pad_id: int = 0, temperature: float = 1.0, greedy: bool = False, seed: int = 0,
                 cuda_graphs: bool = False, device_policy: bool = False) -> None:
        self.model = model
        self.cache = cache
        self.policy = policy
        self.budget = int(context_budget)
        self.bs = cache.block_size
        self.pad_to_block = pad_to_block
        self.pad_id = int(pad_id)
        self.temperature = float(temperature)
        self.greedy = greedy
        self.gen = torch.Generator(device=model.device).manual_seed(seed)
        self.seed = int(seed)
        self._draws = 0  # sampling calls so far: the Philox offset of the next one (ops.sample)
        self._next_seq = 0
        # decode steps replayed as CUDA graphs (one per batch size), see engine/graphs.py
        self.cuda_graphs = cuda_graphs
        self._graphs = None
        # compaction planned and applied on the device (compaction/device.py)
        self.device_policy = device_policy
        self._dev = None

    # ------------------------------------------------------------------ helpers
    def _reserve(self, run: _Run) -> int:
        """engine/base.py:146-153: reply length + 1, plus the padding bound."""
        pad = self.bs - 1 if self.pad_to_block else 0
        return run.ep.reply_lens[run.turn + 1] + 1 + pad

    def _maybe_compact(self, runs: Sequence[_Run]) -> None:
        """engine/base.py:260-285 for every rollout about to start a turn, one batched eviction."""
        if self.device_policy:
            self._dev.compact([self.cache.slot(r.seq_id) for r in runs], [len(r.pending) for r in runs],
                              [len(r.ep.observations[r.turn + 1]) + self._reserve(r) for r in runs],
                              [r.n_tokens for r in runs])
            return
        todo, plans = [], []
        for run in runs:
            incoming = len(run.ep.observations[run.turn + 1])
            live = run.live + len(run.pending)
            required = live + incoming + self._reserve(run)
            if required <= self.budget:
                continue
            plan = self.policy.plan(run.segments, live, self.budget, required)
            if plan.spans:
                todo.append(run)
                plans.append(plan)
        # (no early return when nothing is evicted: the overflow count below still applies,
        # engine/base.py:274-275)
        evicted = self.cache.evict_positions_batch([r.seq_id for r in todo], [p.spans for p in plans]) if todo else []
        for run, plan, ev in zip(todo, plans, evicted):
            if not ev:
                continue
            t = run.n_tokens
            live_before = run.live + len(run.pending)
            removed = sum(e - s for s, e in ev)
            run.live -= removed
            event = CompactionEvent(time=t, evicted=list(ev), requested=list(plan.spans), live_before=live_before,
                                    live_after=run.live + len(run.pending), policy=self.policy.name,
                                    segments=list(plan.segments))
            run.log.append(event)
            run.stats.compactions += 1
            run.stats.evicted_tokens += removed
            for seg in run.segments:
                if not seg.alive:
                    continue
                covered = sum(max(0, min(seg.end, e) - max(seg.start, s)) for s, e in ev)
                if covered >= seg.length:
                    seg.evicted_at = t
                    seg.partially_evicted = False
                elif covered:
                    seg.partially_evicted = True
        for run in runs:
            live = run.live + len(run.pending)
            if live + len(run.ep.observations[run.turn + 1]) + self._reserve(run) > self.budget:
                run.stats.budget_overflows += 1

    def _collect_device_compaction(self, runs: Sequence[_Run]) -> None:
        """Segments' eviction marks, compaction log and stats from the device (one read)."""
        res = self._dev.read([self.cache.slot(r.seq_id) for r in runs])
        for r, d in zip(runs, res):
            for seg, ev_at, part in zip(r.segments, d["evicted_at"], d["partial"]):
                seg.evicted_at = None if ev_at < 0 else ev_at
                seg.partially_evicted = part
            for ev in d["events"]:
                r.log.append(ev)
            r.stats.compactions = d["stats"]["compactions"]
            r.stats.evicted_tokens = d["stats"]["evicted_tokens"]
            r.stats.budget_overflows = d["stats"]["budget_overflows"]
            # the live count only drops at compactions: its peak is before one of them or at the end
            r.stats.peak_live_tokens = max(d["peak_cached"], self.cache.num_tokens(r.seq_id))
            r.live = self.cache.num_tokens(r.seq_id)

    def _sample(self, logits: torch.Tensor, forced: Optional[torch.Tensor]):
        """Next token and its log-prob under temperature (engine/base.py:176-193), on the device:
        on CUDA one pass per logits row (``kvs_sample``; ``kvs_lse_gather`` for forced tokens)."""
        if logits.is_cuda:
            from .. import ops

            x = logits.float()  # log-probs are kept in float32 (as the torch path below)
            if forced is not None:
                return forced, ops.lse_gather(x, forced, self.temperature)[0]
            tok, lp = ops.sample(x, self.temperature, self.greedy, seed=self.seed, offset=self._draws)
            self._draws += 1
            return tok, lp
        logp = torch.log_softmax(logits.float() / self.temperature, dim=-1)
        if forced is not None:
            tok = forced
        elif self.greedy:
            tok = logp.argmax(-1)
        else:
            tok = torch.multinomial(logp.exp(), 1, generator=self.gen).squeeze(1)
        return tok, logp.gather(1, tok.view(-1, 1)).squeeze(1)

    # ------------------------------------------------------------------ main loop
    @torch.no_grad()
    def run(self, episodes: Sequence[SyntheticEpisode], max_iterations: Optional[int] = None,
            on_iteration=None) -> list[Rollout]:
        """Play ``episodes`` to the end (or for ``max_iterations`` loop iterations);
        ``on_iteration(i, decode_tokens, prefill_tokens)`` is called after each iteration with
        the tokens it forwarded."""
        dev = self.model.device
        runs = []
        for i, ep in enumerate(episodes):
            seq = self._next_seq
            self._next_seq += 1
            self.cache.add_sequence(seq)
            run = _Run(i, ep, seq)
            run.pending = [int(x) for x in ep.prompt]
            run.host_spans.append((0, np.asarray(ep.prompt, dtype=np.int64)))
            run.n_tokens = len(ep.prompt)
            if self.pad_to_block and run.n_tokens % self.bs:
                pads = [self.pad_id] * (-run.n_tokens % self.bs)
                run.host_spans.append((run.n_tokens, np.asarray(pads, dtype=np.int64)))
                run.pending += pads
                run.stats.padding_tokens += len(pads)
                run.n_tokens += len(pads)
            run.segments.append(Segment(0, "prompt", 0, run.n_tokens, protected=True))
            if self.device_policy:
                if self._dev is None:
                    from ..compaction.device import DeviceCompaction

                    self._dev = DeviceCompaction(self.cache, self.policy, self.budget)
                slot = self.cache.slot(seq)
                self._dev.reset_slot(slot)
                self._dev.add_segment(slot, run.segments[0])
            runs.append(run)
        total_gen = sum(sum(ep.reply_lens) for ep in episodes)
        gen_tok = torch.zeros(max(total_gen, 1), dtype=torch.long, device=dev)
        gen_logp = torch.zeros(max(total_gen, 1), dtype=torch.float32, device=dev)
        gen_base = np.cumsum([0] + [sum(ep.reply_lens) for ep in episodes])
        gen_used = [0] * len(runs)
        # forced reply tokens, flattened per rollout in the same layout as the generated buffer
        forced_all = None
        if all(ep.replies is not None for ep in episodes):
            forced_all = torch.from_numpy(np.concatenate([np.concatenate(ep.replies) for ep in episodes]
                                                         or [np.zeros(1, np.int64)])).to(dev)
        # the token each decoding rollout forwards next: device slot per rollout
        cur = torch.zeros(len(runs), dtype=torch.long, device=dev)
        t0 = time.perf_counter()
        # host index lists reach the device through pinned memory: the loop never waits on the GPU
        def _to_dev(values):
            return N.to_device(values, torch.long, dev)

        it = 0
        while True:
            active = [r for r in runs if r.phase != _DONE]
            if not active or (max_iterations is not None and it >= max_iterations):
                break
            it += 1
            n_dec = n_pre = 0
            starting = [r for r in active if r.phase == _PREFILL]

            def decode_step(logits: torch.Tensor) -> None:
                """Sample the next token of every generating rollout from its logits row."""
                rows = _to_dev([r.idx for r in decoding])
                idx = _to_dev([gen_base[r.idx] + gen_used[r.idx] for r in decoding])
                forced = forced_all.index_select(0, idx) if forced_all is not None else None
                tok, lp = self._sample(logits, forced)
                gen_tok.index_copy_(0, idx, tok)
                gen_logp.index_copy_(0, idx, lp)
                cur.index_copy_(0, rows, tok)
                for r in decoding:
                    r.n_tokens += 1
                    r.live += 1
                    r.step += 1
                    gen_used[r.idx] += 1
                    r.stats.decode_tokens += 1
                    r.stats.tokens_forwarded += 1
                    r.stats.peak_live_tokens = max(r.stats.peak_live_tokens, r.live)

            # a rollout forwarding the last token of its reply sends it with the turn's block
            # padding as one chunk: the padding is in the cache before the next compaction
            # check, as in the reference (engine/base.py:241-245, then :260)
            finishing = [r for r in active if r.phase == _DECODE and r.step + 1 == r.ep.reply_lens[r.turn]]
            decoding = [r for r in active if r.phase == _DECODE and r.step + 1 < r.ep.reply_lens[r.turn]]
            # ---- chunks: turn starts (after their compaction check) and reply ends
            if starting or finishing:
                if starting:
                    self._maybe_compact(starting)
                host_tok, counts, pos, dev_rows, dev_at = [], [], [], [], []
                base = 0
                for r in starting:
                    obs = r.ep.observations[r.turn + 1]
                    r.host_spans.append((r.n_tokens, np.asarray(obs, dtype=np.int64)))
                    toks = r.pending + [int(x) for x in obs]
                    start = r.n_tokens - len(r.pending)
                    r.turn_start = r.n_tokens
                    r.n_tokens += len(obs)
                    r.pending = []
                    host_tok.append(np.asarray(toks, dtype=np.int64))
                    counts.append(len(toks))
                    pos.append(np.arange(start, start + len(toks), dtype=np.int64))
                    r.live += len(toks)
                    r.stats.prefill_tokens += len(toks)
                    r.stats.tokens_forwarded += len(toks)
                    r.stats.peak_live_tokens = max(r.stats.peak_live_tokens, r.live)
                    base += len(toks)
                for r in finishing:
                    pads = (-(r.n_tokens + 1) % self.bs) if self.pad_to_block else 0
                    dev_rows.append(r.idx)
                    dev_at.append(base)
                    host_tok.append(np.full(1 + pads, self.pad_id, dtype=np.int64))
                    counts.append(1 + pads)
                    pos.append(np.arange(r.n_tokens, r.n_tokens + 1 + pads, dtype=np.int64))
                    if pads:
                        r.host_spans.append((r.n_tokens + 1, np.full(pads, self.pad_id, dtype=np.int64)))
                    r.stats.decode_tokens += 1
                    r.stats.padding_tokens += pads
                    r.stats.prefill_tokens += pads
                    r.stats.tokens_forwarded += 1 + pads
                    r.n_tokens += 1 + pads
                    r.live += 1 + pads
                    r.stats.peak_live_tokens = max(r.stats.peak_live_tokens, r.live)
                    base += 1 + pads
                n_pre = base - len(finishing)
                n_dec = len(finishing)
                # the generating rollouts ride along in the same forward (one weight read per
                # iteration): one token each, after the chunks (the decode kernel's sub-batch)
                merged = list(decoding)
                for r in merged:
                    dev_rows.append(r.idx)
                    dev_at.append(base)
                    host_tok.append(np.zeros(1, dtype=np.int64))
                    counts.append(1)
                    pos.append(np.asarray([r.n_tokens], dtype=np.int64))
                    base += 1
                tok_t = _to_dev(np.concatenate(host_tok))
                if dev_rows:  # last reply tokens and generating rollouts' tokens come from the device
                    tok_t.index_copy_(0, _to_dev(dev_at), cur.index_select(0, _to_dev(dev_rows)))
                pos_t = _to_dev(np.concatenate(pos))
                order = starting + finishing + merged
                logits_all = self.model.forward_cached_batch(tok_t, pos_t, self.cache, [r.seq_id for r in order],
                                                             counts=counts, last_only=True)
                if merged:
                    decode_step(logits_all[len(starting) + len(finishing):])
                if starting:
                    logits = logits_all[: len(starting)]
                    idx = _to_dev([gen_base[r.idx] + gen_used[r.idx] for r in starting])
                    forced = forced_all.index_select(0, idx) if forced_all is not None else None
                    tok, lp = self._sample(logits, forced)
                    gen_tok.index_copy_(0, idx, tok)
                    gen_logp.index_copy_(0, idx, lp)
                    cur.index_copy_(0, _to_dev([r.idx for r in starting]), tok)
                for r in starting:
                    r.turn += 1
                    r.phase = _DECODE
                    r.step = 0
                    r.gen_ranges.append((r.n_tokens, gen_base[r.idx] + gen_used[r.idx], r.ep.reply_lens[r.turn]))
                    gen_used[r.idx] += 1
                for r in finishing:
                    r.segments.append(Segment(len(r.segments), "turn", r.turn_start, r.n_tokens))
                    if self.device_policy:
                        self._dev.add_segment(self.cache.slot(r.seq_id), r.segments[-1])
                    r.phase = _PREFILL if r.turn + 1 < r.ep.turns else _DONE
            # ---- an iteration without chunks: the decode step alone (a replayed graph)
            elif decoding:
                rows = _to_dev([r.idx for r in decoding])
                tok_in = cur.index_select(0, rows)
                if self.cuda_graphs:
                    if self._graphs is None:
                        from .graphs import DecodeGraphs

                        self._graphs = DecodeGraphs(self.model, self.cache, len(runs))
                    logits = self._graphs.step([r.seq_id for r in decoding], tok_in, [r.n_tokens for r in decoding])
                else:
                    pos_t = _to_dev([r.n_tokens for r in decoding])
                    logits = self.model.forward_cached_batch(tok_in, pos_t, self.cache, [r.seq_id for r in decoding])
                decode_step(logits)
            n_dec += len(decoding)
            if on_iteration is not None:
                on_iteration(it, n_dec, n_pre)
        torch.cuda.synchronize(dev)
        wall = time.perf_counter() - t0
        # ---- assemble the rollouts (one device-to-host copy)
        toks_h = gen_tok.cpu().numpy()
        logp_h = gen_logp.cpu().numpy()
        if self.device_policy:
            self._collect_device_compaction(runs)
        out = []
        for r in runs:
            n = r.n_tokens
            tokens = np.full(n, self.pad_id, dtype=np.int64)
            loss = np.zeros(n, dtype=bool)
            inf = np.zeros(n, dtype=np.float64)
            for start, arr in r.host_spans:
                tokens[start:start + len(arr)] = arr
            for start, off, length in r.gen_ranges:
                length = min(length, n - start)
                tokens[start:start + length] = toks_h[off:off + length]
                loss[start:start + length] = True
                inf[start:start + length] = logp_h[off:off + length]
            r.stats.wall_time = wall
            self.cache.free_sequence(r.seq_id)
            out.append(Rollout(engine=self.name, tokens=tokens.tolist(), loss_mask=loss.tolist(),
                               inf_logprobs=inf.tolist(), segments=r.segments, log=r.log, stats=r.stats,
                               block_size=self.bs, temperature=self.temperature))
        self.last_iterations = it
        self.last_wall = wall
        return out
