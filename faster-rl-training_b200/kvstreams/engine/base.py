"""Multi-turn rollout engines over the device-resident paged cache.

Behaviour (what a rollout contains) is the reference's rollout loop (engine/base.py:85-308):
the system prompt is forwarded and padded to the block size; every turn first checks the
context budget (``live + incoming + reserve > budget`` asks the policy for a plan, possibly a
summary turn, then evicts), forwards the user turn (after the uncommitted tail of the previous
turn when partial blocks are not committed), then generates the reply token by token (or
teacher-forces ``env.oracle()``), closes it at the length cap with an untrained end tag, and pads
to the block size.  Token streams, loss masks, segments, compaction events and stats are the
reference's for the same inputs.

Structure (this library's own): each episode is a coroutine (:meth:`BaseEngine._episode`) that
yields a :class:`_Forward` request whenever it needs tokens pushed through the model and
receives their logits; :meth:`BaseEngine.rollout_batch` drives any number of episodes, merging
their pending requests into one ``forward_cached_batch`` call per step (chunks first, then the
one-token decodes, which the fused decode kernel takes as one sub-batch).  ``rollout`` is a
batch of one.  Engines differ only in two hooks: the RoPE positions of new tokens and how an
eviction plan is carried out.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Generator, Optional, Sequence

import torch

from .. import _native as N
from ..chat import ChatTemplate
from ..compaction.events import CompactionEvent, CompactionLog
from ..compaction.policies import CompactionPlan, CompactionPolicy
from ..compaction.segments import Segment
from ..config import CacheConfig, RolloutConfig, SamplingConfig
from ..envs.base import Env
from ..paged_cache import PagedKVCache
from ..tokenizer import CharTokenizer
from ..utils.spans import Span
from .rollout import Rollout, RolloutStats


@dataclass
class _Forward:
    """Request from an episode: forward stream indices ``idx`` (``kind`` = prefill, decode or
    reprefill, for the stats); the reply is their ``[len(idx), vocab]`` logits."""

    idx: list[int]
    kind: str


@dataclass
class _Episode:
    """Everything one rollout accumulates, plus its cache bookkeeping."""

    seq_id: int
    generator: Optional[torch.Generator]
    tokens: list[int] = field(default_factory=list)
    loss_mask: list[bool] = field(default_factory=list)
    inf_logprobs: list[float] = field(default_factory=list)
    full_logprobs: dict = field(default_factory=dict)
    segments: list[Segment] = field(default_factory=list)
    log: CompactionLog = field(default_factory=CompactionLog)
    stats: RolloutStats = field(default_factory=RolloutStats)
    completions: list[str] = field(default_factory=list)
    context: list[int] = field(default_factory=list)  # stream indices with live KV, in cache order
    pending: list[int] = field(default_factory=list)  # uncommitted tail, forwarded again next turn
    reward: float = 0.0
    finished_at: float = 0.0

    def extend(self, ids: Sequence[int], trained: bool = False) -> list[int]:
        """Append tokens to the stream; returns their stream indices."""
        first = len(self.tokens)
        self.tokens += [int(t) for t in ids]
        self.loss_mask += [trained] * len(ids)
        self.inf_logprobs += [0.0] * len(ids)
        return list(range(first, len(self.tokens)))


Program = Generator[_Forward, torch.Tensor, float]


class BaseEngine:
    name = "base"

    def __init__(self, model, tokenizer: CharTokenizer, policy: CompactionPolicy,
                 cache_cfg: Optional[CacheConfig] = None, rollout_cfg: Optional[RolloutConfig] = None,
                 sampling: Optional[SamplingConfig] = None, cache: Optional[PagedKVCache] = None) -> None:
        self.model = model
        self.tok = tokenizer
        self.template = ChatTemplate(tokenizer)
        self.policy = policy
        self.cache_cfg = cache_cfg or CacheConfig()
        self.rollout_cfg = rollout_cfg or RolloutConfig()
        self.sampling = sampling or SamplingConfig()
        # a cache may be shared between engines (or be a test double)
        self.cache = cache if cache is not None else PagedKVCache.from_config(
            model.cfg, self.cache_cfg, device=model.device, dtype=getattr(model, "attention_dtype", model.dtype))
        self._seq_counter = 0

    @property
    def block_size(self) -> int:
        return self.cache_cfg.block_size

    # ------------------------------------------------------------------ engine hooks
    def _positions(self, ep: _Episode, idx: list[int]) -> list[int]:
        """RoPE positions of stream indices ``idx`` about to be forwarded."""
        raise NotImplementedError

    def _evict(self, ep: _Episode, spans: list[Span]) -> tuple[list[Span], Optional[list[int]]]:
        """Carry out an eviction request: the spans actually evicted, and the stream indices to
        forward again afterwards (None: nothing is rebuilt)."""
        raise NotImplementedError

    # ------------------------------------------------------------------ public
    def rollout(self, env: Env, generator: Optional[torch.Generator] = None, teacher_forcing: bool = False) -> Rollout:
        """Play one episode; with ``teacher_forcing`` replies come from ``env.oracle()`` (their
        log-probs are still recorded).  Compaction is identical in both modes."""
        return self.rollout_batch([env], [generator], teacher_forcing)[0]

    def rollout_batch(self, envs: Sequence[Env], generators: Optional[Sequence[Optional[torch.Generator]]] = None,
                      teacher_forcing: bool = False) -> list[Rollout]:
        """Play several episodes together: every step forwards the pending tokens of all of them
        in one batched call.  Each episode's contents equal those of ``rollout`` on its own."""
        gens = list(generators) if generators is not None else [None] * len(envs)
        if len(gens) != len(envs):
            raise ValueError("one generator (or None) per environment")
        was_training = self.model.training
        self.model.eval()
        t0 = time.perf_counter()
        eps = [self._new_episode(g) for g in gens]
        progs = [self._episode(ep, env, teacher_forcing) for ep, env in zip(eps, envs)]
        waiting: dict[int, _Forward] = {}
        try:
            with torch.no_grad():
                for i in range(len(progs)):
                    self._resume(i, eps[i], progs[i], None, waiting)
                while waiting:
                    # chunks first, one-token requests last: they form the decode sub-batch
                    order = sorted(waiting, key=lambda i: len(waiting[i].idx) == 1)
                    outs = self._forward_many([eps[i] for i in order], [waiting[i] for i in order])
                    for i, logits in zip(order, outs):
                        self._resume(i, eps[i], progs[i], logits, waiting)
        finally:
            for p in progs:
                p.close()  # an unfinished episode frees its sequence
            self.model.train(was_training)
        out = []
        for ep, env in zip(eps, envs):
            ep.stats.wall_time = ep.finished_at - t0
            out.append(Rollout(engine=self.name, tokens=ep.tokens, loss_mask=ep.loss_mask,
                               inf_logprobs=ep.inf_logprobs, segments=ep.segments, log=ep.log, stats=ep.stats,
                               reward=ep.reward, completions=ep.completions, block_size=self.block_size,
                               temperature=self.sampling.temperature, full_logprobs=ep.full_logprobs,
                               env_seed=getattr(env, "seed", None)))
        return out

    # ------------------------------------------------------------------ scheduler
    def _new_episode(self, generator) -> _Episode:
        ep = _Episode(self._seq_counter, generator)
        self._seq_counter += 1
        return ep

    @staticmethod
    def _resume(i: int, ep: _Episode, prog: Program, value, waiting: dict) -> None:
        try:
            waiting[i] = prog.send(value)
        except StopIteration as done:
            waiting.pop(i, None)
            ep.reward = float(done.value or 0.0)
            ep.finished_at = time.perf_counter()

    def _forward_many(self, eps: list[_Episode], reqs: list[_Forward]) -> list[torch.Tensor]:
        """One model call for the requests of several episodes (distinct sequences)."""
        dev = self.model.device
        toks, pos = [], []
        for ep, req in zip(eps, reqs):
            toks += [ep.tokens[j] for j in req.idx]
            pos += self._positions(ep, req.idx)
        tok_t = N.to_device(toks, torch.long, dev)
        pos_t = N.to_device(pos, torch.long, dev)
        if len(eps) == 1:
            parts = [self.model.forward_cached(tok_t, pos_t, self.cache, eps[0].seq_id)]
        else:
            counts = [len(r.idx) for r in reqs]
            logits = self.model.forward_cached_batch(tok_t, pos_t, self.cache, [ep.seq_id for ep in eps],
                                                     counts=counts)
            parts = list(torch.split(logits, counts))
        for ep, req in zip(eps, reqs):
            ep.context += req.idx
            st = ep.stats
            n = len(req.idx)
            st.tokens_forwarded += n
            if req.kind == "decode":
                st.decode_tokens += n
            elif req.kind == "reprefill":
                st.reprefill_tokens += n
            else:
                st.prefill_tokens += n
            st.peak_live_tokens = max(st.peak_live_tokens, self.cache.num_tokens(ep.seq_id))
        return parts

    # ------------------------------------------------------------------ one episode
    def _episode(self, ep: _Episode, env: Env, forcing: bool) -> Program:
        self.cache.add_sequence(ep.seq_id)
        try:
            start = env.reset()
            yield from self._open(ep, start.system)
            user = start.user
            for _ in range(self.rollout_cfg.max_turns):
                header = self.template.user_turn(user)
                target = env.oracle() if forcing else None
                yield from self._fit(ep, env, len(header), self._headroom(target), forcing)
                reply = yield from self._turn(ep, header, "turn", target)
                ep.completions.append(reply)
                step = env.step(reply)
                if step.done:
                    return step.reward
                user = step.user
            return 0.0
        finally:
            self.cache.free_sequence(ep.seq_id)

    def _open(self, ep: _Episode, system: str):
        """Prompt segment: system message, block padding, protected."""
        yield _Forward(ep.extend(self.template.system(system)), "prefill")
        yield from self._pad(ep)
        ep.segments.append(Segment(0, "prompt", 0, len(ep.tokens), protected=True))
        self._leave_tail_uncommitted(ep)

    def _headroom(self, target: Optional[str]) -> int:
        """Entries a reply may add: its tokens and end tag (the sampling cap when not forced),
        plus the worst-case block padding."""
        reply = len(self.tok.encode(target)) + 1 if target is not None else self.sampling.max_new_tokens + 1
        return reply + (self.block_size - 1 if self.cache_cfg.pad_to_block else 0)

    def _live(self, ep: _Episode) -> int:
        return self.cache.num_tokens(ep.seq_id) + len(ep.pending)

    def _pad(self, ep: _Episode):
        if self.cache_cfg.pad_to_block:
            pads = self.template.padding(len(ep.tokens), self.block_size)
            if pads:
                yield _Forward(ep.extend(pads), "prefill")
                ep.stats.padding_tokens += len(pads)

    def _leave_tail_uncommitted(self, ep: _Episode) -> None:
        """Without committed partial blocks (vLLM-style), the trailing partial block leaves the
        cache and is forwarded again at the start of the next turn."""
        if self.cache_cfg.commit_partial_blocks:
            return
        tail = self.cache.num_tokens(ep.seq_id) % self.block_size
        if tail:
            self.cache.truncate(ep.seq_id, tail)
            ep.pending = ep.context[-tail:]
            del ep.context[-tail:]

    def _log_softmax(self, logits: torch.Tensor) -> torch.Tensor:
        # float32 for half-precision models (the reference stays in the model dtype)
        if logits.dtype in (torch.bfloat16, torch.float16):
            logits = logits.float()
        return torch.log_softmax(logits / self.sampling.temperature, dim=-1)

    def _note_logprob(self, ep: _Episode, idx: int, row: torch.Tensor) -> None:
        ep.inf_logprobs[idx] = float(row[ep.tokens[idx]])
        if self.rollout_cfg.record_full_logprobs:
            ep.full_logprobs[idx] = row.detach().cpu().clone()

    def _draw(self, ep: _Episode, row: torch.Tensor) -> int:
        if self.sampling.greedy:
            return int(row.argmax())
        probs = row.exp()
        g = ep.generator
        if g is not None and g.device.type != probs.device.type:
            probs = probs.cpu()  # the caller's generator decides where the draw happens
        return int(torch.multinomial(probs, 1, generator=g))

    def _turn(self, ep: _Episode, header: list[int], kind: str, target: Optional[str]):
        """One user turn and the reply; returns the reply text."""
        seg_start = len(ep.tokens)
        new = ep.extend(header)
        redo, ep.pending = ep.pending, []
        if redo:
            ep.stats.recomputed_tokens += len(redo)
            if any(ev.evicted and ev.time > redo[0] for ev in ep.log):
                ep.stats.stale_recomputed_tokens += len(redo)
        last = (yield _Forward(redo + new, "prefill"))[-1]
        end = self.tok.end_id
        if target is not None:
            reply = self.tok.encode(target) + [end]
            idx = ep.extend(reply, trained=True)
            chunk = yield _Forward(idx, "prefill")
            rows = self._log_softmax(torch.cat([last[None], chunk[:-1]], dim=0))
            for k, i in enumerate(idx):
                self._note_logprob(ep, i, rows[k])
        else:
            reply = []
            capped = True
            for _ in range(self.sampling.max_new_tokens):
                row = self._log_softmax(last)
                tok = self._draw(ep, row)
                (i,) = ep.extend([tok], trained=True)
                self._note_logprob(ep, i, row)
                reply.append(tok)
                last = (yield _Forward([i], "decode"))[-1]
                if tok == end:
                    capped = False
                    break
            if capped:  # the length cap closes the message with an untrained end tag
                yield _Forward(ep.extend([end]), "decode")
        yield from self._pad(ep)
        ep.segments.append(Segment(len(ep.segments), kind, seg_start, len(ep.tokens)))
        self._leave_tail_uncommitted(ep)
        return self.tok.decode(reply)

    def _fit(self, ep: _Episode, env: Env, incoming: int, headroom: int, forcing: bool):
        """Budget check before a turn: plan, optional summary turn, eviction, overflow count."""
        budget = self.rollout_cfg.context_budget
        need = self._live(ep) + incoming + headroom
        if need <= budget:
            return
        plan = self.policy.plan(ep.segments, self._live(ep), budget, need)
        if plan.summary_request is not None:
            target = env.summary_oracle() if forcing else None
            header = self.template.user_turn(plan.summary_request)
            ep.completions.append((yield from self._turn(ep, header, "summary", target)))
        if plan.spans:
            yield from self._apply(ep, plan)
        if self._live(ep) + incoming + headroom > budget:
            ep.stats.budget_overflows += 1

    def _apply(self, ep: _Episode, plan: CompactionPlan):
        """Evict a plan's spans through the engine hook and record the event."""
        pending = set(ep.pending)
        if any(s <= p < e for p in pending for s, e in plan.spans):
            raise RuntimeError("compaction policy tried to evict uncommitted tokens of the latest turn")
        now = len(ep.tokens)
        before = self._live(ep)
        evicted, rebuild = self._evict(ep, plan.spans)
        if rebuild is not None:
            if rebuild:
                yield _Forward(rebuild, "reprefill")
            self._leave_tail_uncommitted(ep)
        if not evicted:
            return
        ev = CompactionEvent(time=now, evicted=evicted, requested=list(plan.spans), live_before=before,
                             live_after=self._live(ep), policy=self.policy.name, segments=list(plan.segments))
        ep.log.append(ev)
        ep.stats.compactions += 1
        ep.stats.evicted_tokens += ev.num_evicted
        for seg in ep.segments:
            if not seg.alive:
                continue
            covered = sum(max(0, min(seg.end, e) - max(seg.start, s)) for s, e in evicted)
            if covered >= seg.length:
                seg.evicted_at = now
                seg.partially_evicted = False
            elif covered:
                seg.partially_evicted = True
