"""Training sequences from a rollout plus its compaction log (training/replay.py:1-149).

KV-streams replay (:func:`kvstream_sequence`) is one sequence over the whole stream
with positions ``0..T-1`` and the visibility rule

    visible(t, s) = s <= t and t < evicted_at[s]

Here the mask stays factored: a sequence carries its compaction log, the batch
carries ``evicted_at [B, T]`` (built by the device evicted_at kernel) and lengths,
and the masked replay kernel applies the rule tile by tile.  ``.mask`` still
returns the dense boolean matrix when asked for it.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from ..compaction.events import CompactionLog
from ..engine.rollout import Rollout
from ..ops import ReplayMask, evicted_at_from_spans


@dataclass
class TrainSequence:
    tokens: torch.Tensor  # [T] long
    positions: torch.Tensor  # [T] long
    loss_mask: torch.Tensor  # [T] bool
    inf_logprobs: torch.Tensor  # [T] float64
    stream_index: torch.Tensor  # [T] long
    log: CompactionLog = field(default_factory=CompactionLog)  # empty log = causal

    @property
    def length(self) -> int:
        return int(self.tokens.numel())

    def evicted_at(self, device=None) -> torch.Tensor:
        return self.log.evicted_at(self.length, device)

    @property
    def mask(self) -> torch.Tensor:
        """Dense ``[T, T]`` mask (replay.py:62); inspection only."""
        rm = ReplayMask(self.evicted_at("cuda")[None], torch.tensor([self.length], dtype=torch.int32, device="cuda"))
        return rm.dense()[0]


def _tensors(rollout: Rollout):
    return (
        torch.tensor(rollout.tokens, dtype=torch.long),
        torch.tensor(rollout.loss_mask, dtype=torch.bool),
        torch.tensor(rollout.inf_logprobs, dtype=torch.float64),
    )


def kvstream_sequence(rollout: Rollout) -> TrainSequence:
    """replay.py:55-63: the whole stream, original positions, the rollout's compaction log."""
    tokens, loss, inf = _tensors(rollout)
    idx = torch.arange(tokens.numel())
    return TrainSequence(tokens, idx.clone(), loss, inf, idx.clone(), rollout.log)


def full_context_sequence(rollout: Rollout) -> TrainSequence:
    """replay.py:66-71: naive replay, plain causal mask."""
    tokens, loss, inf = _tensors(rollout)
    idx = torch.arange(tokens.numel())
    return TrainSequence(tokens, idx.clone(), loss, inf, idx.clone())


def window_sequences(rollout: Rollout) -> list[TrainSequence]:
    """replay.py:74-99: one re-numbered causal window per compaction interval."""
    tokens, loss, inf = _tensors(rollout)
    T = tokens.numel()
    ev = np.full(T, np.iinfo(np.int64).max, dtype=np.int64)
    for s, e, t in rollout.log.span_triples():
        e = min(int(e), T)
        if s < e:
            np.minimum(ev[s:e], t, out=ev[s:e])
    times = sorted({e.time for e in rollout.log if e.evicted})
    bounds = [0, *times, T]
    out = []
    for a, b in zip(bounds[:-1], bounds[1:]):
        if a >= b:
            continue
        ctx = [s for s in range(a) if ev[s] > a]
        idx = torch.tensor(ctx + list(range(a, b)), dtype=torch.long)
        wl = loss[idx].clone()
        wl[: len(ctx)] = False
        out.append(TrainSequence(tokens[idx], torch.arange(idx.numel()), wl, inf[idx], idx))
    return out


def build_sequences(rollout: Rollout, mode: str = "auto") -> list[TrainSequence]:
    """``mode``: ``auto`` (match the engine), ``kvstream``, ``windows`` or ``full``."""
    if mode == "auto":
        mode = "kvstream" if rollout.engine == "kvstream" else "windows"
    if mode == "kvstream":
        return [kvstream_sequence(rollout)]
    if mode == "windows":
        return window_sequences(rollout)
    if mode == "full":
        return [full_context_sequence(rollout)]
    raise ValueError(f"unknown replay mode {mode!r}")


@dataclass
class Batch:
    tokens: torch.Tensor  # [B, T]
    positions: torch.Tensor  # [B, T]
    evicted_at: torch.Tensor  # [B, T] int64 (device)
    loss_mask: torch.Tensor  # [B, T]
    inf_logprobs: torch.Tensor  # [B, T]
    lengths: torch.Tensor  # [B]

    def to(self, device) -> "Batch":
        return Batch(*(getattr(self, f).to(device) for f in self.__dataclass_fields__))

    @property
    def mask(self) -> ReplayMask:
        """The replay mask in factored form (dense via ``.mask.dense()``)."""
        return ReplayMask(self.evicted_at, self.lengths.to(self.evicted_at.device, torch.int32))

    @property
    def num_tokens(self) -> int:
        return int(self.lengths.sum())


def collate(seqs: list[TrainSequence], pad_id: int = 0, device=None) -> Batch:
    """replay.py:132-149: pad to the longest sequence; padded rows attend to themselves."""
    B = len(seqs)
    T = max(s.length for s in seqs)
    tokens = torch.full((B, T), pad_id, dtype=torch.long)
    positions = torch.zeros(B, T, dtype=torch.long)
    loss_mask = torch.zeros(B, T, dtype=torch.bool)
    inf = torch.zeros(B, T, dtype=torch.float64)
    for b, s in enumerate(seqs):
        n = s.length
        tokens[b, :n] = s.tokens
        positions[b, :n] = s.positions
        loss_mask[b, :n] = s.loss_mask
        inf[b, :n] = s.inf_logprobs
    lengths = torch.tensor([s.length for s in seqs], dtype=torch.long)
    triples = [s.log.span_triples() for s in seqs]
    cu = np.zeros(B + 1, dtype=np.int32)
    np.cumsum([len(t) for t in triples], out=cu[1:])
    flat = np.concatenate(triples, axis=0) if sum(len(t) for t in triples) else np.zeros((1, 3), dtype=np.int64)
    dev = torch.device(device) if device is not None else torch.device("cuda")
    ev = evicted_at_from_spans(cu, flat, [s.length for s in seqs], dev, T)
    return Batch(tokens, positions, ev, loss_mask, inf, lengths)
