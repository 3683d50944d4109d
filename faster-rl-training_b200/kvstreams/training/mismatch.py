"""How far the trainer's replayed log-probabilities are from the ones recorded at inference
(training/mismatch.py:21-86 in the reference: same report fields and estimators).

For every loss token, with ``d = log p_train - log p_inf`` under the inference distribution:

* ``kl_k3`` = mean(e^d - 1 - d), ``kl_k1`` = mean(-d) (sample estimators of KL(inf || train)),
* ``exact_kl`` = mean over tokens of sum_v p_inf(v) (log p_inf(v) - log p_train(v)) when the
  rollouts recorded whole inference rows,
* ``max_abs_logprob_diff`` / ``mean_abs_logprob_diff`` of |d|.

Here the statistics are running float64 sums (:class:`_Tally`) fed one replay batch at a time,
so nothing per token is kept across batches; whole-vocabulary rows are requested from the
replay only when every rollout that has loss tokens recorded its inference rows.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Optional, Sequence

import torch

from ..engine.rollout import Rollout
from .logprobs import token_logprobs
from .replay import build_sequences, collate


@dataclass
class MismatchReport:
    kl_k3: float  # E_inf[r - 1 - log r], r = p_train / p_inf
    kl_k1: float  # E_inf[log p_inf - log p_train]
    exact_kl: Optional[float]  # full-vocabulary KL when inference rows were recorded
    max_abs_logprob_diff: float
    mean_abs_logprob_diff: float
    num_tokens: int

    def to_dict(self) -> dict:
        return asdict(self)


class _Tally:
    """Float64 running sums of the report's statistics."""

    def __init__(self) -> None:
        self.tokens = 0
        self.k3 = 0.0
        self.k1 = 0.0
        self.abs_max = 0.0
        self.abs_sum = 0.0
        self.rows = 0
        self.kl_sum = 0.0

    def tokens_(self, inf: torch.Tensor, train: torch.Tensor) -> None:
        """Add matched 1-D log-prob vectors (any device, any float dtype)."""
        if inf.numel() == 0:
            return
        d = train.to(torch.float64) - inf.to(device=train.device, dtype=torch.float64)
        a = d.abs()
        self.tokens += d.numel()
        self.k3 += float((torch.expm1(d) - d).sum())
        self.k1 -= float(d.sum())
        self.abs_max = max(self.abs_max, float(a.max()))
        self.abs_sum += float(a.sum())

    def rows_(self, inf_rows: torch.Tensor, train_rows: torch.Tensor) -> None:
        """Add ``[n, V]`` log-softmax rows: sum_v p_inf (log p_inf - log p_train) per row."""
        if inf_rows.numel() == 0:
            return
        li = inf_rows.to(torch.float64)
        lt = train_rows.to(device=li.device, dtype=torch.float64)
        self.kl_sum += float((li.exp() * (li - lt)).sum())
        self.rows += li.shape[0]

    def report(self, with_rows: bool) -> MismatchReport:
        n = self.tokens
        if n == 0:
            return MismatchReport(0.0, 0.0, None, 0.0, 0.0, 0)
        exact = self.kl_sum / self.rows if with_rows and self.rows else None
        return MismatchReport(self.k3 / n, self.k1 / n, exact, self.abs_max, self.abs_sum / n, n)


def mismatch_report(inf_logp: torch.Tensor, train_logp: torch.Tensor, mask: torch.Tensor,
                    inf_full: Optional[torch.Tensor] = None,
                    train_full: Optional[torch.Tensor] = None) -> MismatchReport:
    """The report over the tokens selected by ``mask`` (same shape as the log-prob tensors);
    ``inf_full`` / ``train_full`` are matching ``[..., V]`` rows for the exact KL."""
    tally = _Tally()
    tally.tokens_(inf_logp[mask], train_logp[mask])
    rows = inf_full is not None and train_full is not None
    if rows:
        tally.rows_(inf_full.reshape(-1, inf_full.shape[-1]), train_full.reshape(-1, train_full.shape[-1]))
    return tally.report(rows)


@torch.no_grad()
def measure_mismatch(model, rollouts: Sequence[Rollout], mode: str = "auto", batch_size: int = 8) -> MismatchReport:
    """Replay ``rollouts`` as the trainer would (``mode`` as in :func:`build_sequences`), in
    batches of ``batch_size`` sequences at the temperature of each batch's first rollout, and
    compare with the inference log-probs they recorded."""
    was_training = model.training
    model.eval()
    try:
        with_rows = all(r.full_logprobs for r in rollouts if r.num_loss_tokens)
        work = [(r, seq) for r in rollouts for seq in build_sequences(r, mode)]
        tally = _Tally()
        for lo in range(0, len(work), batch_size):
            part = work[lo:lo + batch_size]
            batch = collate([seq for _, seq in part], device=model.device)
            got = token_logprobs(model, batch, part[0][0].temperature, return_full=with_rows)
            train, full = got if with_rows else (got, None)
            loss = batch.loss_mask.to(train.device)
            for b, (r, seq) in enumerate(part):
                keep = loss[b, : seq.length]
                tally.tokens_(batch.inf_logprobs[b, : seq.length][keep.cpu()], train[b, : seq.length][keep])
                if with_rows:
                    where = torch.nonzero(keep).flatten()
                    inf_rows = torch.stack([r.full_logprobs[int(seq.stream_index[j])] for j in where.tolist()]) \
                        if where.numel() else full.new_zeros(0, full.shape[-1])
                    tally.rows_(inf_rows, full[b].index_select(0, where))
        return tally.report(with_rows)
    finally:
        model.train(was_training)
