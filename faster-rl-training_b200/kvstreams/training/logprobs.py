"""Trainer-side log-probabilities (training/logprobs.py:10-25)."""

from __future__ import annotations

import torch

from .. import ops
from .replay import Batch

# tokens per lm_head chunk: bounds the [chunk, vocab] logits held at once
_CHUNK_TOKENS = 8192


class _LmHeadLogprob(torch.autograd.Function):
    """One chunk of lm_head -> log_softmax(logits / T) -> gather (logprobs.py:17-20).

    Forward: for a bf16 lm_head, one tensor-core GEMM whose epilogue reduces each 256-wide
    vocab tile of every row (``kvs_lm_head_logprobs``: the logits are never stored); otherwise
    the lm_head GEMM (cuBLAS) and one pass over each logits row (``kvs_lse_gather``).  Only the
    hidden states and each row's log-sum-exp are kept; backward recomputes the chunk's logits,
    turns them into dlogits = g (onehot - softmax) / T in place (``kvs_lse_gather_backward``,
    in the weight's dtype) and runs the two GEMMs of dh and dW."""

    @staticmethod
    def forward(ctx, h, weight, targets, temperature, model):
        if ops.lm_head_logprobs_supported(h, weight):
            logp, lse = ops.lm_head_logprobs(h, weight, targets, temperature)
        else:
            logits = model.logits(h)
            if logits.dtype in (torch.bfloat16, torch.float16):
                logits = logits.float()
            logp, lse = ops.lse_gather(logits, targets, temperature)
        ctx.save_for_backward(h, weight, targets, lse)
        ctx.temperature, ctx.model = temperature, model
        return logp

    @staticmethod
    def backward(ctx, g):
        h, weight, targets, lse = ctx.saved_tensors
        logits = ctx.model.logits(h)
        if logits.dtype in (torch.bfloat16, torch.float16):
            logits = logits.float()
        if weight.dtype == logits.dtype:
            dlog = ops.lse_gather_backward(logits, targets, lse, g, ctx.temperature, out=logits)
        else:
            dlog = ops.lse_gather_backward(logits, targets, lse, g, ctx.temperature, out_dtype=weight.dtype)
        del logits
        dh = dlog @ weight if ctx.needs_input_grad[0] else None
        dw = dlog.t() @ h.to(weight.dtype) if ctx.needs_input_grad[1] else None
        return dh, dw, None, None, None


def token_logprobs(model, batch: Batch, temperature: float = 1.0, return_full: bool = False):
    """Log-probability of ``tokens[:, t]`` given the replayed context of ``t - 1``.

    Returns ``[B, T]`` (position 0 is 0); with ``return_full`` also the ``[B, T, V]``
    log-softmax rows aligned the same way.  The replay forward runs the masked replay
    kernel; lm_head + log-softmax + gather are done in token chunks so the full
    ``[B, T, V]`` logits never exist at once.  Half-precision models get float32 logits
    (float32 accumulation, no half-precision rounding) and float32 log-softmax.
    """
    dev = model.device
    tokens = batch.tokens.to(dev)
    hidden = model.forward_hidden(tokens, batch.positions.to(dev), batch.mask.to(dev))
    B, T, _ = hidden.shape
    want = torch.float32 if hidden.dtype in (torch.bfloat16, torch.float16) else hidden.dtype
    out = torch.zeros((B, T), dtype=want, device=dev)
    full = torch.zeros((B, T, model.cfg.vocab_size), dtype=want, device=dev) if return_full else None
    flat_h = hidden[:, :-1].reshape(-1, hidden.shape[-1])
    flat_next = tokens[:, 1:].reshape(-1)
    if full is None and flat_h.is_cuda:
        # fused path: lm_head GEMM + one pass per row, recomputed in backward
        parts = [_LmHeadLogprob.apply(flat_h[a:a + _CHUNK_TOKENS], model.lm_head.weight,
                                      flat_next[a:a + _CHUNK_TOKENS], float(temperature), model)
                 for a in range(0, flat_h.shape[0], _CHUNK_TOKENS)]
        res = torch.cat(parts) if parts else torch.empty(0, dtype=want, device=dev)
        out = torch.cat([torch.zeros(B, 1, dtype=res.dtype, device=dev), res.view(B, T - 1)], dim=1)
        return out
    res = torch.empty(flat_next.numel(), dtype=want, device=dev)
    for a in range(0, flat_h.shape[0], _CHUNK_TOKENS):
        z = slice(a, a + _CHUNK_TOKENS)
        logits = model.logits(flat_h[z]).to(want)
        logp = torch.log_softmax(logits / temperature, dim=-1)
        res[z] = logp.gather(-1, flat_next[z, None]).squeeze(-1)
        if full is not None:
            rows = torch.arange(a, a + logp.shape[0], device=dev)
            full[rows // (T - 1), rows % (T - 1) + 1] = logp
    out[:, 1:] = res.view(B, T - 1)
    if not return_full:
        return out
    return out, full
