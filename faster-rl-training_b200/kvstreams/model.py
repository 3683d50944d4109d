"""Llama-style decoder with the two forward paths of kvstreams/model.py:1-188.

* :meth:`TinyLM.forward` -- full-sequence forward with explicit positions and the
  KV-streams replay mask; attention runs in the masked replay kernel, which skips
  fully hidden tiles (the trainer's replay).
* :meth:`TinyLM.forward_cached` -- incremental forward through a
  :class:`~kvstreams.paged_cache.PagedKVCache`; per layer one call rotates q/k at
  their logical positions, appends k/v to the paged pool and attends to every live
  entry (prefill and decode).  :meth:`TinyLM.forward_cached_batch` does the same
  for many sequences at once.

Module and parameter names equal the reference's, so state dicts load unchanged.
Dense projections stay in PyTorch (cuBLAS); attention, RoPE, every cache operation and, for
half-precision models, RMSNorm and the MLP's silu(gate) * up are this library's kernels.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.nn.functional as F
from torch import nn

from . import _native
from . import _native as N
from . import ops
from .config import ModelConfig
from .ops import ReplayMask
from .rope import RotaryEmbedding


def _half_kernels(x: torch.Tensor, width: int) -> bool:
    """bf16/fp16 CUDA rows of a width the library's elementwise kernels take (fp32/fp64 models
    keep PyTorch's ops, whose rounding the reference shares)."""
    return x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and width % 8 == 0


class _RMSNormFn(torch.autograd.Function):
    """RMSNorm (model.py:29-36) as one kernel pass; backward (one pass, deterministic weight
    gradient) from the saved per-row rstd."""

    @staticmethod
    def forward(ctx, x, w, eps):
        y, rstd = ops.rms_norm(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w, rstd = ctx.saved_tensors
        gx, gw = ops.rms_norm_backward(x, w, rstd, gy)
        return gx, gw.to(w.dtype), None


class _SiluMulFn(torch.autograd.Function):
    """silu(gate) * up of the fused gate|up output (model.py:78-86) in one pass, and its backward."""

    @staticmethod
    def forward(ctx, gu):
        ctx.save_for_backward(gu)
        return ops.silu_mul(gu)

    @staticmethod
    def backward(ctx, go):
        (gu,) = ctx.saved_tensors
        return ops.silu_mul_backward(gu, go)


def _silu_mul(gu: torch.Tensor) -> torch.Tensor:
    if _half_kernels(gu, gu.shape[-1] // 2):
        return _SiluMulFn.apply(gu)
    g, u = gu.chunk(2, dim=-1)
    return F.silu(g) * u


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # x * rsqrt(mean(x^2) + eps) * weight: one pass of the library's kernel for half precision
        # (fp32 reduction and arithmetic), PyTorch's fused op otherwise
        if _half_kernels(x, x.shape[-1]) and self.weight.dtype == x.dtype:
            return _RMSNormFn.apply(x, self.weight, self.eps)
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


def _fused_weight(owner: nn.Module, name: str, parts) -> torch.Tensor:
    """Row-concatenation of several Linear weights, cached on ``owner`` and rebuilt when any
    of them is replaced or updated in place, so one GEMM serves several projections."""
    key = tuple((w.data_ptr(), w._version) for w in parts)
    cached = owner.__dict__.get(name)
    if cached is None or cached[0] != key or torch.is_grad_enabled():
        w = torch.cat(list(parts), dim=0)
        if torch.is_grad_enabled():
            return w  # differentiable, not cached
        owner.__dict__[name] = (key, w)
        return w
    return cached[1]


class Attention(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.n_heads = cfg.n_heads
        self.n_kv_heads = cfg.n_kv_heads
        self.head_dim = cfg.head_dim
        self.scale = self.head_dim ** -0.5  # model.py:71
        self.q_proj = nn.Linear(cfg.d_model, cfg.n_heads * cfg.head_dim, bias=False)
        self.k_proj = nn.Linear(cfg.d_model, cfg.n_kv_heads * cfg.head_dim, bias=False)
        self.v_proj = nn.Linear(cfg.d_model, cfg.n_kv_heads * cfg.head_dim, bias=False)
        self.o_proj = nn.Linear(cfg.n_heads * cfg.head_dim, cfg.d_model, bias=False)

    def project_qkv(self, x: torch.Tensor) -> torch.Tensor:
        """The fused ``[..., (Hq + 2 Hkv) D]`` q|k|v projection of ``x`` (one GEMM over the
        concatenated projection weights)."""
        w = _fused_weight(self, "_qkv", (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight))
        return F.linear(x, w)

    def project(self, x: torch.Tensor):
        """q, k, v of ``x``: views of :meth:`project_qkv`'s output."""
        lead = x.shape[:-1]
        qkv = self.project_qkv(x)
        nq, nk = self.n_heads * self.head_dim, self.n_kv_heads * self.head_dim
        q = qkv[..., :nq].reshape(*lead, self.n_heads, self.head_dim)
        k = qkv[..., nq:nq + nk].reshape(*lead, self.n_kv_heads, self.head_dim)
        v = qkv[..., nq + nk:].reshape(*lead, self.n_kv_heads, self.head_dim)
        return q, k, v


class MLP(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.gate = nn.Linear(cfg.d_model, cfg.d_ff, bias=False)
        self.up = nn.Linear(cfg.d_model, cfg.d_ff, bias=False)
        self.down = nn.Linear(cfg.d_ff, cfg.d_model, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # gate and up as one GEMM over the concatenated weights
        gu = F.linear(x, _fused_weight(self, "_gate_up", (self.gate.weight, self.up.weight)))
        return self.down(_silu_mul(gu))


class Block(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.attn_norm = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.attn = Attention(cfg)
        self.mlp_norm = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.mlp = MLP(cfg)

    # Residual updates of rows ``x [N, d_model]``: x + o_proj(a) and x + mlp(mlp_norm(x))
    # (model.py:149-152 order), the output projection and the add as one GEMM.
    def attn_residual(self, x: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
        return torch.addmm(x, a, self.attn.o_proj.weight.t())

    def mlp_residual(self, x: torch.Tensor) -> torch.Tensor:
        h = self.mlp_norm(x)
        gu = F.linear(h, _fused_weight(self.mlp, "_gate_up", (self.mlp.gate.weight, self.mlp.up.weight)))
        return torch.addmm(x, _silu_mul(gu), self.mlp.down.weight.t())


def causal_mask(T: int, device=None) -> torch.Tensor:
    return torch.ones(T, T, dtype=torch.bool, device=device).tril()


class _ReplayAttention(torch.autograd.Function):
    """RoPE of q/k at ``positions`` plus masked replay attention, as one autograd node over the
    fused q|k|v projection output ``qkv [B, T, (Hq + 2 Hkv) D]``; ``heads`` = (Hq, Hkv, D).

    Backward: the replay attention backward kernels give the gradients of the rotated q/k and of
    v; RoPE is a rotation, so its backward rotates back (RoPE at -positions), written straight
    into the column blocks of the fused gradient (no zero-filled slice gradients to add up)."""

    @staticmethod
    def forward(ctx, qkv, heads, positions, evicted_at, lengths, inv_freq, scale):
        Hq, Hkv, D = heads
        B, T, _ = qkv.shape
        nq, nk = Hq * D, Hkv * D
        qkv = qkv.detach()
        # rotated copies straight out of the projection output, one pass each
        q = ops.rope(qkv[..., :nq].view(B, T, Hq, D), positions, inv_freq)
        k = ops.rope(qkv[..., nq:nq + nk].view(B, T, Hkv, D), positions, inv_freq)
        v = qkv[..., nq + nk:].reshape(B, T, Hkv, D).contiguous()
        grads = ctx.needs_input_grad[0]
        lse = ops.row_lse_buffer(B, Hq, T, q.device) if grads else None
        out = ops.replay_attention(q, k, v, evicted_at, lengths, scale, row_lse=lse)
        if grads:
            ctx.save_for_backward(q, k, v, out, positions, evicted_at, lengths, inv_freq, lse)
        ctx.scale, ctx.heads = scale, heads
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, out, positions, evicted_at, lengths, inv_freq, lse = ctx.saved_tensors
        dq, dk, dv = ops.replay_attention_backward(q, k, v, evicted_at, lengths, ctx.scale, out, grad_out, row_lse=lse)
        Hq, Hkv, D = ctx.heads
        B, T = dq.shape[:2]
        nq, nk = Hq * D, Hkv * D
        dqkv = torch.empty(B, T, nq + 2 * nk, dtype=dq.dtype, device=dq.device)
        neg = -positions
        ops.rope(dq, neg, inv_freq, out=dqkv[..., :nq].view(B, T, Hq, D))
        ops.rope(dk, neg, inv_freq, out=dqkv[..., nq:nq + nk].view(B, T, Hkv, D))
        dqkv[..., nq + nk:].copy_(dv.view(B, T, nk))
        return dqkv, None, None, None, None, None, None


def as_replay_mask(mask, B: int, T: int, device) -> ReplayMask:
    if mask is None:
        return ReplayMask.causal(B, T, device)
    if isinstance(mask, ReplayMask):
        return mask.to(device)
    m = mask.to(device)
    if m.dim() == 3 and m.shape[0] == 1 and B > 1:
        m = m.expand(B, T, T)
    return ReplayMask.from_dense(m)


class TinyLM(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList(Block(cfg) for _ in range(cfg.n_layers))
        self.norm = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        self.rope = RotaryEmbedding(cfg.head_dim, cfg.rope_theta)
        self.apply(self._init_weights)

    def _init_weights(self, module: nn.Module) -> None:
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, mean=0.0, std=self.cfg.init_std)

    @property
    def device(self) -> torch.device:
        return self.embed.weight.device

    @property
    def dtype(self) -> torch.dtype:
        return self.embed.weight.dtype

    @property
    def attention_dtype(self) -> torch.dtype:
        """Element type of q/k/v, the KV cache and the attention kernels: the model's dtype unless
        set otherwise (e.g. ``torch.bfloat16`` under float32 weights: bf16 KV pool and bf16
        attention kernels, everything else in float32).  The paged cache must have this dtype."""
        return self.__dict__.get("_attention_dtype") or self.dtype

    @attention_dtype.setter
    def attention_dtype(self, dtype: Optional[torch.dtype]) -> None:
        self.__dict__["_attention_dtype"] = dtype

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        """lm_head of final hidden states.  Half-precision models accumulate and return the
        logits in float32 (one GEMM with a float32 result): a bf16 logit of magnitude ~4 would
        carry a rounding step of 2^-5, more than the replay-vs-inference log-prob tolerance."""
        w = self.lm_head.weight
        if w.dtype in (torch.bfloat16, torch.float16) and h.is_cuda:
            flat = h.reshape(-1, h.shape[-1])
            return torch.mm(flat, w.t(), out_dtype=torch.float32).view(*h.shape[:-1], w.shape[0])
        return self.lm_head(h)

    # ------------------------------------------------------------------ replay path
    def forward_hidden(self, tokens: torch.Tensor, positions: Optional[torch.Tensor] = None, mask=None) -> torch.Tensor:
        """Final normed hidden states ``[B, T, d_model]`` of the masked full-sequence forward."""
        B, T = tokens.shape
        dev = self.device
        tokens = tokens.to(dev)
        if positions is None:
            positions = torch.arange(T, device=dev).expand(B, T)
        positions = positions.to(dev)
        rm = as_replay_mask(mask, B, T, dev)
        adt = self.attention_dtype
        inv = self.rope.table(dev, adt)
        x = self.embed(tokens)
        for blk in self.layers:
            at = blk.attn
            qkv = at.project_qkv(blk.attn_norm(x))
            a = _ReplayAttention.apply(qkv.to(adt), (at.n_heads, at.n_kv_heads, at.head_dim), positions,
                                       rm.evicted_at, rm.lengths, inv, at.scale)
            x2 = blk.attn_residual(x.reshape(B * T, -1), a.reshape(B * T, -1).to(x.dtype))
            x = blk.mlp_residual(x2).view(B, T, -1)
        return self.norm(x)

    def forward(self, tokens: torch.Tensor, positions: Optional[torch.Tensor] = None, mask=None) -> torch.Tensor:
        """Full-sequence forward (model.py:132-157).

        mask: None (causal), a :class:`ReplayMask`, or a dense ``[B, T, T]`` boolean mask of
        KV-streams form (``s <= t and t < evicted_at[s]``).  Returns ``[B, T, vocab]`` logits."""
        return self.logits(self.forward_hidden(tokens, positions, mask))

    # ------------------------------------------------------------------ paged path
    @torch.no_grad()
    def forward_cached(self, tokens: torch.Tensor, positions: torch.Tensor, cache, seq_id: int) -> torch.Tensor:
        """Incremental forward of one sequence (model.py:160-188); returns ``[T, vocab]``."""
        T = tokens.numel()
        return self.forward_cached_batch(tokens.reshape(T), positions.reshape(T), cache, [seq_id], counts=[T])

    @torch.no_grad()
    def forward_cached_batch(self, tokens: torch.Tensor, positions: torch.Tensor, cache, seq_ids: Sequence[int],
                             counts: Optional[Sequence[int]] = None, last_only: bool = False) -> torch.Tensor:
        """Incremental forward of many sequences: ``tokens``/``positions`` concatenate the new
        tokens of each sequence in order (``counts`` per sequence, default one each).
        Returns logits of every new token (or only of each sequence's last one)."""
        dev = self.device
        tokens = tokens.to(dev).reshape(-1)
        positions = positions.to(dev, torch.long).reshape(-1)
        one_each = counts is None or all(c == 1 for c in counts)
        mapping = cache.append_slots_batch(seq_ids, positions, None if one_each else counts)
        slots = [cache.slot(s) for s in seq_ids]
        batch = cache._batch(slots, None if one_each else counts)  # shared by every layer
        ends = None
        if last_only and not one_each:
            ends = N.to_device(counts, torch.long, dev).cumsum(0) - 1
        return self.forward_layers(tokens, positions, cache, batch, mapping, None if one_each else counts, ends)

    @torch.no_grad()
    def forward_layers(self, tokens: torch.Tensor, positions: torch.Tensor, cache, batch, mapping,
                       counts: Optional[Sequence[int]] = None, rows: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The layers and logits of :meth:`forward_cached_batch` once the slots are appended:
        ``batch`` (kvs_batch, keep-alive) and ``mapping`` describe the new tokens; with ``rows``
        only those tokens' logits.  Device work only (CUDA-graph capturable with static inputs)."""
        N = tokens.numel()
        # trailing one-token sequences of a chunked batch run on the decode kernel
        tail = 0
        if counts is not None:
            while tail < len(counts) and counts[len(counts) - 1 - tail] == 1:
                tail += 1
        adt = self.attention_dtype
        inv = self.rope.table(self.device, adt)
        x = self.embed(tokens)
        for i, blk in enumerate(self.layers):
            q, k, v = blk.attn.project(blk.attn_norm(x))
            if adt != q.dtype:
                q, k, v = q.to(adt), k.to(adt), v.to(adt)
            # every layer has the same batch: the first stores the decode kernel's plan, the
            # others reuse it
            a = ops.paged_forward(cache, None, counts, i, q, k, v, positions, mapping, inv, blk.attn.scale,
                                  batch=batch, tail_singles=tail,
                                  plan=_native.PLAN_BUILD if i == 0 else _native.PLAN_REUSE)
            x = blk.mlp_residual(blk.attn_residual(x, a.reshape(N, -1).to(x.dtype)))
        if rows is not None:
            x = x.index_select(0, rows)
        return self.logits(self.norm(x))
