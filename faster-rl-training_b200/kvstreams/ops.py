"""PyTorch-facing wrappers of the libkvs_b200.so kernels.

Every function here launches this library's own sm_100a kernels on the current
CUDA stream; none has a CPU implementation.  Tensors must already be on the GPU.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np
import torch

from . import _native as N

NEVER = N.NEVER


def _check_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        N.require_cuda(t, "tensor")


def rope_(x: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """Rotate ``x [..., H, D]`` in place at ``positions [...]`` (rope.py:42-46 semantics)."""
    _check_cuda(x)
    if not x.is_contiguous():
        raise ValueError("rope_ needs a contiguous tensor")
    H, D = x.shape[-2], x.shape[-1]
    n = x.numel() // (H * D)
    pos = positions.reshape(-1).to(device=x.device, dtype=torch.long).contiguous()
    if pos.numel() != n:
        raise ValueError("positions do not match x")
    rc = N.lib().kvs_rope(x.data_ptr(), N.DTYPE_CODE[x.dtype], pos.data_ptr(), n, H, D, inv_freq.data_ptr(),
                          N.stream_ptr(x.device))
    N.check(rc, "kvs_rope")
    return x


def evicted_at_device(logs: Sequence, lengths: Sequence[int], device: torch.device,
                      t_stride: Optional[int] = None) -> torch.Tensor:
    """``[len(logs), t_stride]`` int64 evicted_at of each compaction log (events.py:66-74),
    computed by the evicted_at kernel; entries past a stream's length are NEVER."""
    triples = [log.span_triples() for log in logs]
    cu = np.zeros(len(logs) + 1, dtype=np.int32)
    np.cumsum([len(t) for t in triples], out=cu[1:])
    flat = np.concatenate(triples, axis=0) if triples else np.zeros((0, 3), dtype=np.int64)
    if flat.shape[0] == 0:
        flat = np.zeros((1, 3), dtype=np.int64)
    T = int(t_stride if t_stride is not None else (max(lengths) if len(lengths) else 0))
    return evicted_at_from_spans(cu, flat, lengths, device, T)


def evicted_at_from_spans(cu: np.ndarray, triples: np.ndarray, lengths: Sequence[int], device, t_stride: int):
    dev = torch.device(device)
    out = torch.empty((len(lengths), max(t_stride, 1)), dtype=torch.long, device=dev)
    cu_t = torch.from_numpy(np.ascontiguousarray(cu, dtype=np.int32)).to(dev)
    tr = np.ascontiguousarray(triples, dtype=np.int64)
    ss = torch.from_numpy(np.ascontiguousarray(tr[:, 0])).to(dev)
    se = torch.from_numpy(np.ascontiguousarray(tr[:, 1])).to(dev)
    st = torch.from_numpy(np.ascontiguousarray(tr[:, 2])).to(dev)
    ln = torch.as_tensor(np.asarray(lengths, dtype=np.int32)).to(dev)
    with torch.cuda.device(dev):
        rc = N.lib().kvs_evicted_at(cu_t.data_ptr(), ss.data_ptr(), se.data_ptr(), st.data_ptr(), ln.data_ptr(),
                                    len(lengths), max(t_stride, 1), out.data_ptr(), N.stream_ptr(dev))
    N.check(rc, "kvs_evicted_at")
    return out[:, :t_stride]


def replay_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, evicted_at: torch.Tensor,
                     lengths: torch.Tensor, scale: float, out: Optional[torch.Tensor] = None,
                     force_generic: bool = False, one_head_per_cta: bool = False,
                     row_lse: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Masked replay attention (model.py:71-74 with the replay.py:62 mask).

    q ``[B, T, Hq, D]``, k/v ``[B, T, Hkv, D]`` already rotated; evicted_at ``[B, T]``
    int64; lengths ``[B]`` int32 (rows past the length attend to themselves only).
    ``force_generic`` selects the exact SIMT kernel; ``one_head_per_cta`` keeps the
    tensor-core path on its one-query-head-per-CTA kernel for even GQA group sizes.
    ``row_lse`` (float32 ``[B, Hq, T_pad]``, :func:`row_lse_buffer`) receives each row's
    log2-sum-exp, which :func:`replay_attention_backward` uses."""
    _check_cuda(q, k, v, evicted_at, lengths)
    B, T, Hq, D = q.shape
    Hkv = k.shape[2]
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    ev = evicted_at.to(torch.long).contiguous()
    ln = lengths.to(torch.int32).contiguous()
    if out is None:
        out = torch.empty_like(q)
    lib = N.lib()
    nbytes = lib.kvs_replay_scratch_bytes(B, T)
    scratch = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=q.device)
    a = N.KvsReplayArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), evicted_at=ev.data_ptr(),
                        lengths=ln.data_ptr(), out=out.data_ptr(), scratch=scratch.data_ptr(),
                        scratch_bytes=scratch.numel(), batch=B, seq_len=T, n_heads=Hq, n_kv_heads=Hkv, head_dim=D,
                        dtype=N.DTYPE_CODE[q.dtype], scale=float(scale),
                        flags=(1 if force_generic else 0) | (2 if one_head_per_cta else 0),
                        row_lse=_lse_ptr(row_lse, B, Hq, T))
    N.check(lib.kvs_replay_attention(C.byref(a), N.stream_ptr(q.device)), "kvs_replay_attention")
    return out


def row_lse_buffer(B: int, Hq: int, T: int, device) -> torch.Tensor:
    """Row statistics buffer of the replay forward: float32 ``[B, Hq, T rounded up to 128]``."""
    return torch.empty(B, Hq, (T + 127) // 128 * 128, dtype=torch.float32, device=device)


def _lse_ptr(row_lse: Optional[torch.Tensor], B: int, Hq: int, T: int):
    if row_lse is None:
        return None
    want = (B, Hq, (T + 127) // 128 * 128)
    if tuple(row_lse.shape) != want or row_lse.dtype != torch.float32 or not row_lse.is_contiguous():
        raise ValueError(f"row_lse must be a contiguous float32 tensor of shape {want}")
    return row_lse.data_ptr()


def replay_attention_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, evicted_at: torch.Tensor,
                              lengths: torch.Tensor, scale: float, out: torch.Tensor, grad_out: torch.Tensor,
                              row_lse: Optional[torch.Tensor] = None, force_exact: bool = False,
                              report_path: Optional[list] = None):
    """Gradients (dq, dk, dv) of :func:`replay_attention` (q and k rotated, ``out`` its
    output) for the upstream gradient ``grad_out``.  With the forward's ``row_lse``, bf16
    and head_dim 128 run the tcgen05 kernels; otherwise (or ``force_exact``) the exact
    kernels.  ``report_path`` (a list) receives 1 when the tcgen05 kernels ran, 0 otherwise."""
    _check_cuda(q, k, v, evicted_at, lengths)
    B, T, Hq, D = q.shape
    Hkv = k.shape[2]
    q, k, v, out = q.contiguous(), k.contiguous(), v.contiguous(), out.contiguous()
    g = grad_out.to(q.dtype).contiguous()
    ev = evicted_at.to(torch.long).contiguous()
    ln = lengths.to(torch.int32).contiguous()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    lib = N.lib()
    code = N.DTYPE_CODE[q.dtype]
    nbytes = lib.kvs_replay_backward_scratch_bytes(B, T, Hq, code)
    scratch = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=q.device)
    a = N.KvsReplayArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), evicted_at=ev.data_ptr(),
                        lengths=ln.data_ptr(), out=out.data_ptr(), scratch=scratch.data_ptr(),
                        scratch_bytes=scratch.numel(), batch=B, seq_len=T, n_heads=Hq, n_kv_heads=Hkv, head_dim=D,
                        dtype=code, scale=float(scale), flags=1 if force_exact else 0,
                        row_lse=_lse_ptr(row_lse, B, Hq, T))
    if report_path is not None:
        report_path.append(int(lib.kvs_replay_backward_path(C.byref(a), N.stream_ptr(q.device))))
    N.check(lib.kvs_replay_attention_backward(C.byref(a), g.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                              N.stream_ptr(q.device)), "kvs_replay_attention_backward")
    return dq, dk, dv


def rope(x: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor,
         out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """RoPE of ``x [..., H, D]`` at ``positions [...]`` (rope.py:42-46) in one pass, out of place:
    ``x`` is read where it lies when each token's ``[H][D]`` block is dense (the q or k column
    block of a fused projection output); the result goes to a new contiguous tensor, or to
    ``out`` (same shape, dense token blocks, e.g. a column block of a fused gradient)."""
    _check_cuda(x)
    H, D = x.shape[-2], x.shape[-1]
    lead = tuple(x.shape[:-2])
    n = int(np.prod(lead)) if lead else 1
    rows, stride = _token_rows(x.reshape(n, H, D))
    pos = positions.reshape(-1).to(device=x.device, dtype=torch.long).contiguous()
    if pos.numel() != n:
        raise ValueError("positions do not match x")
    if out is None:
        out = torch.empty(*lead, H, D, dtype=x.dtype, device=x.device)
        dst, dstride = out, 0
    else:
        if out.shape != x.shape or out.dtype != x.dtype or out.device != x.device:
            raise ValueError("out must match x in shape, dtype and device")
        dst = out.reshape(n, H, D)
        if dst.data_ptr() != out.data_ptr() or dst.stride(2) != 1 or dst.stride(1) != D or dst.stride(0) < H * D:
            raise ValueError("out needs dense [H][D] token blocks")
        dstride = int(dst.stride(0))
    rc = N.lib().kvs_rope_copy(rows.data_ptr(), stride, dst.data_ptr(), dstride, N.DTYPE_CODE[x.dtype],
                               pos.data_ptr(), n, H, D, inv_freq.data_ptr(), N.stream_ptr(x.device))
    N.check(rc, "kvs_rope_copy")
    return out


def _token_rows(x: torch.Tensor):
    """``(x, row stride)`` when each token's ``[heads][head_dim]`` block of ``x`` is dense (the
    stride between tokens is then passed to the kernels), else ``(contiguous copy, 0)``."""
    if x.dim() == 3 and x.stride(2) == 1 and x.stride(1) == x.shape[2] and x.stride(0) >= x.shape[1] * x.shape[2]:
        return x, (0 if x.is_contiguous() else int(x.stride(0)))
    return x.contiguous(), 0


def paged_forward(cache, slots: Sequence[int], counts: Optional[Sequence[int]], layer: int, q: torch.Tensor,
                  k_new: torch.Tensor, v_new: torch.Tensor, positions: torch.Tensor, mapping,
                  inv_freq: torch.Tensor, scale: float, out: Optional[torch.Tensor] = None,
                  grid_ctas: int = 0, batch=None, tail_singles: int = 0,
                  report_path: Optional[list] = None, plan: int = 0) -> torch.Tensor:
    """One layer of the paged incremental forward (model.py:50-75 + hook :182-185) for the
    new tokens of a batch of sequences: RoPE of q/k, append of k/v, paged GQA attention.

    q ``[N, Hq, D]``, k_new/v_new ``[N, Hkv, D]`` (not rotated), positions ``[N]``; ``mapping``
    is the SlotMapping returned by append_slots for the same tokens; ``batch`` a descriptor from
    ``cache._batch(slots, counts)`` that the layers of one forward can share; ``tail_singles``
    the number of trailing sequences with exactly one new token (they then run on the decode
    kernel while the chunks before them run on the prefill path, in one call).  ``plan``: 1 on
    the first layer of a decode step stores the decode kernel's batch plan, 2 on the later
    layers of the same step reuses it (same batch, lengths and tables; ``kvs_decode_plan``).
    ``report_path``
    (a list) receives the call's kernel families as ``kvs_paged_decode_path`` bits: 1 fused
    decode, 2 tensor-core prefill, 4 exact kernels."""
    # q, k_new, v_new may be row-strided views (the column blocks of a fused q|k|v projection
    # output): each token's [heads][head_dim] block dense, rows any distance apart
    q, q_stride = _token_rows(q)
    k_new, kv_stride = _token_rows(k_new)
    v_new, v_stride = _token_rows(v_new)
    if v_stride != kv_stride:
        k_new, v_new, kv_stride = k_new.contiguous(), v_new.contiguous(), 0
    if q.dtype != cache.dtype or k_new.dtype != cache.dtype or v_new.dtype != cache.dtype:
        raise ValueError("activations must have the cache dtype")
    pos = positions.to(device=q.device, dtype=torch.long).contiguous()
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    b, keep = batch if batch is not None else cache._batch(slots, counts)
    lib = N.lib()
    nbytes = int(lib.kvs_decode_scratch_bytes(C.byref(cache.struct), b.num_seqs, q.shape[1], grid_ctas))
    scratch = cache._decode_scratch(nbytes) if nbytes else None
    a = N.KvsDecodeArgs(q=q.data_ptr(), k_new=k_new.data_ptr(), v_new=v_new.data_ptr(), positions=pos.data_ptr(),
                        slot_blocks=mapping.blocks.data_ptr(), slot_offsets=mapping.offsets.data_ptr(),
                        inv_freq=inv_freq.data_ptr(), out=out.data_ptr(),
                        scratch=scratch.data_ptr() if scratch is not None else None,
                        scratch_bytes=scratch.numel() if scratch is not None else 0, scale=float(scale),
                        layer=int(layer), n_heads=int(q.shape[1]), grid_ctas=int(grid_ctas),
                        tail_singles=int(tail_singles) if counts is not None else 0,
                        q_stride=q_stride, kv_stride=kv_stride, plan=int(plan))
    if report_path is not None:
        report_path.append(int(lib.kvs_paged_decode_path(C.byref(cache.struct), C.byref(b), C.byref(a))))
    N.check(lib.kvs_paged_decode(C.byref(cache.struct), C.byref(b), C.byref(a), N.stream_ptr(q.device)),
            "kvs_paged_decode")
    return out


@dataclass
class ReplayMask:
    """The KV-streams replay mask in factored form (replay.py:55-63, collate :221-222):
    ``visible(t, s) = s <= t and t < evicted_at[b, s]`` for ``t < lengths[b]``; padded rows
    see only themselves.  Never materialised as ``[B, T, T]`` on the device path."""

    evicted_at: torch.Tensor  # [B, T] int64
    lengths: torch.Tensor  # [B] int32

    def to(self, device) -> "ReplayMask":
        return ReplayMask(self.evicted_at.to(device), self.lengths.to(device))

    @property
    def shape(self):
        B, T = self.evicted_at.shape
        return (B, T, T)

    def dense(self) -> torch.Tensor:
        """``[B, T, T]`` bool mask (for inspection and API compatibility only)."""
        B, T = self.evicted_at.shape
        dev = self.evicted_at.device
        t = torch.arange(T, device=dev)
        m = (t[None, None, :] <= t[None, :, None]) & (t[None, :, None] < self.evicted_at[:, None, :])
        pad = t[None, :] >= self.lengths.to(dev)[:, None].long()  # [B, T] padded query rows
        eye = torch.eye(T, dtype=torch.bool, device=dev)[None]
        m = torch.where(pad[:, :, None] | pad[:, None, :], eye.expand(B, T, T), m)
        return m

    @classmethod
    def causal(cls, B: int, T: int, device) -> "ReplayMask":
        return cls(torch.full((B, T), NEVER, dtype=torch.long, device=device),
                   torch.full((B,), T, dtype=torch.int32, device=device))

    @classmethod
    def from_dense(cls, mask: torch.Tensor) -> "ReplayMask":
        """Factor a dense ``[B, T, T]`` boolean mask; raises if it is not of KV-streams form."""
        if mask.dim() == 2:
            mask = mask[None]
        B, T, _ = mask.shape
        m = mask.to(torch.bool)
        dev = m.device
        t = torch.arange(T, device=dev)
        lower = t[:, None] >= t[None, :]  # [t, s]: s <= t
        # evicted_at[s] = first row t >= s where column s is hidden, else NEVER
        hidden = (~m) & lower[None]
        first = torch.where(hidden, t[None, :, None].expand(B, T, T), torch.full_like(t, T)[None, None, :].expand(B, T, T))
        e = first.min(dim=1).values
        ev = torch.where(e >= T, torch.full_like(e, NEVER), e)
        rm = cls(ev.long(), torch.full((B,), T, dtype=torch.int32, device=dev))
        if not torch.equal(rm.dense(), m):
            raise ValueError(
                "attention mask is not a KV-streams replay mask (s <= t and t < evicted_at[s]); "
                "pass a ReplayMask for padded batches"
            )
        return rm


def lse_gather(logits: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0):
    """``(logp, lse)``: ``log_softmax(logits / T)[r, targets[r]]`` and ``logsumexp(logits[r] / T)``
    for a 2-D float32/float64 CUDA tensor (training/logprobs.py:17-20), one pass per row."""
    _check_cuda(logits, targets)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a 2-D tensor with contiguous rows")
    n, vocab = logits.shape
    t = targets.to(torch.long).contiguous().reshape(-1)
    logp = torch.empty(n, dtype=logits.dtype, device=logits.device)
    lse = torch.empty(n, dtype=logits.dtype, device=logits.device)
    rc = N.lib().kvs_lse_gather(logits.data_ptr(), logits.stride(0), n, vocab, t.data_ptr(), float(temperature),
                                N.DTYPE_CODE[logits.dtype], logp.data_ptr(), lse.data_ptr(), N.stream_ptr(logits.device))
    N.check(rc, "kvs_lse_gather")
    return logp, lse


_LMHEAD_OK: dict = {}


def lm_head_logprobs_supported(h: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether :func:`lm_head_logprobs` can take these operands on this device."""
    if not (h.is_cuda and weight.is_cuda and h.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16):
        return False
    if h.dim() != 2 or weight.dim() != 2 or h.stride(1) != 1 or weight.stride(1) != 1:
        return False
    K = h.shape[1]
    if weight.shape[1] != K or K % 64 or h.stride(0) % 8 or weight.stride(0) % 8:
        return False
    if h.data_ptr() % 16 or weight.data_ptr() % 16:
        return False
    key = (h.device.index, K)
    if key not in _LMHEAD_OK:
        with torch.cuda.device(h.device):
            _LMHEAD_OK[key] = bool(N.lib().kvs_lm_head_logprobs_supported(K))
    return _LMHEAD_OK[key]


def lm_head_logprobs(h: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0):
    """``(logp, lse)`` of ``log_softmax((h @ weight.T) / T)`` at ``targets`` and its log-sum-exp,
    float32, without storing the ``[rows, vocab]`` logits (training/logprobs.py:17-20): one
    tensor-core GEMM whose epilogue reduces each 256-wide vocab tile, then a merge of the tiles.
    h ``[rows, K]`` and weight ``[vocab, K]`` bf16 (see :func:`lm_head_logprobs_supported`)."""
    _check_cuda(h, weight, targets)
    n, K = h.shape
    V = weight.shape[0]
    t = targets.to(torch.long).contiguous().reshape(-1)
    logp = torch.empty(n, dtype=torch.float32, device=h.device)
    lse = torch.empty(n, dtype=torch.float32, device=h.device)
    lib = N.lib()
    nbytes = int(lib.kvs_lm_head_logprobs_scratch_bytes(n, V))
    scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=h.device)
    rc = lib.kvs_lm_head_logprobs(h.data_ptr(), h.stride(0), weight.data_ptr(), weight.stride(0), n, V, K,
                                  t.data_ptr(), float(temperature), logp.data_ptr(), lse.data_ptr(),
                                  scratch.data_ptr(), scratch.numel(), N.stream_ptr(h.device))
    N.check(rc, "kvs_lm_head_logprobs")
    return logp, lse


def sample(logits: torch.Tensor, temperature: float = 1.0, greedy: bool = False, seed: int = 0, offset: int = 0):
    """``(tokens, logp)``: one next token per row of 2-D float32/float64 CUDA logits and its
    ``log_softmax(logits / T)`` value (engine/base.py:180-193), in one launch.  Greedy takes the
    row's argmax (first maximum); otherwise a draw from ``softmax(logits / T)`` by the Gumbel-max
    rule over a Philox4x32-10 stream keyed by ``seed`` and ``offset`` (same pair, same tokens)."""
    _check_cuda(logits)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a 2-D tensor with contiguous rows")
    n, vocab = logits.shape
    tokens = torch.empty(n, dtype=torch.long, device=logits.device)
    logp = torch.empty(n, dtype=logits.dtype, device=logits.device)
    mask = (1 << 64) - 1
    rc = N.lib().kvs_sample(logits.data_ptr(), logits.stride(0), n, vocab, float(temperature),
                            N.DTYPE_CODE[logits.dtype], int(bool(greedy)), int(seed) & mask, int(offset) & mask,
                            tokens.data_ptr(), logp.data_ptr(), N.stream_ptr(logits.device))
    N.check(rc, "kvs_sample")
    return tokens, logp


def lse_gather_backward(logits: torch.Tensor, targets: torch.Tensor, lse: torch.Tensor, grad: torch.Tensor,
                        temperature: float = 1.0, out_dtype: Optional[torch.dtype] = None,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gradient of :func:`lse_gather`'s logp with respect to the logits for upstream ``grad``,
    in ``out_dtype`` (default the logits' dtype); ``out`` may be ``logits`` itself."""
    n, vocab = logits.shape
    out_dtype = out_dtype or logits.dtype
    if out is None:
        out = torch.empty(n, vocab, dtype=out_dtype, device=logits.device)
    t = targets.to(torch.long).contiguous().reshape(-1)
    g = grad.to(logits.dtype).contiguous()
    rc = N.lib().kvs_lse_gather_backward(logits.data_ptr(), logits.stride(0), n, vocab, t.data_ptr(), lse.data_ptr(),
                                         g.data_ptr(), float(temperature), N.DTYPE_CODE[logits.dtype], out.data_ptr(),
                                         out.stride(0), N.DTYPE_CODE[out.dtype], N.stream_ptr(logits.device))
    N.check(rc, "kvs_lse_gather_backward")
    return out


def _rows2d(x: torch.Tensor) -> torch.Tensor:
    """``x`` as a 2-D ``[rows, last]`` tensor with contiguous rows (a view when possible)."""
    if x.stride(-1) != 1:
        x = x.contiguous()
    try:
        return x.view(-1, x.shape[-1])
    except RuntimeError:
        return x.contiguous().view(-1, x.shape[-1])


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float):
    """``(y, rstd)``: RMSNorm of the last dimension (model.py:29-36) for bf16/fp16 CUDA tensors,
    fp32 arithmetic with one rounding; ``rstd`` float32 per row."""
    _check_cuda(x, weight)
    x2 = _rows2d(x)
    y = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
    rc = N.lib().kvs_rms_norm(x2.data_ptr(), weight.contiguous().data_ptr(), y.data_ptr(), rstd.data_ptr(),
                              x2.shape[0], x2.shape[1], x2.stride(0), y.stride(0), float(eps), N.DTYPE_CODE[x.dtype],
                              N.stream_ptr(x.device))
    N.check(rc, "kvs_rms_norm")
    return y.view(x.shape), rstd.view(x.shape[:-1])


def rms_norm_backward(x: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor, gy: torch.Tensor):
    """``(gx, gw)``: gradients of :func:`rms_norm` for the upstream ``gy`` with the forward's
    ``rstd``, one pass over the rows; ``gw`` float32, summed in a fixed order (deterministic)."""
    _check_cuda(x, weight, rstd, gy)
    x2, g2 = _rows2d(x), _rows2d(gy.to(x.dtype))
    n, dim = x2.shape
    gx = torch.empty(n, dim, dtype=x.dtype, device=x.device)
    gw = torch.empty(dim, dtype=torch.float32, device=x.device)
    r = rstd.reshape(-1).to(torch.float32).contiguous()
    lib = N.lib()
    scratch = torch.empty(max(int(lib.kvs_rms_norm_backward_scratch_bytes(n, dim)) // 4, 1), dtype=torch.float32,
                          device=x.device)
    rc = lib.kvs_rms_norm_backward(x2.data_ptr(), weight.contiguous().data_ptr(), r.data_ptr(), g2.data_ptr(),
                                   gx.data_ptr(), gw.data_ptr(), n, dim, x2.stride(0), g2.stride(0), gx.stride(0),
                                   N.DTYPE_CODE[x.dtype], scratch.data_ptr(), scratch.numel() * 4,
                                   N.stream_ptr(x.device))
    N.check(rc, "kvs_rms_norm_backward")
    return gx.view(x.shape), gw


def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` of a fused ``[..., 2F]`` gate|up tensor (model.py:78-86), one pass."""
    _check_cuda(gu)
    g2 = _rows2d(gu)
    f = g2.shape[1] // 2
    out = torch.empty(g2.shape[0], f, dtype=gu.dtype, device=gu.device)
    rc = N.lib().kvs_silu_mul(g2.data_ptr(), out.data_ptr(), g2.shape[0], f, g2.stride(0), out.stride(0),
                              N.DTYPE_CODE[gu.dtype], N.stream_ptr(gu.device))
    N.check(rc, "kvs_silu_mul")
    return out.view(*gu.shape[:-1], f)


def silu_mul_backward(gu: torch.Tensor, grad: torch.Tensor) -> torch.Tensor:
    """Gradient of :func:`silu_mul` with respect to ``gu`` (``[..., 2F]``)."""
    g2 = _rows2d(gu)
    d2 = _rows2d(grad.to(gu.dtype))
    dgu = torch.empty(g2.shape, dtype=gu.dtype, device=gu.device)
    rc = N.lib().kvs_silu_mul_backward(g2.data_ptr(), d2.data_ptr(), dgu.data_ptr(), g2.shape[0], g2.shape[1] // 2,
                                       g2.stride(0), d2.stride(0), dgu.stride(0), N.DTYPE_CODE[gu.dtype],
                                       N.stream_ptr(gu.device))
    N.check(rc, "kvs_silu_mul_backward")
    return dgu.view(gu.shape)
