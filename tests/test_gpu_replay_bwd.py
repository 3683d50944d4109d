"""Replay attention backward: gradients of the masked replay attention against torch
autograd through a dense masked attention (fp64 1e-10, fp32 1e-4, bf16 on bf16 inputs 5e-2
absolute on O(1) gradients), and TinyLM parameter gradients through token_logprobs against a
pure-torch dense-mask model (fp64 1e-9)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dense_mask(ev, lengths, T):
    t = torch.arange(T)[:, None]
    s = torch.arange(T)[None, :]
    masks = []
    for b in range(ev.shape[0]):
        L = int(lengths[b])
        m = (s <= t) & (t < ev[b][None, :].cpu())
        pad = (t >= L) & (s == t)
        masks.append(torch.where(t >= L, pad, m))
    return torch.stack(masks)  # [B, T, T]


def _dense_attention(q, k, v, mask, scale):
    B, T, Hq, D = q.shape
    G = Hq // k.shape[2]
    kk = k.repeat_interleave(G, dim=2)
    vv = v.repeat_interleave(G, dim=2)
    sc = torch.einsum("bthd,bshd->bhts", q, kk) * scale
    sc = sc.masked_fill(~mask[:, None], float("-inf"))
    p = torch.softmax(sc, dim=-1)
    return torch.einsum("bhts,bshd->bthd", p, vv)


def _case(dtype, D, Hq, Hkv, B=2, T=90, lengths=(90, 61), seed=0):
    from kvstreams.workloads import replay_evicted_at

    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, T, Hq, D, generator=g, device="cuda", dtype=torch.float64)
    k = torch.randn(B, T, Hkv, D, generator=g, device="cuda", dtype=torch.float64)
    v = torch.randn(B, T, Hkv, D, generator=g, device="cuda", dtype=torch.float64)
    go = torch.randn(B, T, Hq, D, generator=g, device="cuda", dtype=torch.float64)
    ev, _ = replay_evicted_at(batch=B, seq_len=T, events_range=(2, 4), mean_turn=12, seed=seed)
    ev_t = torch.from_numpy(ev).cuda()
    ln = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    return [x.to(dtype) for x in (q, k, v, go)] + [ev_t, ln]


@pytest.mark.parametrize("dtype,D,Hq,Hkv,tol", [
    (torch.float64, 16, 4, 2, 1e-10),
    (torch.float64, 128, 4, 4, 1e-10),
    (torch.float32, 128, 8, 2, 1e-4),
    (torch.bfloat16, 128, 8, 2, 5e-2),
])
def test_replay_backward_matches_autograd(dtype, D, Hq, Hkv, tol):
    from kvstreams import ops

    q, k, v, go, ev, ln = _case(dtype, D, Hq, Hkv, seed=D + Hq)
    scale = D ** -0.5
    out = ops.replay_attention(q, k, v, ev, ln, scale)
    dq, dk, dv = ops.replay_attention_backward(q, k, v, ev, ln, scale, out, go)
    # reference on the same (possibly rounded) inputs, in float64
    qr, kr, vr = (x.detach().double().requires_grad_() for x in (q, k, v))
    mask = _dense_mask(ev, ln.cpu(), q.shape[1]).cuda()
    ref = _dense_attention(qr, kr, vr, mask, scale)
    ref.backward(go.double())
    for got, want, name in ((dq, qr.grad, "dq"), (dk, kr.grad, "dk"), (dv, vr.grad, "dv")):
        err = (got.double() - want).abs().max().item()
        assert err <= tol, f"{name}: {err}"


def _torch_rope(x, pos, inv):
    ang = pos.to(inv.dtype)[..., None] * inv  # [B, T, D/2]
    c, s = torch.cos(ang)[:, :, None, :], torch.sin(ang)[:, :, None, :]
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def _dense_tinylm_logprobs(model, tokens, positions, mask):
    """TinyLM forward (model.py:132-157) with torch ops only and a dense mask."""
    import torch.nn.functional as F

    cfg = model.cfg
    inv = model.rope.table(tokens.device, model.dtype)
    x = model.embed(tokens)
    B, T = tokens.shape
    for blk in model.layers:
        h = F.rms_norm(x, (x.shape[-1],), blk.attn_norm.weight, blk.attn_norm.eps)
        a = blk.attn
        q = a.q_proj(h).view(B, T, a.n_heads, a.head_dim)
        k = a.k_proj(h).view(B, T, a.n_kv_heads, a.head_dim)
        v = a.v_proj(h).view(B, T, a.n_kv_heads, a.head_dim)
        q, k = _torch_rope(q, positions, inv), _torch_rope(k, positions, inv)
        o = _dense_attention(q, k, v, mask, a.scale)
        x = x + a.o_proj(o.reshape(B, T, -1))
        h = F.rms_norm(x, (x.shape[-1],), blk.mlp_norm.weight, blk.mlp_norm.eps)
        x = x + blk.mlp.down(F.silu(blk.mlp.gate(h)) * blk.mlp.up(h))
    x = F.rms_norm(x, (x.shape[-1],), model.norm.weight, model.norm.eps)
    logp = torch.log_softmax(model.lm_head(x), dim=-1)
    out = torch.zeros(B, T, dtype=logp.dtype, device=logp.device)
    out[:, 1:] = logp[:, :-1].gather(-1, tokens[:, 1:, None]).squeeze(-1)
    return out


def test_tinylm_gradients_through_token_logprobs_fp64():
    from kvstreams.config import ModelConfig
    from kvstreams.model import TinyLM
    from kvstreams.training.logprobs import token_logprobs
    from kvstreams.training.replay import Batch
    from kvstreams.workloads import replay_evicted_at

    torch.manual_seed(0)
    cfg = ModelConfig()
    with torch.device("cuda"):
        model = TinyLM(cfg).double()
    B, T = 2, 72
    ev, _ = replay_evicted_at(batch=B, seq_len=T, events_range=(2, 4), mean_turn=10, seed=5)
    tokens = torch.randint(1, cfg.vocab_size, (B, T), device="cuda")
    lengths = torch.tensor([T, 50], device="cuda")
    positions = torch.arange(T, device="cuda").expand(B, T)
    batch = Batch(tokens, positions, torch.from_numpy(ev).cuda(), torch.ones(B, T, dtype=torch.bool, device="cuda"),
                  torch.zeros(B, T, dtype=torch.float64, device="cuda"), lengths)
    w = torch.randn(B, T, dtype=torch.float64, device="cuda")
    (token_logprobs(model, batch) * w).sum().backward()
    got = {n: p.grad.clone() for n, p in model.named_parameters()}
    model.zero_grad()
    mask = _dense_mask(torch.from_numpy(ev), lengths.cpu(), T).cuda()
    (_dense_tinylm_logprobs(model, tokens, positions, mask) * w).sum().backward()
    for n, p in model.named_parameters():
        err = (got[n] - p.grad).abs().max().item()
        assert err <= 1e-9, f"{n}: {err}"


def _dense_lse2(q, k, mask, scale):
    B, T, Hq, D = q.shape
    G = Hq // k.shape[2]
    kk = k.double().repeat_interleave(G, dim=2)
    sc = torch.einsum("bthd,bshd->bhts", q.double(), kk) * scale
    sc = sc.masked_fill(~mask[:, None], float("-inf"))
    return torch.logsumexp(sc, dim=-1) / np.log(2.0)  # [B, Hq, T]


@pytest.mark.parametrize("dtype,generic", [(torch.bfloat16, False), (torch.bfloat16, True), (torch.float32, True)])
def test_forward_row_lse(dtype, generic):
    """Every forward path writes the rows' log2-sum-exp (the backward's row statistics):
    bf16 1e-3 (scores from bf16 inputs accumulated in fp32), fp32 1e-5."""
    from kvstreams import ops

    q, k, v, _, ev, ln = _case(dtype, 128, 8, 2, B=2, T=300, lengths=(300, 187), seed=7)
    scale = 128 ** -0.5
    lse = ops.row_lse_buffer(2, 8, 300, q.device)
    ops.replay_attention(q, k, v, ev, ln, scale, force_generic=generic, row_lse=lse)
    mask = _dense_mask(ev, ln.cpu(), 300).cuda()
    want = _dense_lse2(q, k, mask, scale)
    err = (lse[:, :, :300].double() - want).abs().max().item()
    assert err <= (1e-3 if dtype == torch.bfloat16 else 1e-5), err


@pytest.mark.parametrize("B,T,Hq,Hkv,lengths,turn", [
    (2, 300, 8, 2, (300, 211), 24),     # GQA 4, ragged last tile, padded rows
    (1, 1000, 4, 4, (1000,), 60),       # no GQA, 8 key tiles, unmasked tiles in the interior
    (3, 257, 6, 2, (257, 129, 5), 16),  # odd group size, a 5-token stream
    (1, 2048, 8, 1, (1900,), 200),      # MQA, long stream with padding
])
def test_tc_backward_matches_dense_autograd(B, T, Hq, Hkv, lengths, turn):
    """tcgen05 backward (bf16, D 128, the forward's row_lse) against fp64 autograd of the
    dense masked attention on the same bf16 inputs.  P and dS are bf16 UMMA operands, so
    the error is bf16 rounding of O(1) terms summed over up to T rows: the bound is 2% of
    the largest gradient entry, and within 4x the exact kernels' error (which rounds only
    the outputs) plus 0.5% of it."""
    from kvstreams import ops
    from kvstreams.workloads import replay_evicted_at

    g = torch.Generator(device="cuda").manual_seed(T + Hq)
    q = torch.randn(B, T, Hq, 128, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, T, Hkv, 128, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, T, Hkv, 128, generator=g, device="cuda").to(torch.bfloat16)
    go = torch.randn(B, T, Hq, 128, generator=g, device="cuda").to(torch.bfloat16)
    ev_np, _ = replay_evicted_at(batch=B, seq_len=T, events_range=(2, 6), mean_turn=turn, seed=T)
    ev = torch.from_numpy(ev_np).cuda()
    ln = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    scale = 128 ** -0.5
    lse = ops.row_lse_buffer(B, Hq, T, q.device)
    out = ops.replay_attention(q, k, v, ev, ln, scale, row_lse=lse)
    path = []
    tc = ops.replay_attention_backward(q, k, v, ev, ln, scale, out, go, row_lse=lse, report_path=path)
    exact = ops.replay_attention_backward(q, k, v, ev, ln, scale, out, go, force_exact=True, report_path=path)
    assert path == [1, 0], path  # the tensor-core kernels ran, then the exact ones
    qr, kr, vr = (x.detach().double().requires_grad_() for x in (q, k, v))
    mask = _dense_mask(ev, ln.cpu(), T).cuda()
    ref = _dense_attention(qr, kr, vr, mask, scale)
    ref.backward(go.double())
    for got, ex, want, name in zip(tc, exact, (qr.grad, kr.grad, vr.grad), ("dq", "dk", "dv")):
        assert torch.isfinite(got).all(), name
        mag = want.abs().max().item()
        err = (got.double() - want).abs().max().item()
        err_exact = (ex.double() - want).abs().max().item()
        assert err <= 0.02 * mag, f"{name}: {err} (max |grad| {mag})"
        assert err <= 4 * err_exact + 0.005 * mag, f"{name}: {err} vs exact {err_exact} (max |grad| {mag})"


def test_tc_backward_deterministic():
    """No atomics: two backward passes give the same bits."""
    from kvstreams import ops

    q, k, v, go, ev, ln = _case(torch.bfloat16, 128, 8, 2, B=2, T=300, lengths=(300, 211), seed=3)
    scale = 128 ** -0.5
    lse = ops.row_lse_buffer(2, 8, 300, q.device)
    out = ops.replay_attention(q, k, v, ev, ln, scale, row_lse=lse)
    a = ops.replay_attention_backward(q, k, v, ev, ln, scale, out, go, row_lse=lse)
    b = ops.replay_attention_backward(q, k, v, ev, ln, scale, out, go, row_lse=lse)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
