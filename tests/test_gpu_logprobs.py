"""Fused log-softmax + gather of token_logprobs (kvs_lse_gather / _backward,
training/logprobs.py:17-20) against torch: log_softmax(logits / T).gather and its autograd
gradient; the lm_head GEMM with the log-sum-exp in its epilogue (kvs_lm_head_logprobs) against
the float32-result GEMM + kvs_lse_gather (2e-5); token_logprobs through the fused chunks against
the torch chunk loop (fp64 to 1e-12, bf16 models: same float32 logits, 2e-5)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,n,vocab,temp,tol", [
    (torch.float32, 300, 128256, 1.0, 2e-5),
    (torch.float32, 64, 1001, 0.7, 2e-5),     # odd vocabulary: the scalar tail of each row
    (torch.float64, 50, 1001, 1.3, 1e-12),
])
def test_lse_gather_matches_torch(dtype, n, vocab, temp, tol):
    from kvstreams import ops

    g = torch.Generator(device="cuda").manual_seed(vocab)
    x = (torch.randn(n, vocab, generator=g, device="cuda", dtype=torch.float64) * 4).to(dtype)
    t = torch.randint(0, vocab, (n,), generator=g, device="cuda")
    logp, lse = ops.lse_gather(x, t, temp)
    ref = torch.log_softmax(x.double() / temp, dim=-1)
    want = ref.gather(-1, t[:, None]).squeeze(-1)
    assert (logp.double() - want).abs().max().item() <= tol
    assert (lse.double() - torch.logsumexp(x.double() / temp, dim=-1)).abs().max().item() <= tol
    # gradient with respect to the logits for a random upstream gradient
    go = torch.randn(n, generator=g, device="cuda", dtype=torch.float64).to(dtype)
    xr = x.double().requires_grad_()
    (torch.log_softmax(xr / temp, dim=-1).gather(-1, t[:, None]).squeeze(-1) * go.double()).sum().backward()
    d = ops.lse_gather_backward(x, t, lse, go, temp)
    assert (d.double() - xr.grad).abs().max().item() <= tol
    if dtype == torch.float32:
        db = ops.lse_gather_backward(x, t, lse, go, temp, out_dtype=torch.bfloat16)
        assert (db.double() - xr.grad).abs().max().item() <= 1e-2 * xr.grad.abs().max().item() + 1e-6


def _batch(cfg, B, T, seed):
    from kvstreams.training.replay import Batch
    from kvstreams.workloads import replay_evicted_at

    ev, _ = replay_evicted_at(batch=B, seq_len=T, events_range=(2, 4), mean_turn=10, seed=seed)
    g = torch.Generator().manual_seed(seed)
    tokens = torch.randint(1, cfg.vocab_size, (B, T), generator=g).cuda()
    return Batch(tokens, torch.arange(T).expand(B, T).cuda(), torch.from_numpy(ev).cuda(),
                 torch.ones(B, T, dtype=torch.bool, device="cuda"), torch.zeros(B, T, device="cuda"),
                 torch.tensor([T, T - 13], device="cuda"))


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-12), (torch.bfloat16, 2e-5)])
def test_token_logprobs_fused_equals_torch_chunks(dtype, tol):
    from kvstreams.config import ModelConfig
    from kvstreams.model import TinyLM
    from kvstreams.training.logprobs import token_logprobs

    torch.manual_seed(0)
    cfg = ModelConfig()
    with torch.device("cuda"):
        model = TinyLM(cfg).to(dtype)
    batch = _batch(cfg, 2, 96, seed=3)
    with torch.no_grad():
        fused = token_logprobs(model, batch, temperature=0.9)
        _, full = token_logprobs(model, batch, temperature=0.9, return_full=True)  # the torch chunk loop
    ref = full[:, 1:].gather(-1, batch.tokens[:, 1:, None]).squeeze(-1)
    assert (fused[:, 1:].double() - ref.double()).abs().max().item() <= tol
    assert torch.all(fused[:, 0] == 0)


@pytest.mark.parametrize("M,N,K,temp", [
    (512, 1024, 256, 1.0),
    (1000, 5000, 512, 0.7),      # ragged rows (last pair tile half empty) and vocabulary (last tile 136 wide)
    (300, 128256, 4096, 1.0),    # the 8B vocabulary and hidden size
    (2048, 128256, 4096, 1.3),
    (77, 104, 64, 1.0),          # one partial tile each way (the TinyLM lm_head)
])
def test_lm_head_logprobs_matches_gemm_and_lse_gather(M, N, K, temp):
    """The logits are never stored, yet log-probs and log-sum-exps equal the float32-result GEMM
    followed by kvs_lse_gather within 2e-5 (float32 accumulation in both; different order).
    Targets on tile boundaries and at both ends of the vocabulary; an out-of-range target gives
    NaN for its row only."""
    from kvstreams import ops

    g = torch.Generator(device="cuda").manual_seed(M + N)
    h = torch.randn(M, K, generator=g, device="cuda").bfloat16()
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).bfloat16()
    t = torch.randint(0, N, (M,), generator=g, device="cuda")
    edges = [0, N - 1, min(255, N - 1), min(256, N - 1), N // 2]
    t[: len(edges)] = torch.tensor(edges, device="cuda")
    assert ops.lm_head_logprobs_supported(h, w)
    logp, lse = ops.lm_head_logprobs(h, w, t, temp)
    ref_logp, ref_lse = ops.lse_gather(torch.mm(h, w.t(), out_dtype=torch.float32), t, temp)
    assert (logp - ref_logp).abs().max().item() <= 2e-5
    assert (lse - ref_lse).abs().max().item() <= 2e-5
    bad = t.clone()
    bad[3] = N
    lp2, _ = ops.lm_head_logprobs(h, w, bad, temp)
    assert torch.isnan(lp2[3]) and not torch.isnan(lp2[torch.arange(M, device="cuda") != 3]).any()


def test_token_logprobs_bf16_takes_the_epilogue_kernel():
    """A bf16 model's token_logprobs runs the lm_head through kvs_lm_head_logprobs (its
    forward) and still differentiates (the backward recomputes the logits)."""
    from kvstreams import ops
    from kvstreams.config import ModelConfig
    from kvstreams.model import TinyLM
    from kvstreams.training.logprobs import token_logprobs

    torch.manual_seed(1)
    cfg = ModelConfig()
    with torch.device("cuda"):
        model = TinyLM(cfg).to(torch.bfloat16)
    batch = _batch(cfg, 2, 96, seed=4)
    h = torch.zeros(8, cfg.d_model, dtype=torch.bfloat16, device="cuda")
    assert ops.lm_head_logprobs_supported(h, model.lm_head.weight)
    calls = []
    plain = ops.lm_head_logprobs

    def counting(*a, **k):
        calls.append(1)
        return plain(*a, **k)

    ops.lm_head_logprobs = counting
    try:
        lp = token_logprobs(model, batch, temperature=1.0)
        lp.sum().backward()
    finally:
        ops.lm_head_logprobs = plain
    assert calls and torch.isfinite(lp).all()
    assert torch.isfinite(model.lm_head.weight.grad).all() and model.lm_head.weight.grad.abs().sum() > 0
