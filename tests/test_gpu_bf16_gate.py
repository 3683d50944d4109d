"""The bf16 replay gate (max|replay logp - inference logp| <= 2e-2) on the kernels that carry
bf16 attention at the Llama-3-8B attention geometry (32 query / 8 KV heads, D 128, theta 5e5).

The model keeps its dense layers in float32 and runs only attention in bf16
(``TinyLM.attention_dtype``): the bf16 KV pool, the fused paged decode kernel, the tcgen05
paged prefill and the tcgen05 masked replay.  The replay-vs-inference difference is then the
attention kernels' own (different tiling, accumulation order and P rounding between the
inference kernels and the replay kernel) plus the bf16 rounding of q/k/v, and nothing of the
bf16 dense GEMMs, whose shape-dependent rounding dominates a whole-bf16 model at d_model 4096
(test_gpu_batched.py)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

FUSED, PREFILL = 1, 2  # kvs_paged_decode_path bits


def _geometry(**kw):
    from kvstreams.config import ModelConfig

    return ModelConfig(vocab_size=512, d_model=4096, n_layers=2, n_heads=32, n_kv_heads=8, d_ff=1024,
                       rope_theta=5e5, **kw)


@pytest.mark.parametrize("bs", [16, 1])
def test_bf16_attention_replay_gate_llama_heads(monkeypatch, bs):
    from kvstreams import ops
    from kvstreams.compaction.policies import MarkovianPolicy
    from kvstreams.engine.batched import BatchedKVStreams, synthetic_episodes
    from kvstreams.model import TinyLM
    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.training.mismatch import measure_mismatch

    cfg = _geometry()
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = TinyLM(cfg).float()
    model.attention_dtype = torch.bfloat16
    n = 8
    cache = PagedKVCache(cfg.n_layers, cfg.n_kv_heads, cfg.head_dim, block_size=bs, num_blocks=2048 * 16 // bs,
                         dtype=torch.bfloat16, max_seqs=n)
    eng = BatchedKVStreams(model, cache, MarkovianPolicy(keep_last=1), context_budget=640, seed=0)
    eps = synthetic_episodes(n, turns=5, turn_range=(20, 160), prompt_len=40, vocab=cfg.vocab_size, seed=2)

    paths = []
    plain = ops.paged_forward

    def recording(*a, **k):
        k["report_path"] = paths
        return plain(*a, **k)

    monkeypatch.setattr(ops, "paged_forward", recording)
    rolls = eng.run(eps)
    monkeypatch.setattr(ops, "paged_forward", plain)
    assert sum(len(r.log.events) for r in rolls) >= 4, "the budget should force compactions"
    seen = 0
    for p in paths:
        seen |= p
    # decode steps on the fused kernel; turn chunks on the tensor-core prefill (16-token blocks)
    assert seen & FUSED
    if bs == 16:
        assert seen & PREFILL
    rep = measure_mismatch(model, rolls)
    assert rep.num_tokens == sum(sum(ep.reply_lens) for ep in eps)
    assert rep.max_abs_logprob_diff <= 2e-2, rep


def test_bf16_replay_kernel_path_at_llama_heads():
    """The replay of the gate test runs the tcgen05 kernels: q/k/v of the 8B geometry in bf16,
    16-byte aligned, D 128 -- the backward path query (which requires the forward's tensor-core
    path) reports the tensor-core kernels."""
    from kvstreams import ops

    B, T = 2, 300
    q = torch.randn(B, T, 32, 128, device="cuda").bfloat16()
    k = torch.randn(B, T, 8, 128, device="cuda").bfloat16()
    v = torch.randn(B, T, 8, 128, device="cuda").bfloat16()
    ev = torch.full((B, T), (1 << 63) - 1, dtype=torch.long, device="cuda")
    ln = torch.full((B,), T, dtype=torch.int32, device="cuda")
    lse = ops.row_lse_buffer(B, 32, T, q.device)
    out = ops.replay_attention(q, k, v, ev, ln, 128 ** -0.5, row_lse=lse)
    path = []
    ops.replay_attention_backward(q, k, v, ev, ln, 128 ** -0.5, out, torch.randn_like(out), row_lse=lse,
                                  report_path=path)
    assert path == [1]
