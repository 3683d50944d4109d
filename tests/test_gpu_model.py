"""Model- and engine-level parity on the GPU: the reference's own claims (tests/test_model.py,
tests/test_replay.py) reproduced through the kernels, against golden reference outputs."""

import numpy as np
import pytest
import torch

from oracle import kvs_oracle as O

pytestmark = pytest.mark.gpu


def _model(arrays, prefix, dtype, cfg_kw=None):
    from kvstreams.config import ModelConfig
    from kvstreams.model import TinyLM

    sd = {k[len(prefix):]: torch.from_numpy(arrays[k]) for k in arrays.files if k.startswith(prefix)}
    m = TinyLM(ModelConfig(vocab_size=104, **(cfg_kw or {})))
    m.load_state_dict(sd)
    return m.to(device="cuda", dtype=dtype).eval()


def test_masked_forward_matches_reference_logits(golden_tinylm):
    g = golden_tinylm
    m = _model(g, "p::", torch.float64, {"init_std": 0.1})
    T = g["tokens"].shape[0]
    with torch.no_grad():
        logits = m(torch.from_numpy(g["tokens"])[None].cuda(), torch.arange(T)[None].cuda(),
                   torch.from_numpy(g["mask"])[None].cuda())[0]
    np.testing.assert_allclose(logits.cpu().numpy(), g["logits"], rtol=0, atol=1e-10)


def test_cached_forward_matches_full_forward(golden_tinylm):
    """tests/test_model.py:14-26 of the reference, through the paged kernels."""
    from kvstreams.paged_cache import PagedKVCache

    m = _model(golden_tinylm, "p::", torch.float64, {"init_std": 0.1})
    torch.manual_seed(1)
    tokens = torch.randint(0, 104, (23,)).cuda()
    with torch.no_grad():
        full = m(tokens[None])[0]
    cfg = m.cfg
    cache = PagedKVCache(cfg.n_layers, cfg.n_kv_heads, cfg.head_dim, block_size=4, num_blocks=64, dtype=m.dtype)
    cache.add_sequence(0)
    outs = []
    for chunk in (tokens[:10], tokens[10:11], tokens[11:20], tokens[20:]):
        start = cache.num_tokens(0)
        outs.append(m.forward_cached(chunk, torch.arange(start, start + len(chunk)).cuda(), cache, 0))
    assert torch.allclose(torch.cat(outs), full, atol=1e-10)


def test_eviction_matches_masked_forward(golden_tinylm):
    """tests/test_model.py:29-42: evicting a block == masking it for later queries."""
    from kvstreams.model import causal_mask
    from kvstreams.paged_cache import PagedKVCache

    m = _model(golden_tinylm, "p::", torch.float64, {"init_std": 0.1})
    torch.manual_seed(2)
    tokens = torch.randint(0, 104, (20,)).cuda()
    cfg = m.cfg
    cache = PagedKVCache(cfg.n_layers, cfg.n_kv_heads, cfg.head_dim, block_size=4, num_blocks=64, dtype=m.dtype)
    cache.add_sequence(0)
    m.forward_cached(tokens[:12], torch.arange(12).cuda(), cache, 0)
    assert cache.evict_positions(0, [(4, 8)]) == [(4, 8)]
    tail = m.forward_cached(tokens[12:], torch.arange(12, 20).cuda(), cache, 0)
    mask = causal_mask(20).clone()
    mask[12:, 4:8] = False
    with torch.no_grad():
        ref = m(tokens[None], torch.arange(20)[None].cuda(), mask[None].cuda())[0, 12:]
    assert torch.allclose(tail, ref, atol=1e-10)


def test_rope_relative_position_invariance():
    """tests/test_rope.py:11-30 through the rope kernel."""
    from kvstreams.rope import RotaryEmbedding

    rope = RotaryEmbedding(16)
    torch.manual_seed(0)
    q = torch.randn(16, dtype=torch.float64).cuda()
    k = torch.randn(16, dtype=torch.float64).cuda()

    def rot(x, p):
        return rope.rotate_(x.clone()[None, None], torch.tensor([p]).cuda())[0, 0]

    assert torch.allclose(rot(q, 1000) @ rot(k, 990), rot(q, 10) @ rot(k, 0), atol=1e-10)
    assert not torch.allclose(rot(q, 510) @ rot(k, 1000), rot(q, 1010) @ rot(k, 1000))
    x = torch.randn(3, 2, 8, dtype=torch.float64).cuda()
    y = RotaryEmbedding(8).rotate_(x.clone(), torch.tensor([0, 7, 123]).cuda())
    assert torch.allclose(x.norm(dim=-1), y.norm(dim=-1))


def _engine(model, bs, pad, policy, kw, budget=160, max_new=12, engine="kvstream", commit=True):
    from kvstreams.compaction import build_policy
    from kvstreams.config import CacheConfig, RolloutConfig, SamplingConfig
    from kvstreams.engine import build_engine
    from kvstreams.tokenizer import CharTokenizer

    return build_engine(engine, model, CharTokenizer(), build_policy(policy, **kw),
                        CacheConfig(block_size=bs, num_blocks=1024, pad_to_block=pad, commit_partial_blocks=commit),
                        RolloutConfig(context_budget=budget, record_full_logprobs=True),
                        SamplingConfig(max_new_tokens=max_new))


@pytest.mark.parametrize("tag,bs,pad,policy,kw", [
    ("f64_bs16", 16, True, "keep_recent", {"keep_last": 2}),
    ("f64_bs1", 1, False, "keep_recent", {"keep_last": 2}),
    ("f64_bs8_markov", 8, True, "markovian", {"keep_last": 1}),
])
def test_fp64_rollouts_and_replay_match_reference(golden_rollouts, tag, bs, pad, policy, kw):
    """The reference's core claim (tests/test_replay.py:22-38) at EXACT = 1e-9, and the rollout
    log-probs equal the reference's own to 1e-9."""
    from kvstreams.envs import build_env
    from kvstreams.training import measure_mismatch

    arrays, meta = golden_rollouts
    m = _model(arrays, "m64::", torch.float64, {"init_std": 0.1})
    eng = _engine(m, bs, pad, policy, kw)
    rs = [eng.rollout(build_env("recall", seed=i, num_distractors=6), teacher_forcing=True) for i in range(2)]
    for i, r in enumerate(rs):
        key = f"{tag}_{i}"
        assert r.tokens == arrays[key + "_tokens"].tolist()
        assert [e.to_dict() for e in r.log] == meta[key]["events"]
        loss = arrays[key + "_loss"]
        np.testing.assert_allclose(np.asarray(r.inf_logprobs)[loss], arrays[key + "_inf"][loss], rtol=0, atol=1e-9)
    rep = measure_mismatch(m, rs, "kvstream")
    assert rep.max_abs_logprob_diff < 1e-9
    assert abs(rep.exact_kl) < 1e-9
    assert measure_mismatch(m, rs, "full").max_abs_logprob_diff > 1e-3


def test_fp32_bench_config_rollout_and_replay(golden_rollouts):
    """Repo-native CPU bench config (fp32 default TinyLM, keep_recent 2, bs 16 padded,
    budget 256, 24 distractors x filler 64): replay vs inference <= 1e-5 in fp32."""
    from kvstreams.envs import build_env
    from kvstreams.training import measure_mismatch

    arrays, meta = golden_rollouts
    m = _model(arrays, "m32::", torch.float32)
    eng = _engine(m, 16, True, "keep_recent", {"keep_last": 2}, budget=256)
    eng.rollout_cfg.max_turns = 128
    r = eng.rollout(build_env("recall", seed=0, num_distractors=24, filler_len=64), teacher_forcing=True)
    key = "f32_c1_0"
    assert r.tokens == arrays[key + "_tokens"].tolist()
    assert [e.to_dict() for e in r.log] == meta[key]["events"]
    assert r.stats.tokens_forwarded == r.length == 2032
    loss = arrays[key + "_loss"]
    np.testing.assert_allclose(np.asarray(r.inf_logprobs)[loss], arrays[key + "_inf"][loss], rtol=0, atol=1e-4)
    rep = measure_mismatch(m, [r], "kvstream")
    assert rep.max_abs_logprob_diff <= 1e-5, rep


def test_bf16_replay_gate(golden_rollouts):
    """bf16 model (fp32 default weights rounded): replay vs inference within 2e-2."""
    from kvstreams.envs import build_env
    from kvstreams.training import measure_mismatch

    arrays, _ = golden_rollouts
    m = _model(arrays, "m32::", torch.bfloat16)
    eng = _engine(m, 16, True, "keep_recent", {"keep_last": 2}, budget=256)
    eng.rollout_cfg.max_turns = 128
    r = eng.rollout(build_env("recall", seed=0, num_distractors=24, filler_len=64), teacher_forcing=True)
    rep = measure_mismatch(m, [r], "kvstream")
    assert rep.max_abs_logprob_diff <= 2e-2, rep


@pytest.mark.parametrize("tag,engine,bs,pad,commit,policy,kw", [
    ("f64_reprefill_bs16", "reprefill", 16, True, True, "keep_recent", {"keep_last": 2}),
    ("f64_reprefill_bs4_recompute", "reprefill", 4, False, False, "keep_recent", {"keep_last": 1}),
    ("f64_bs16_recompute", "kvstream", 16, False, False, "keep_recent", {"keep_last": 2}),
    ("f64_bs8_summary", "kvstream", 8, True, True, "summary", {"keep_last": 1}),
])
def test_fp64_engine_paths_match_reference(golden_rollouts, tag, engine, bs, pad, commit, policy, kw):
    """Re-prefill, recomputed partial blocks and summary turns through the kernels: tokens and
    events equal the reference's, inference log-probs within 1e-9 of the reference's own."""
    from kvstreams.envs import build_env

    arrays, meta = golden_rollouts
    m = _model(arrays, "m64::", torch.float64, {"init_std": 0.1})
    eng = _engine(m, bs, pad, policy, kw, engine=engine, commit=commit)
    for i in range(2):
        r = eng.rollout(build_env("recall", seed=i, num_distractors=6), teacher_forcing=True)
        key = f"{tag}_{i}"
        assert r.tokens == arrays[key + "_tokens"].tolist()
        assert [e.to_dict() for e in r.log] == meta[key]["events"]
        assert r.stats.tokens_forwarded == meta[key]["stats"]["tokens_forwarded"]
        assert r.stats.reprefill_tokens == meta[key]["stats"]["reprefill_tokens"]
        loss = arrays[key + "_loss"]
        np.testing.assert_allclose(np.asarray(r.inf_logprobs)[loss], arrays[key + "_inf"][loss], rtol=0, atol=1e-9)


def test_fp32_bench_config_reprefill_arm(golden_rollouts):
    """The comparison arm of the CPU bench configuration: the same episode through the
    re-prefill engine forwards 6816 tokens (KV-streams: 2032), with the reference's tokens,
    events and log-probs."""
    from kvstreams.envs import build_env

    arrays, meta = golden_rollouts
    m = _model(arrays, "m32::", torch.float32)
    eng = _engine(m, 16, True, "keep_recent", {"keep_last": 2}, budget=256, engine="reprefill")
    eng.rollout_cfg.max_turns = 128
    r = eng.rollout(build_env("recall", seed=0, num_distractors=24, filler_len=64), teacher_forcing=True)
    key = "f32_c1_reprefill_0"
    assert r.tokens == arrays[key + "_tokens"].tolist()
    assert [e.to_dict() for e in r.log] == meta[key]["events"]
    assert r.stats.tokens_forwarded == 6816 == meta[key]["stats"]["tokens_forwarded"]
    loss = arrays[key + "_loss"]
    np.testing.assert_allclose(np.asarray(r.inf_logprobs)[loss], arrays[key + "_inf"][loss], rtol=0, atol=1e-4)


@pytest.mark.parametrize("engine", ["kvstream", "reprefill"])
def test_rollout_batch_equals_one_at_a_time(golden_rollouts, engine):
    """rollout_batch plays several episodes with one batched forward per step; every episode
    equals its own rollout() (fp64: tokens, events, stats; log-probs within 1e-10), teacher
    forced and sampled (greedy, so the draws do not depend on batching)."""
    from kvstreams.envs import build_env

    arrays, _ = golden_rollouts
    m = _model(arrays, "m64::", torch.float64, {"init_std": 0.1})
    for forcing in (True, False):
        eng = _engine(m, 8, True, "keep_recent", {"keep_last": 1}, engine=engine)
        eng.sampling.greedy = not forcing
        envs = [build_env("recall", seed=i, num_distractors=4 + i) for i in range(4)]
        batch = eng.rollout_batch(envs, teacher_forcing=forcing)
        singles = [eng.rollout(build_env("recall", seed=i, num_distractors=4 + i), teacher_forcing=forcing)
                   for i in range(4)]
        assert eng.cache.allocator.num_used == 0
        for a, b in zip(batch, singles):
            assert a.tokens == b.tokens and a.loss_mask == b.loss_mask and a.completions == b.completions
            assert [e.to_dict() for e in a.log] == [e.to_dict() for e in b.log]
            sa, sb = a.stats.to_dict(), b.stats.to_dict()
            sa.pop("wall_time"), sb.pop("wall_time")
            assert sa == sb
            np.testing.assert_allclose(a.inf_logprobs, b.inf_logprobs, rtol=0, atol=1e-10)
