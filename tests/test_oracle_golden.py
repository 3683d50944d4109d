"""The oracle (oracle/kvs_oracle.py) reproduces the reference's own outputs.

Golden fixtures were produced by running the reference (tests/golden/make_golden.py).
These tests pin the oracle before it is used to check the CUDA kernels."""

import numpy as np
import pytest

from oracle import kvs_oracle as O


@pytest.mark.parametrize("name", ["scripted_bs4", "random_bs16", "random_bs8", "random_bs1", "random_bs16_tight"])
def test_cache_trace_bit_exact(golden_traces, name):
    t = golden_traces[name]
    _, obs = O.replay_trace(t["ops"], t["num_blocks"], t["block_size"])
    assert len(obs) == len(t["obs"])
    for i, (got, want) in enumerate(zip(obs, t["obs"])):
        assert got == want, f"{name}: op {i} {t['ops'][i][:2]} differs"


def test_evicted_at(golden_evicted_at):
    g = golden_evicted_at
    n = len([k for k in g.files if k.endswith("_out")])
    assert n >= 10
    for i in range(n):
        got = O.evicted_at(g[f"c{i}_triples"], int(g[f"c{i}_len"][0]))
        np.testing.assert_array_equal(got, g[f"c{i}_out"])


@pytest.mark.parametrize("D", [16, 128])
@pytest.mark.parametrize("prec", ["f32", "f64"])
def test_rope(golden_rope, D, prec):
    g = golden_rope
    x, y, pos = g[f"D{D}_{prec}_x"], g[f"D{D}_{prec}_y"], g[f"D{D}_{prec}_pos"]
    theta = float(g[f"D{D}_{prec}_theta"][0])
    dt = np.float32 if prec == "f32" else np.float64
    got = O.rope_apply(x, pos, theta, dt)
    # float32: libm cos/sin of numpy vs torch differ by an ulp; float64 to ~1e-15
    tol = 2e-6 if prec == "f32" else 1e-12
    np.testing.assert_allclose(got, y, rtol=0, atol=tol * max(1.0, np.abs(y).max()))


def _params(arrays, prefix):
    return {k[len(prefix):]: arrays[k] for k in arrays.files if k.startswith(prefix)}


def test_tinylm_masked_forward(golden_tinylm):
    g = golden_tinylm
    params = _params(g, "p::")
    cfg = dict(n_layers=2, n_heads=4, n_kv_heads=2, d_model=64, norm_eps=1e-6, rope_theta=1e4)
    T = g["tokens"].shape[0]
    got = O.tinylm_forward(params, cfg, g["tokens"], np.arange(T), g["mask"])
    np.testing.assert_allclose(got, g["logits"], rtol=0, atol=1e-10)


@pytest.mark.parametrize("tag", ["f64_bs16_0", "f64_bs1_0", "f64_bs8_markov_1"])
def test_oracle_replay_matches_reference_logprobs(golden_rollouts, tag):
    arrays, meta = golden_rollouts
    params = _params(arrays, "m64::")
    cfg = dict(n_layers=2, n_heads=4, n_kv_heads=2, d_model=64, norm_eps=1e-6, rope_theta=1e4)
    tokens = arrays[tag + "_tokens"]
    ev = arrays[tag + "_evicted_at"]
    T = tokens.shape[0]
    trip = [(s, e, ev_["time"]) for ev_ in meta[tag]["events"] for s, e in ev_["evicted"]]
    np.testing.assert_array_equal(O.evicted_at(trip, T), ev)
    logits = O.tinylm_forward(params, cfg, tokens, np.arange(T), O.kvstream_mask(ev))
    lp = O.log_softmax(logits)
    got = np.zeros(T)
    got[1:] = lp[np.arange(T - 1), tokens[1:]]
    np.testing.assert_allclose(got, arrays[tag + "_replay"], rtol=0, atol=1e-10)
    loss = arrays[tag + "_loss"]
    # the reference's core claim, reproduced by the oracle: replay == inference
    assert np.abs(got[loss] - arrays[tag + "_inf"][loss]).max() < 1e-9


def test_row_sampled_replay_oracle_equals_dense():
    """replay_attention_rows (the full-length checker) equals the dense-mask replay oracle."""
    rng = np.random.default_rng(0)
    T = 300
    q, k, v = rng.standard_normal((T, 8, 16)), rng.standard_normal((T, 2, 16)), rng.standard_normal((T, 2, 16))
    ev = np.full(T, O.NEVER, dtype=np.int64)
    ev[40:80], ev[100:120] = 150, 200
    rows = [0, 1, 79, 149, 150, 199, 200, 299]
    dense = O.replay_attention(q[None], k[None], v[None], ev[None], np.array([T]), 0.25)[0]
    np.testing.assert_allclose(O.replay_attention_rows(q, k, v, ev, rows, 0.25), dense[rows], rtol=0, atol=1e-12)
