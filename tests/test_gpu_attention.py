"""RoPE, paged attention (decode + prefill) and masked replay attention kernels vs the oracle.

Tolerances: float64 1e-10, float32 2e-5 (absolute on O(1) outputs), bfloat16 3e-2
(against the float64 oracle evaluated on the same bf16-rounded inputs)."""

import numpy as np
import pytest
import torch

from oracle import kvs_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float64: 1e-10, torch.float32: 2e-5, torch.bfloat16: 3e-2}


def _np(t):
    return t.detach().float().cpu().numpy().astype(np.float64) if t.dtype == torch.bfloat16 else t.detach().cpu().numpy()


@pytest.mark.parametrize("D", [16, 128])
@pytest.mark.parametrize("prec", ["f32", "f64"])
def test_rope_kernel_matches_reference(golden_rope, D, prec):
    from kvstreams.rope import RotaryEmbedding

    g = golden_rope
    dt = torch.float32 if prec == "f32" else torch.float64
    x = torch.from_numpy(g[f"D{D}_{prec}_x"]).cuda()
    pos = torch.from_numpy(g[f"D{D}_{prec}_pos"]).cuda()
    rope = RotaryEmbedding(D, float(g[f"D{D}_{prec}_theta"][0]))
    y = rope.rotate_(x.clone().to(dt), pos)
    want = g[f"D{D}_{prec}_y"]
    tol = 2e-6 if prec == "f32" else 1e-12
    np.testing.assert_allclose(y.cpu().numpy(), want, rtol=0, atol=tol * max(1.0, np.abs(want).max()))


def _setup_cache(dtype, D, Hkv, bs, S, ctx, seed):
    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.workloads import decode_state

    st = decode_state(num_streams=S, ctx_range=ctx, block_size=bs, num_blocks=S * (ctx[1] // bs + 8),
                      evicted_spans_range=(1, 3), seed=seed)
    cache = PagedKVCache(1, Hkv, D, block_size=bs, num_blocks=st.num_blocks, dtype=dtype, max_seqs=S)
    cache.load_state(range(S), st.tables, st.positions, st.free_list)
    g = torch.Generator(device="cuda").manual_seed(seed)
    cache.k.copy_(torch.randn(cache.k.shape, generator=g, device="cuda").to(dtype))
    cache.v.copy_(torch.randn(cache.v.shape, generator=g, device="cuda").to(dtype))
    return cache, st


@pytest.mark.parametrize("dtype,D,Hq,Hkv,bs,T,S,ctx", [
    (torch.float64, 16, 4, 2, 16, 1, 5, (3, 200)),
    (torch.float64, 16, 4, 2, 4, 5, 5, (3, 200)),
    (torch.float32, 16, 4, 2, 16, 1, 5, (3, 200)),
    (torch.float32, 32, 8, 2, 1, 3, 5, (3, 200)),
    (torch.bfloat16, 128, 32, 8, 16, 1, 5, (3, 200)),
    # fused kernel with CTA ranges spanning several sequences and sequences spanning several CTAs
    (torch.bfloat16, 128, 32, 8, 16, 1, 12, (500, 3000)),
    (torch.bfloat16, 128, 32, 8, 16, 1, 40, (16, 40)),
    (torch.bfloat16, 128, 32, 8, 16, 7, 5, (3, 200)),
    (torch.bfloat16, 64, 8, 8, 1, 1, 5, (3, 200)),
])
def test_paged_forward_matches_oracle(dtype, D, Hq, Hkv, bs, T, S, ctx):
    from kvstreams import ops
    from kvstreams.rope import RotaryEmbedding

    cache, st = _setup_cache(dtype, D, Hkv, bs, S, ctx, seed=D + T + S)
    theta = 5e5 if D == 128 else 1e4
    rope = RotaryEmbedding(D, theta)
    g = torch.Generator(device="cuda").manual_seed(7)
    N = S * T
    q = torch.randn(N, Hq, D, generator=g, device="cuda").to(dtype)
    k = torch.randn(N, Hkv, D, generator=g, device="cuda").to(dtype)
    v = torch.randn(N, Hkv, D, generator=g, device="cuda").to(dtype)
    pos = torch.cat([torch.arange(int(p), int(p) + T) for p in st.next_positions]).cuda()
    counts = [T] * S
    old_k = cache.k.clone()
    old_tables = [cache.block_table(s) for s in range(S)]
    old_len = [cache.num_tokens(s) for s in range(S)]
    mapping = cache.append_slots_batch(list(range(S)), pos, None if T == 1 else counts)
    out = ops.paged_forward(cache, list(range(S)), None if T == 1 else counts, 0, q, k, v, pos, mapping,
                            rope.table(q.device, dtype), D ** -0.5)
    torch.cuda.synchronize()
    odt = np.float64 if dtype == torch.float64 else np.float32
    qn, kn, vn, pn = _np(q), _np(k), _np(v), pos.cpu().numpy()
    q_rot = O.rope_apply(qn, pn, theta, odt).astype(np.float64)
    k_rot = O.rope_apply(kn, pn, theta, odt).astype(np.float64)
    pool_k, pool_v = _np(old_k)[0], _np(cache.v)[0]
    new_k = _np(cache.k)[0]
    blocks = mapping.blocks.cpu().numpy()
    offs = mapping.offsets.cpu().numpy()
    # the appended keys are the rotated new keys (bf16: rounded once)
    np.testing.assert_allclose(new_k[blocks, offs], k_rot, rtol=0, atol=TOL[dtype] * 0.5)
    np.testing.assert_array_equal(cache.slot_pos.cpu().numpy()[blocks, offs], pn)
    got = _np(out)
    for s in range(S):
        tab = old_tables[s] + cache.block_table(s)[len(old_tables[s]):]
        n_old = old_len[s]
        ks = pool_k[tab].reshape(-1, Hkv, D)[:n_old]
        vs = pool_v[tab].reshape(-1, Hkv, D)[:n_old + T]
        sl = slice(s * T, (s + 1) * T)
        keys = np.concatenate([ks, k_rot[sl]])
        mask = np.ones((T, n_old + T), dtype=bool)
        mask[:, n_old:] = np.tril(np.ones((T, T), dtype=bool))
        want = O.gqa_attention(q_rot[sl], keys, vs, mask, D ** -0.5)
        np.testing.assert_allclose(got[sl], want, rtol=0, atol=TOL[dtype], err_msg=f"stream {s}")


@pytest.mark.parametrize("dtype,D,Hq,Hkv", [
    (torch.float64, 16, 4, 2),
    (torch.float32, 16, 4, 2),
    (torch.bfloat16, 128, 8, 2),
    (torch.bfloat16, 64, 4, 4),
])
def test_replay_attention_matches_oracle(dtype, D, Hq, Hkv):
    from kvstreams import ops
    from kvstreams.workloads import replay_evicted_at

    B, T = 3, 333
    ev, _ = replay_evicted_at(batch=B, seq_len=T, events_range=(2, 4), mean_turn=24, seed=D)
    lengths = np.array([T, T - 40, 97], dtype=np.int32)
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(B, T, Hq, D, generator=g, device="cuda").to(dtype)
    k = torch.randn(B, T, Hkv, D, generator=g, device="cuda").to(dtype)
    v = torch.randn(B, T, Hkv, D, generator=g, device="cuda").to(dtype)
    out = ops.replay_attention(q, k, v, torch.from_numpy(ev).cuda(), torch.from_numpy(lengths).cuda(), D ** -0.5)
    want = O.replay_attention(_np(q), _np(k), _np(v), ev, lengths, D ** -0.5)
    np.testing.assert_allclose(_np(out), want, rtol=0, atol=TOL[dtype])


def test_replay_mask_factoring_roundtrip():
    from kvstreams.ops import ReplayMask

    T = 20
    m = torch.ones(T, T, dtype=torch.bool).tril()
    m[12:, 4:8] = False
    rm = ReplayMask.from_dense(m[None].cuda())
    assert rm.evicted_at[0, 4:8].tolist() == [12] * 4
    assert torch.equal(rm.dense()[0].cpu(), m)
    bad = m.clone()
    bad[15, 5] = True
    with pytest.raises(ValueError):
        ReplayMask.from_dense(bad[None].cuda())


def test_evicted_at_kernel_matches_reference(golden_evicted_at):
    from kvstreams.ops import evicted_at_from_spans

    g = golden_evicted_at
    n = len([k for k in g.files if k.endswith("_out")])
    trips = [g[f"c{i}_triples"].reshape(-1, 3) for i in range(n)]
    lens = [int(g[f"c{i}_len"][0]) for i in range(n)]
    cu = np.zeros(n + 1, dtype=np.int32)
    np.cumsum([len(t) for t in trips], out=cu[1:])
    flat = np.concatenate(trips) if cu[-1] else np.zeros((1, 3), dtype=np.int64)
    out = evicted_at_from_spans(cu, flat, lens, "cuda", max(lens)).cpu().numpy()
    for i in range(n):
        np.testing.assert_array_equal(out[i, : lens[i]], g[f"c{i}_out"])
        assert (out[i, lens[i]:] == O.NEVER).all()
