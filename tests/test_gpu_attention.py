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


def _setup_cache(dtype, D, Hkv, bs, S, ctx, seed, extra_tokens=0):
    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.workloads import decode_state

    per_stream = (ctx[1] + extra_tokens) // bs + 8
    st = decode_state(num_streams=S, ctx_range=ctx, block_size=bs, num_blocks=S * per_stream,
                      evicted_spans_range=(1, 3), seed=seed)
    cache = PagedKVCache(1, Hkv, D, block_size=bs, num_blocks=st.num_blocks, dtype=dtype, max_seqs=S)
    cache.load_state(range(S), st.tables, st.positions, st.free_list)
    g = torch.Generator(device="cuda").manual_seed(seed)
    cache.k.copy_(torch.randn(cache.k.shape, generator=g, device="cuda").to(dtype))
    cache.v.copy_(torch.randn(cache.v.shape, generator=g, device="cuda").to(dtype))
    return cache, st


FUSED, PREFILL, EXACT = 1, 2, 4  # kvs_paged_decode_path bits


@pytest.mark.parametrize("dtype,D,Hq,Hkv,bs,T,S,ctx,grid,path", [
    (torch.float64, 16, 4, 2, 16, 1, 5, (3, 200), 0, EXACT),
    (torch.float64, 16, 4, 2, 4, 5, 5, (3, 200), 0, EXACT),
    (torch.float32, 16, 4, 2, 16, 1, 5, (3, 200), 0, EXACT),
    (torch.float32, 32, 8, 2, 1, 3, 5, (3, 200), 0, EXACT),
    (torch.bfloat16, 128, 32, 8, 16, 1, 5, (3, 200), 0, FUSED),
    # fused kernel with CTA ranges spanning several sequences and sequences spanning several CTAs
    (torch.bfloat16, 128, 32, 8, 16, 1, 12, (500, 3000), 0, FUSED),
    (torch.bfloat16, 128, 32, 8, 16, 1, 40, (16, 40), 0, FUSED),
    (torch.bfloat16, 128, 32, 8, 16, 1, 2, (12000, 16000), 0, FUSED),   # ~74 partials per stream to combine
    (torch.bfloat16, 128, 32, 8, 16, 1, 300, (1, 40), 0, FUSED),        # several whole streams per CTA
    (torch.bfloat16, 128, 32, 8, 16, 7, 5, (3, 200), 0, PREFILL),
    (torch.bfloat16, 64, 8, 8, 1, 1, 5, (3, 200), 0, EXACT),
    # one-token blocks (SGLang-style) on the fused decode kernel
    (torch.bfloat16, 128, 32, 8, 1, 1, 5, (3, 200), 0, FUSED),
    (torch.bfloat16, 128, 32, 8, 1, 1, 12, (500, 3000), 0, FUSED),
    (torch.bfloat16, 128, 32, 8, 1, 1, 2, (12000, 16000), 0, FUSED),
    (torch.bfloat16, 128, 32, 8, 1, 1, 300, (1, 40), 0, FUSED),
    (torch.bfloat16, 128, 32, 8, 1, 1, 300, (1, 17), 0, FUSED),          # every stream within one group
    # few CTAs: ranges of ~600 groups, so the table window of 128 groups moves several times
    (torch.bfloat16, 128, 32, 8, 1, 1, 6, (3000, 9000), 4, FUSED),
    (torch.bfloat16, 128, 32, 8, 16, 1, 6, (3000, 9000), 4, FUSED),
    # one-token blocks, chunks: the exact kernels
    (torch.bfloat16, 128, 32, 8, 1, 5, 4, (3, 200), 0, EXACT),
])
def test_paged_forward_matches_oracle(dtype, D, Hq, Hkv, bs, T, S, ctx, grid, path):
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
    ran = []
    out = ops.paged_forward(cache, list(range(S)), None if T == 1 else counts, 0, q, k, v, pos, mapping,
                            rope.table(q.device, dtype), D ** -0.5, grid_ctas=grid, report_path=ran)
    torch.cuda.synchronize()
    assert ran == [path]
    odt = np.float64 if dtype == torch.float64 else np.float32
    qn, kn, vn, pn = _np(q), _np(k), _np(v), pos.cpu().numpy()
    q_rot = O.rope_apply(qn, pn, theta, odt).astype(np.float64)
    k_rot = O.rope_apply(kn, pn, theta, odt).astype(np.float64)
    pool_k, pool_v = _np(old_k)[0], _np(cache.v)[0]
    new_k = _np(cache.k)[0]
    blocks = mapping.blocks.cpu().numpy()
    offs = mapping.offsets.cpu().numpy()
    # the appended keys are the rotated new keys (bf16: rounded once, so within one bf16 ulp of
    # the float32 rotation, 2^-7 relative: a fixed absolute bound fails for keys above ~4)
    if dtype == torch.bfloat16:
        np.testing.assert_allclose(new_k[blocks, offs], k_rot, rtol=2.0 ** -7, atol=1e-6)
    else:
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


@pytest.mark.parametrize("Hq,Hkv,counts,ctx", [
    (32, 8, [300, 1, 129, 128], (3, 700)),   # several query tiles, a single token, tile edges
    (8, 2, [17, 256, 200], (1000, 2500)),    # long contexts: key tiles across many blocks
    (4, 2, [5, 64, 130, 1, 90], (1, 40)),    # group of 2; tiny contexts
])
def test_paged_prefill_chunks_match_oracle(Hq, Hkv, counts, ctx):
    """Ragged bf16 chunks (D 128, 16-token blocks, even GQA group) take the tensor-core paged
    prefill: RoPE + append, then attention over the pool through the block tables."""
    from kvstreams import ops
    from kvstreams.rope import RotaryEmbedding

    dtype, D, bs = torch.bfloat16, 128, 16
    S = len(counts)
    cache, st = _setup_cache(dtype, D, Hkv, bs, S, ctx, seed=sum(counts) + Hq, extra_tokens=max(counts))
    rope = RotaryEmbedding(D, 5e5)
    g = torch.Generator(device="cuda").manual_seed(11)
    N = sum(counts)
    q = torch.randn(N, Hq, D, generator=g, device="cuda").to(dtype)
    k = torch.randn(N, Hkv, D, generator=g, device="cuda").to(dtype)
    v = torch.randn(N, Hkv, D, generator=g, device="cuda").to(dtype)
    pos = torch.cat([torch.arange(int(p), int(p) + c) for p, c in zip(st.next_positions, counts)]).cuda()
    old_k = cache.k.clone()
    old_tables = [cache.block_table(s) for s in range(S)]
    old_len = [cache.num_tokens(s) for s in range(S)]
    mapping = cache.append_slots_batch(list(range(S)), pos, counts)
    out = ops.paged_forward(cache, list(range(S)), counts, 0, q, k, v, pos, mapping, rope.table(q.device, dtype),
                            D ** -0.5)
    cache.sync()
    qn, kn, pn = _np(q), _np(k), pos.cpu().numpy()
    q_rot = O.rope_apply(qn, pn, 5e5, np.float32).astype(np.float64)
    k_rot = O.rope_apply(kn, pn, 5e5, np.float32).astype(np.float64)
    pool_k, pool_v = _np(old_k)[0], _np(cache.v)[0]
    got = _np(out)
    start = 0
    for s, T in enumerate(counts):
        tab = old_tables[s] + cache.block_table(s)[len(old_tables[s]):]
        n_old = old_len[s]
        ks = pool_k[tab].reshape(-1, Hkv, D)[:n_old]
        vs = pool_v[tab].reshape(-1, Hkv, D)[:n_old + T]
        sl = slice(start, start + T)
        keys = np.concatenate([ks, k_rot[sl]])
        mask = np.ones((T, n_old + T), dtype=bool)
        mask[:, n_old:] = np.tril(np.ones((T, T), dtype=bool))
        want = O.gqa_attention(q_rot[sl], keys, vs, mask, D ** -0.5)
        np.testing.assert_allclose(got[sl], want, rtol=0, atol=TOL[dtype], err_msg=f"stream {s}")
        start += T


def _oracle_paged(q_rot, k_rot, pool_k, pool_v, table, n_old, T, Hkv, D):
    ks = pool_k[table].reshape(-1, Hkv, D)[:n_old]
    vs = pool_v[table].reshape(-1, Hkv, D)[:n_old + T]
    keys = np.concatenate([ks, k_rot])
    mask = np.ones((T, n_old + T), dtype=bool)
    mask[:, n_old:] = np.tril(np.ones((T, T), dtype=bool))
    return O.gqa_attention(q_rot, keys, vs, mask, D ** -0.5)


def test_prefill_then_decode_share_scratch_any_slot_order():
    """Chunked prefills and decode steps of different batch sizes, slots in any order, one
    after the other on one cache: they share one scratch buffer, which every call must leave
    as the next expects (regressions: arrival counters at a batch-size dependent offset, and
    prefill tile offsets read back as counters)."""
    from kvstreams import ops
    from kvstreams.rope import RotaryEmbedding

    dtype, D, Hq, Hkv, bs, S = torch.bfloat16, 128, 32, 8, 16, 12
    cache, st = _setup_cache(dtype, D, Hkv, bs, S, (50, 900), seed=5, extra_tokens=200)
    rope = RotaryEmbedding(D, 5e5)
    inv = rope.table("cuda", dtype)
    g = torch.Generator(device="cuda").manual_seed(3)
    nxt = [int(p) for p in st.next_positions]
    steps = [([5, 2, 9], [40, 7, 130]), ([7, 0, 11, 3, 1, 10, 4, 8, 6, 2, 9, 5], None),
             ([4, 1, 10, 6, 2], None), ([3, 8], [17, 64]), ([0, 11, 5, 9, 7, 3, 1], None),
             (list(range(12)), None)]
    for seqs, counts in steps:
        c = counts or [1] * len(seqs)
        N = sum(c)
        q = torch.randn(N, Hq, D, generator=g, device="cuda").to(dtype)
        k = torch.randn(N, Hkv, D, generator=g, device="cuda").to(dtype)
        v = torch.randn(N, Hkv, D, generator=g, device="cuda").to(dtype)
        pos = torch.cat([torch.arange(nxt[s], nxt[s] + n) for s, n in zip(seqs, c)]).cuda()
        old_k, old_tables = cache.k.clone(), [cache.block_table(s) for s in seqs]
        old_len = [cache.num_tokens(s) for s in seqs]
        mapping = cache.append_slots_batch(seqs, pos, counts)
        out = ops.paged_forward(cache, seqs, counts, 0, q, k, v, pos, mapping, inv, D ** -0.5)
        cache.sync()
        pn = pos.cpu().numpy()
        q_rot = O.rope_apply(_np(q), pn, 5e5, np.float32).astype(np.float64)
        k_rot = O.rope_apply(_np(k), pn, 5e5, np.float32).astype(np.float64)
        pool_k, pool_v = _np(old_k)[0], _np(cache.v)[0]
        got = _np(out)
        start = 0
        for i, (s, n) in enumerate(zip(seqs, c)):
            tab = old_tables[i] + cache.block_table(s)[len(old_tables[i]):]
            sl = slice(start, start + n)
            want = _oracle_paged(q_rot[sl], k_rot[sl], pool_k, pool_v, tab, old_len[i], n, Hkv, D)
            np.testing.assert_allclose(got[sl], want, rtol=0, atol=TOL[dtype], err_msg=f"sequence {s}")
            start += n
            nxt[s] += n


@pytest.mark.parametrize("S,ctx,grid", [
    (40, (50, 900), 0),      # one CTA per SM, every range's block ids staged in shared memory
    (4, (8500, 9500), 1),    # one CTA over > 2048 groups: block ids read from the plan in global memory
    (2, (40, 60), 0),        # fewer groups than CTAs: most stored ranges are empty
])
def test_decode_plan_reuse_equals_recompute(S, ctx, grid):
    """The layers of a decode step with the batch plan stored by the first layer and read back
    by the others (KVS_PLAN_BUILD / KVS_PLAN_REUSE) give the same bits as layers that each
    compute it; a REUSE call after a BUILD for another batch size computes the plan itself."""
    from kvstreams import _native as N
    from kvstreams import ops
    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.rope import RotaryEmbedding
    from kvstreams.workloads import decode_state

    dtype, D, Hq, Hkv, bs, L = torch.bfloat16, 128, 32, 8, 16, 3
    st = decode_state(num_streams=S, ctx_range=ctx, block_size=bs, num_blocks=S * (ctx[1] // bs + 16), seed=11)
    cache = PagedKVCache(L, Hkv, D, block_size=bs, num_blocks=st.num_blocks, dtype=dtype, max_seqs=S,
                         max_blocks_per_seq=ctx[1] // bs + 16)
    cache.load_state(range(S), st.tables, st.positions, st.free_list)
    g = torch.Generator(device="cuda").manual_seed(4)
    cache.k.copy_(torch.randn(cache.k.shape, generator=g, device="cuda").to(dtype))
    cache.v.copy_(torch.randn(cache.v.shape, generator=g, device="cuda").to(dtype))
    inv = RotaryEmbedding(D, 5e5).table("cuda", dtype)
    pos = torch.as_tensor(st.next_positions, device="cuda")
    for step in range(3):
        seqs = list(range(S)) if step != 1 else list(range(S - 1))  # step 1: another batch size
        p = pos[: len(seqs)] + step
        q = torch.randn(len(seqs), L, Hq, D, generator=g, device="cuda").to(dtype)
        k = torch.randn(len(seqs), L, Hkv, D, generator=g, device="cuda").to(dtype)
        v = torch.randn(len(seqs), L, Hkv, D, generator=g, device="cuda").to(dtype)
        mapping = cache.append_slots_batch(seqs, p)
        batch = cache._batch(seqs)
        for mode in ("plan", "none"):
            outs = []
            for layer in range(L):
                if mode == "none":
                    plan = N.PLAN_NONE
                elif step == 1:
                    plan = N.PLAN_REUSE  # the stored plan is for S sequences: computed instead
                else:
                    plan = N.PLAN_BUILD if layer == 0 else N.PLAN_REUSE
                path = []
                outs.append(ops.paged_forward(cache, seqs, None, layer, q[:, layer], k[:, layer], v[:, layer], p,
                                              mapping, inv, D ** -0.5, grid_ctas=grid, batch=batch, plan=plan,
                                              report_path=path))
                assert path == [FUSED]
            if mode == "plan":
                with_plan = outs
        for layer in range(L):
            assert torch.equal(with_plan[layer], outs[layer]), f"step {step} layer {layer}"
    # the plan path against the oracle on the last step's first layer
    pn = p.cpu().numpy()
    q_rot = O.rope_apply(_np(q[:, 0]), pn, 5e5, np.float32).astype(np.float64)
    got = _np(with_plan[0])
    for s in (0, S - 1):
        tab = torch.as_tensor(cache.block_table(s), device="cuda")
        n = cache.num_tokens(s)
        keys = _np(cache.k[0].index_select(0, tab).reshape(-1, Hkv, D)[:n])
        vals = _np(cache.v[0].index_select(0, tab).reshape(-1, Hkv, D)[:n])
        want = O.gqa_attention(q_rot[s:s + 1], keys, vals, np.ones((1, n), dtype=bool), D ** -0.5)
        np.testing.assert_allclose(got[s:s + 1], want, rtol=0, atol=TOL[dtype], err_msg=f"stream {s}")


@pytest.mark.parametrize("dtype,D,Hq,Hkv,counts", [
    (torch.bfloat16, 128, 32, 8, [1] * 9),               # fused decode kernel
    (torch.bfloat16, 128, 32, 8, [40, 17, 1, 1, 1]),     # mixed step: prefill chunks + decode tail
    (torch.float32, 32, 8, 2, [3, 1, 5]),                # generic path (RoPE kernels + exact attention)
])
def test_paged_forward_strided_qkv_equals_packed(dtype, D, Hq, Hkv, counts):
    """q, k_new, v_new given as the column blocks of one fused [tokens, q|k|v] projection output
    (rows q_stride / kv_stride apart, no copies) give the same bits as packed tensors: the
    output and the keys/values appended to the pool."""
    from kvstreams import ops
    from kvstreams.rope import RotaryEmbedding

    S = len(counts)
    cache, st = _setup_cache(dtype, D, Hkv, 16, S, (30, 600), seed=9, extra_tokens=max(counts))
    rope = RotaryEmbedding(D, 5e5)
    inv = rope.table("cuda", dtype)
    g = torch.Generator(device="cuda").manual_seed(4)
    n = sum(counts)
    nq, nk = Hq * D, Hkv * D
    qkv = torch.randn(n, nq + 2 * nk, generator=g, device="cuda").to(dtype)
    q = qkv[:, :nq].reshape(n, Hq, D)
    k = qkv[:, nq:nq + nk].reshape(n, Hkv, D)
    v = qkv[:, nq + nk:].reshape(n, Hkv, D)
    assert not q.is_contiguous() and q.stride(0) == nq + 2 * nk
    pos = torch.cat([torch.arange(int(p), int(p) + c) for p, c in zip(st.next_positions, counts)]).cuda()
    tail = 0  # one-token sequences at the end, after at least one chunk
    while tail < len(counts) and counts[-1 - tail] == 1:
        tail += 1
    if tail == len(counts):
        tail = 0
    snap = cache.snapshot_state()
    outs, pools = [], []
    for packed in (False, True):
        cache.restore_state(snap)
        mapping = cache.append_slots_batch(list(range(S)), pos, counts)
        args = (q.contiguous(), k.contiguous(), v.contiguous()) if packed else (q, k, v)
        out = ops.paged_forward(cache, list(range(S)), counts, 0, *args, pos, mapping, inv, D ** -0.5,
                                tail_singles=tail)
        cache.sync()
        outs.append(out.clone())
        pools.append((cache.k.clone(), cache.v.clone()))
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(pools[0][0], pools[1][0]) and torch.equal(pools[0][1], pools[1][1])


def test_paged_decode_unaligned_inputs_take_the_exact_path():
    """q / k_new / v_new that are not 16-byte aligned (views one element into a buffer) run the
    exact kernels instead of the fused decode kernel, which reads them with 16-byte loads: the
    appended keys and values are bit-identical and the outputs agree within bf16 tolerance."""
    from kvstreams import ops
    from kvstreams.rope import RotaryEmbedding

    dtype, D, Hq, Hkv, S = torch.bfloat16, 128, 32, 8, 9
    cache, st = _setup_cache(dtype, D, Hkv, 16, S, (30, 600), seed=21)
    inv = RotaryEmbedding(D, 5e5).table("cuda", dtype)
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(S, Hq, D, generator=g, device="cuda").to(dtype)
    k = torch.randn(S, Hkv, D, generator=g, device="cuda").to(dtype)
    v = torch.randn(S, Hkv, D, generator=g, device="cuda").to(dtype)

    def shifted(t):  # same values, one element past a 16-byte boundary
        buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
        view = buf[1:].view(t.shape)
        view.copy_(t)
        assert view.data_ptr() % 16 != 0
        return view

    pos = torch.as_tensor(st.next_positions, device="cuda")
    snap = cache.snapshot_state()
    outs, pools = [], []
    for args in ((q, k, v), (shifted(q), shifted(k), shifted(v))):
        cache.restore_state(snap)
        mapping = cache.append_slots_batch(list(range(S)), pos)
        out = ops.paged_forward(cache, list(range(S)), None, 0, *args, pos, mapping, inv, D ** -0.5)
        cache.sync()
        outs.append(out.float().clone())
        pools.append((cache.k.clone(), cache.v.clone()))
    assert torch.equal(pools[0][0], pools[1][0]) and torch.equal(pools[0][1], pools[1][1])
    assert (outs[0] - outs[1]).abs().max().item() <= TOL[dtype]


@pytest.mark.parametrize("dtype,D,H", [(torch.bfloat16, 128, 32), (torch.float16, 64, 8), (torch.float32, 128, 8),
                                       (torch.float64, 16, 4)])
def test_rope_vector_path_equals_scalar_path(dtype, D, H):
    """The 16-byte-chunk RoPE kernel (one angle per token and frequency, shared by the heads)
    gives the same bits as the per-pair kernel, which unaligned rows still take."""
    from kvstreams import ops
    from kvstreams.rope import RotaryEmbedding

    n = 1000
    g = torch.Generator(device="cuda").manual_seed(D + H)
    x = torch.randn(n, H, D, generator=g, device="cuda", dtype=torch.float64).to(dtype)
    pos = torch.randint(0, 200_000, (n,), generator=g, device="cuda")
    inv = RotaryEmbedding(D, 5e5).table("cuda", dtype)
    a = ops.rope_(x.clone(), pos, inv)
    buf = torch.empty(x.numel() + 1, dtype=dtype, device="cuda")
    xs = buf[1:].view(x.shape)
    xs.copy_(x)
    assert xs.data_ptr() % 16 != 0
    b = ops.rope_(xs, pos, inv)
    assert torch.equal(a, b)


def test_rope_copy_from_fused_projection_equals_in_place():
    """ops.rope on the q / k column blocks of a fused [tokens, q|k|v] output (one pass, strided
    rows) gives the same bits as copying them out and rotating in place."""
    from kvstreams import ops
    from kvstreams.rope import RotaryEmbedding

    B, T, Hq, Hkv, D = 2, 300, 32, 8, 128
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn(B, T, (Hq + 2 * Hkv) * D, generator=g, device="cuda").bfloat16()
    q = qkv[..., : Hq * D].view(B, T, Hq, D)
    k = qkv[..., Hq * D: (Hq + Hkv) * D].view(B, T, Hkv, D)
    pos = torch.randint(0, 40_000, (B, T), generator=g, device="cuda")
    inv = RotaryEmbedding(D, 5e5).table("cuda", torch.bfloat16)
    for x in (q, k):
        got = ops.rope(x, pos, inv)
        assert got.is_contiguous() and got.shape == x.shape
        assert torch.equal(got, ops.rope_(x.contiguous().clone(), pos, inv))
    # and back: packed rows rotated into a column block of a fused tensor
    dst = torch.zeros_like(qkv)
    ops.rope(q.contiguous(), -pos, inv, out=dst[..., : Hq * D].view(B, T, Hq, D))
    assert torch.equal(dst[..., : Hq * D].reshape(B, T, Hq, D), ops.rope_(q.contiguous().clone(), -pos, inv))
    assert not dst[..., Hq * D:].any()
