"""Device parity at the benchmark configurations' full sizes.

* Compaction (256 streams x 512-block tables, pool 200000, Geometric(96) turns padded to the
  block size, 1-8 keep-recent events per stream with keep_last ~U[1,4], prompt pinned; block
  size 16 and 1): tables, free list, slot_pos, lengths, evicted spans, stats and evicted_at
  bit-exact against the sequential oracle.
* Paged decode (64 streams, live contexts ~U[1024,16384], pool of 131072 16-token blocks or
  the same bytes in one-token blocks, 32q/8kv, D 128, theta 5e5, bf16): the fused kernel's
  outputs for sampled streams (the longest and shortest included) against the float64 oracle.
* Masked replay (one stream of 32768 tokens, 3-8 keep-recent events, 32q/8kv, D 128, bf16):
  the tensor-core replay against the float64 oracle on sampled rows -- the last query tile,
  the rows on both sides of every eviction time and random rows.

Tolerance for bf16 outputs: 3e-2 absolute against the float64 oracle evaluated on the same
bf16-rounded inputs (as the other kernel tests)."""

import numpy as np
import pytest
import torch

from oracle import kvs_oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 3e-2


def _f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("bs", [16, 1])
def test_compaction_full_size_bit_exact(bs):
    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.workloads import compaction_plan

    streams, blocks, pool = 256, 512, 200000
    rounds = compaction_plan(num_streams=streams, blocks_per_stream=blocks, block_size=bs, num_events_range=(1, 8),
                             seed=11)
    assert max(len(rd.evict_seqs) for rd in rounds[1:]) > 0 and len(rounds) >= 3
    cache = PagedKVCache(1, 1, 2, block_size=bs, num_blocks=pool, dtype=torch.bfloat16, max_seqs=streams,
                         max_blocks_per_seq=blocks + 256)
    ref = O.OracleCache(pool, bs)
    next_pos = [0] * streams
    triples = [[] for _ in range(streams)]
    for s in range(streams):
        cache.add_sequence(s)
        ref.add_sequence(s)
    for rd in rounds:
        if rd.evict_seqs:
            got = cache.evict_positions_batch(rd.evict_seqs, rd.evict_spans)
            want = [ref.evict_positions(s, sp) for s, sp in zip(rd.evict_seqs, rd.evict_spans)]
            assert got == want
            for s, spans in zip(rd.evict_seqs, got):
                triples[s] += [(a, b, next_pos[s]) for a, b in spans]
            cache.check_invariants_batch(rd.evict_seqs)
        # appends: batches of distinct sequences, in plan order
        seqs, poss = rd.append_seqs, rd.append_positions
        start = 0
        while start < len(seqs):
            seen, end = set(), start
            while end < len(seqs) and seqs[end] not in seen:
                seen.add(seqs[end])
                end += 1
            cache.append_slots_batch(seqs[start:end], torch.as_tensor(np.concatenate(poss[start:end])),
                                     [p.size for p in poss[start:end]])
            for s, p in zip(seqs[start:end], poss[start:end]):
                ref.append_slots(s, p.tolist())
                next_pos[s] = int(p[-1]) + 1
            start = end
        tables = cache._tables.cpu().numpy()
        n_blocks = cache._n_blocks.cpu().numpy()
        lengths = cache._lengths.cpu().numpy()
        for s in range(streams):
            slot = cache.slot(s)
            assert tables[slot, : n_blocks[slot]].tolist() == ref.tables[s], f"stream {s}"
            assert int(lengths[slot]) == ref.lengths[s]
        assert cache.allocator.free_list() == ref.free
    st = cache.stats
    assert [st.written_tokens, st.evicted_tokens, st.evicted_blocks, st.truncated_tokens, st.peak_blocks,
            st.eviction_calls, st.shrunk_tokens] == ref.stats.as_list()
    np.testing.assert_array_equal(cache.slot_pos.cpu().numpy(), ref.slot_pos)
    # evicted_at of every stream's compaction log (the evicted_at kernel, events.py:66-74)
    from kvstreams import ops

    lengths = list(next_pos)
    cu = np.zeros(streams + 1, dtype=np.int32)
    np.cumsum([len(t) for t in triples], out=cu[1:])
    flat = np.asarray([x for t in triples for x in t], dtype=np.int64).reshape(-1, 3)
    dev = ops.evicted_at_from_spans(cu, flat, lengths, "cuda", max(lengths)).cpu().numpy()
    for s in range(streams):
        np.testing.assert_array_equal(dev[s, : lengths[s]], O.evicted_at(triples[s], lengths[s]))
        assert (dev[s, lengths[s]:] == O.NEVER).all()


@pytest.mark.parametrize("bs", [16, 1])
def test_paged_decode_full_size(bs):
    from kvstreams import ops
    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.rope import RotaryEmbedding
    from kvstreams.workloads import decode_state

    S, Hq, Hkv, D, theta = 64, 32, 8, 128, 5e5
    nb = 131072 * 16 // bs
    st = decode_state(num_streams=S, ctx_range=(1024, 16384), block_size=bs, num_blocks=nb, seed=1000)
    cache = PagedKVCache(1, Hkv, D, block_size=bs, num_blocks=nb, dtype=torch.bfloat16, max_seqs=S,
                         max_blocks_per_seq=(16384 + 4096) // bs)
    cache.load_state(range(S), st.tables, st.positions, st.free_list)
    g = torch.Generator(device="cuda").manual_seed(5)
    for t in (cache.k, cache.v):
        t.view(-1)[:] = torch.randn(t.numel(), generator=g, device="cuda").bfloat16()
    q = torch.randn(S, Hq, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(S, Hkv, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(S, Hkv, D, generator=g, device="cuda").bfloat16()
    pos = torch.as_tensor(st.next_positions, device="cuda")
    old_len = st.lengths.copy()
    mapping = cache.append_slots_batch(list(range(S)), pos)
    ran = []
    out = ops.paged_forward(cache, list(range(S)), None, 0, q, k, v, pos, mapping,
                            RotaryEmbedding(D, theta).table("cuda", torch.bfloat16), D ** -0.5, report_path=ran)
    torch.cuda.synchronize()
    assert ran == [1], "the fused decode kernel"
    order = np.argsort(old_len)
    sample = sorted({int(order[0]), int(order[1]), int(order[-1]), int(order[-2]), *range(0, S, 9)})
    assert len(sample) >= 8
    pn = pos.cpu().numpy()
    q_rot = O.rope_apply(_f64(q), pn, theta, np.float32).astype(np.float64)
    k_rot = O.rope_apply(_f64(k), pn, theta, np.float32).astype(np.float64)
    got = _f64(out)
    for s in sample:
        tab = torch.as_tensor(cache.block_table(s), device="cuda")
        n = int(old_len[s]) + 1
        keys = _f64(cache.k[0].index_select(0, tab).reshape(-1, Hkv, D)[:n])
        vals = _f64(cache.v[0].index_select(0, tab).reshape(-1, Hkv, D)[:n])
        # the appended key is the rotated new key, rounded once to bf16
        np.testing.assert_allclose(keys[-1], k_rot[s], rtol=2.0 ** -7, atol=1e-6)
        np.testing.assert_array_equal(vals[-1], _f64(v)[s])
        want = O.gqa_attention(q_rot[s:s + 1], keys, vals, np.ones((1, n), dtype=bool), D ** -0.5)
        np.testing.assert_allclose(got[s:s + 1], want, rtol=0, atol=BF16_TOL, err_msg=f"stream {s} ({n} entries)")


def test_replay_full_length_stream():
    from kvstreams import ops
    from kvstreams.workloads import replay_evicted_at

    T, Hq, Hkv, D = 32768, 32, 8, 128
    ev, triples = replay_evicted_at(batch=1, seq_len=T, seed=4)
    assert len(triples[0]) >= 3
    g = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn(1, T, Hq, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(1, T, Hkv, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(1, T, Hkv, D, generator=g, device="cuda").bfloat16()
    out = ops.replay_attention(q, k, v, torch.from_numpy(ev).cuda(), torch.full((1,), T, dtype=torch.int32,
                                                                                device="cuda"), D ** -0.5)
    rng = np.random.default_rng(0)
    rows = set(range(T - 128, T, 2))            # the last query tile (the 256-tile list's edge)
    for s, e, t in triples[0]:                  # both sides of every eviction time
        rows.update(x for x in (t - 1, t, t + 1) if 0 <= x < T)
    rows.update({0, 1, 127, 128, 129})
    rows.update(int(x) for x in rng.integers(0, T, size=64))
    rows = sorted(rows)
    want = O.replay_attention_rows(_f64(q[0]), _f64(k[0]), _f64(v[0]), ev[0], rows, D ** -0.5)
    got = _f64(out[0, rows])
    np.testing.assert_allclose(got, want, rtol=0, atol=BF16_TOL)
