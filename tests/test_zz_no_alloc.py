"""kvs_evict_positions_noalloc, the eviction entry point for callers that cannot allocate
device memory (hosts binding the C ABI without a device allocator, or rollout loops that
must not cudaMalloc between steps), gives exactly what kvs_evict_positions gives.

Two identical caches are evicted twice in a row -- one through the allocating entry point
(scratch from the caller), one through the no-alloc entry point called directly over the
C ABI -- and every output and every piece of cache state must be bit-identical (integer
work: the tolerance is zero).  Runs alone in a fresh process or after the other tests."""

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

STREAMS, BLOCKS, BS = 40, 64, 16


def _build():
    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.workloads import compaction_plan

    rounds = compaction_plan(num_streams=STREAMS, blocks_per_stream=BLOCKS, block_size=BS, seed=11,
                             num_events_range=(2, 2))
    cache = PagedKVCache(1, 1, 2, block_size=BS, num_blocks=STREAMS * BLOCKS + 32, dtype=torch.float32,
                         max_seqs=STREAMS, max_blocks_per_seq=BLOCKS + 16)
    for s in range(STREAMS):
        cache.add_sequence(s)
    return cache, rounds


def _append_round(cache, rd):
    seqs, poss = rd.append_seqs, rd.append_positions
    start = 0
    while start < len(seqs):
        seen, end = set(), start
        while end < len(seqs) and seqs[end] not in seen:
            seen.add(seqs[end])
            end += 1
        cache.append_slots_batch(seqs[start:end], torch.as_tensor(np.concatenate(poss[start:end])),
                                 [p.size for p in poss[start:end]])
        start = end


def _noalloc_evict(cache, seq_ids, spans, cap):
    """Call kvs_evict_positions_noalloc through the C ABI with device inputs/outputs."""
    from kvstreams import _native as N
    from kvstreams.utils.spans import merge_spans

    merged = [merge_spans(sp) for sp in spans]
    cu = np.zeros(len(seq_ids) + 1, dtype=np.int32)
    cu[1:] = np.cumsum([len(m) for m in merged])
    flat = np.asarray([x for m in merged for x in m], dtype=np.int64).reshape(-1, 2)
    dev = cache.device
    cu_t = torch.from_numpy(cu).to(dev)
    st_t = torch.from_numpy(np.ascontiguousarray(flat[:, 0])).to(dev)
    en_t = torch.from_numpy(np.ascontiguousarray(flat[:, 1])).to(dev)
    out = torch.full((len(seq_ids), cap, 2), -7, dtype=torch.long, device=dev)
    counts = torch.full((len(seq_ids),), -7, dtype=torch.int32, device=dev)
    slots = [cache.slot(s) for s in seq_ids]
    b, keep = cache._batch(slots)
    rc = N.lib().kvs_evict_positions_noalloc(C.byref(cache.struct), C.byref(b), cu_t.data_ptr(), st_t.data_ptr(),
                                             en_t.data_ptr(), out.data_ptr(), counts.data_ptr(), cap,
                                             N.stream_ptr(dev))
    assert rc == 0, rc
    torch.cuda.synchronize()
    cache.refresh(seq_ids)
    return out, counts


def _state(cache):
    st = cache.stats
    return {
        "tables": [cache.block_table(s) for s in range(STREAMS)],
        "lengths": [cache.num_tokens(s) for s in range(STREAMS)],
        "free": cache.allocator.free_list(),
        "slot_pos": cache.slot_pos.cpu().numpy().tobytes(),
        "stats": (st.evicted_tokens, st.evicted_blocks, st.eviction_calls, st.shrunk_tokens),
        "status": cache._status.cpu().tolist(),
    }


def test_noalloc_eviction_equals_allocating_entry_point_twice():
    a, rounds = _build()
    b, _ = _build()
    _append_round(a, rounds[0])
    _append_round(b, rounds[0])
    assert _state(a) == _state(b)
    cap = 64
    for rd in rounds[1:3]:  # two eviction calls in a row
        assert rd.evict_seqs
        out_a, counts_a, _ = a.evict_positions_async(rd.evict_seqs, rd.evict_spans, span_cap=cap)
        torch.cuda.synchronize()
        a.refresh(rd.evict_seqs)
        out_b, counts_b = _noalloc_evict(b, rd.evict_seqs, rd.evict_spans, cap)
        ca = counts_a.cpu().numpy()
        assert np.array_equal(ca, counts_b.cpu().numpy())
        oa, ob = out_a.cpu().numpy(), out_b.cpu().numpy()
        for i, n in enumerate(ca):
            assert np.array_equal(oa[i, :n], ob[i, :n])
        assert _state(a) == _state(b)
        _append_round(a, rd)
        _append_round(b, rd)
        assert _state(a) == _state(b)


def test_noalloc_on_a_second_stream_after_synchronising():
    """The supported reuse pattern: a later call on another stream, once the earlier calls have
    finished, finds the shared array (and this device's cached address) as good as new."""
    a, rounds = _build()
    b, _ = _build()
    cap = 64
    for rd in rounds[:2]:  # a round evicts first, then appends its refills
        if rd.evict_seqs:
            a.evict_positions_async(rd.evict_seqs, rd.evict_spans, span_cap=cap)
            torch.cuda.synchronize()
            a.refresh(rd.evict_seqs)
            _noalloc_evict(b, rd.evict_seqs, rd.evict_spans, cap)
        _append_round(a, rd)
        _append_round(b, rd)
    rd = rounds[2]
    out_a, counts_a, _ = a.evict_positions_async(rd.evict_seqs, rd.evict_spans, span_cap=cap)
    torch.cuda.synchronize()
    a.refresh(rd.evict_seqs)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        out_b, counts_b = _noalloc_evict(b, rd.evict_seqs, rd.evict_spans, cap)
    torch.cuda.synchronize()
    ca = counts_a.cpu().numpy()
    assert np.array_equal(ca, counts_b.cpu().numpy())
    oa, ob = out_a.cpu().numpy(), out_b.cpu().numpy()
    for i, n in enumerate(ca):
        assert np.array_equal(oa[i, :n], ob[i, :n])
    assert _state(a) == _state(b)


def test_noalloc_rejects_more_sequences_than_its_limit():
    """257 sequences (one more than the built-in scratch holds): KVS_E_NOALLOC_LIMIT, and the
    cache is untouched."""
    from kvstreams import _native as N
    from kvstreams.paged_cache import PagedKVCache

    n = 257
    cache = PagedKVCache(1, 1, 2, block_size=16, num_blocks=n * 4, dtype=torch.float32, max_seqs=n,
                         max_blocks_per_seq=4)
    for s in range(n):
        cache.add_sequence(s)
    cache.append_slots_batch(list(range(n)), torch.arange(n * 32) % 32, [32] * n)
    before = (cache._tables.clone(), cache._lengths.clone(), cache._free_stack.clone(), cache.slot_pos.clone())
    b, keep = cache._batch([cache.slot(s) for s in range(n)])
    dummy = torch.zeros(n * 4, dtype=torch.long, device=cache.device)
    rc = N.lib().kvs_evict_positions_noalloc(C.byref(cache.struct), C.byref(b), dummy.data_ptr(), dummy.data_ptr(),
                                             dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), 1,
                                             N.stream_ptr(cache.device))
    torch.cuda.synchronize()
    assert rc == -5
    after = (cache._tables, cache._lengths, cache._free_stack, cache.slot_pos)
    assert all(torch.equal(x, y) for x, y in zip(before, after))


def test_noalloc_rejects_batches_beyond_its_limit():
    from kvstreams import _native as N
    from kvstreams.paged_cache import PagedKVCache

    big = PagedKVCache(1, 1, 2, block_size=1, num_blocks=4096, dtype=torch.float32, max_seqs=4,
                       max_blocks_per_seq=2048)
    big.add_sequence(0)
    b, keep = big._batch([big.slot(0)])
    dummy = torch.zeros(4, dtype=torch.long, device=big.device)
    rc = N.lib().kvs_evict_positions_noalloc(C.byref(big.struct), C.byref(b), dummy.data_ptr(), dummy.data_ptr(),
                                             dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), 1,
                                             N.stream_ptr(big.device))
    assert rc == -5  # KVS_E_NOALLOC_LIMIT: nothing launched
