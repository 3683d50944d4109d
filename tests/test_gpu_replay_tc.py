"""tcgen05/TMEM path: the UMMA self-test against a plain matmul, and the masked replay
kernel against the exact SIMT kernel and the oracle (bf16 tolerance 3e-2 on O(1) outputs)."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import kvs_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_umma_selftest_matches_matmul(mode):
    """mode bit 0: B MN-major (else K-major); bit 1: A staged in TMEM (else shared memory)."""
    from kvstreams import _native as N

    b_mn = mode & 1
    g = torch.Generator(device="cuda").manual_seed(mode)
    a = torch.randn(128, 128, generator=g, device="cuda").bfloat16()
    b = torch.randn(128, 128, generator=g, device="cuda").bfloat16()  # bt[n][k] or b[k][n]
    c = torch.zeros(128, 128, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = N.lib().kvs_selftest_umma(a.data_ptr(), b.data_ptr(), c.data_ptr(), mode, err.data_ptr(),
                                   N.stream_ptr())
    assert rc == 0
    torch.cuda.synchronize()
    assert err.item() == 0
    want = a.float() @ (b.float() if b_mn else b.float().t())
    torch.testing.assert_close(c, want, rtol=1e-3, atol=1e-2)


def _inputs(B, T, Hq, Hkv, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, T, Hq, 128, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, T, Hkv, 128, generator=g, device="cuda").bfloat16()
    v = torch.randn(B, T, Hkv, 128, generator=g, device="cuda").bfloat16()
    return q, k, v


@pytest.mark.parametrize("one_head", [False, True])
@pytest.mark.parametrize("B,T,Hq,Hkv,evict,lengths", [
    (2, 1024, 8, 2, True, None),        # GQA group of 4: head pairs share K/V tiles
    (2, 1000, 4, 4, True, [1000, 700]),  # group of 1: one head per CTA
    (1, 1536, 4, 1, False, None),       # causal only: unmasked fast-path tiles
    (3, 300, 8, 2, True, [300, 129, 1]),
    (1, 600, 6, 3, True, None),         # group of 2, ragged last query tile
])
def test_replay_tc_matches_exact_kernel(B, T, Hq, Hkv, evict, lengths, one_head):
    from kvstreams import ops
    from kvstreams.workloads import replay_evicted_at

    q, k, v = _inputs(B, T, Hq, Hkv, seed=T + Hq)
    if evict:
        ev, _ = replay_evicted_at(batch=B, seq_len=T, events_range=(2, 5), mean_turn=48, seed=T)
    else:
        ev = np.full((B, T), O.NEVER, dtype=np.int64)
    ln = np.asarray(lengths or [T] * B, dtype=np.int32)
    ev_t, ln_t = torch.from_numpy(ev).cuda(), torch.from_numpy(ln).cuda()
    fast = ops.replay_attention(q, k, v, ev_t, ln_t, 128 ** -0.5, one_head_per_cta=one_head)
    exact = ops.replay_attention(q, k, v, ev_t, ln_t, 128 ** -0.5, force_generic=True)
    torch.cuda.synchronize()
    torch.testing.assert_close(fast.float(), exact.float(), rtol=0, atol=3e-2)
    # and the oracle on a slice of rows of the first stream
    f = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    want = O.replay_attention(f(q[:1]), f(k[:1]), f(v[:1]), ev[:1], ln[:1], 128 ** -0.5)
    np.testing.assert_allclose(f(fast[:1]), want, rtol=0, atol=3e-2)
