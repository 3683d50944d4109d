"""The sampling oracle (oracle/sampling.py) on the CPU: its Philox4x32-10 rounds against the
known-answer vectors published with the generator (Salmon et al., SC 2011, Random123
kat_vectors), the uniform mapping, and the Gumbel-max rule drawing from softmax(x / T)."""

import numpy as np
import pytest

from oracle import sampling as S

KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,want", KAT)
def test_philox_known_answers(ctr, key, want):
    got = S.philox4x32_10(np.array(ctr, dtype=np.uint32), np.array(key, dtype=np.uint32))
    assert [int(v) for v in got] == list(want)


def test_uniform_layout_and_range():
    seed, off, row = 0x0123456789ABCDEF, (7 << 32) | 9, 5
    u = S.uniforms(row, 10, seed, off)
    blocks = [S.philox4x32_10(np.array([g, row, 9, 7], dtype=np.uint32),
                              np.array([0x89ABCDEF, 0x01234567], dtype=np.uint32)) for g in range(3)]
    bits = np.concatenate(blocks)[:10]
    assert np.array_equal(u, ((bits >> 9).astype(np.float32) + np.float32(0.5)) * np.float32(2.0 ** -23))
    big = S.uniforms(0, 200_000, 1, 0)
    assert big.min() >= 2.0 ** -24 and big.max() <= 1 - 2.0 ** -24
    assert abs(float(big.mean()) - 0.5) < 5e-3


def test_greedy_is_argmax_with_first_maximum():
    x = np.array([[0.5, 2.0, 2.0, -1.0], [3.0, 1.0, 0.0, 3.0]])
    tok, logp, _ = S.sample(x, 0.8, True, 0, 0)
    assert tok.tolist() == [1, 0]
    z = x / 0.8
    lse = np.log(np.exp(z).sum(axis=1))
    assert np.allclose(logp, z[[0, 1], [1, 0]] - lse, atol=1e-14)


def test_gumbel_max_draws_from_the_softmax():
    logits = np.array([1.0, 0.0, -0.5, 2.0, 0.3, -2.0])
    temp = 0.9
    rows = 20_000
    tok, _, _ = S.sample(np.tile(logits, (rows, 1)), temp, False, 1234, 0)
    p = np.exp(logits / temp)
    p /= p.sum()
    counts = np.bincount(tok, minlength=len(logits))
    chi2 = float((((counts - rows * p) ** 2) / (rows * p)).sum())
    assert chi2 < 35.0, (counts, rows * p)   # 5 degrees of freedom: p-value ~2e-6 at 35
