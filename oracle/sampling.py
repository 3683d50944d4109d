"""CPU oracle of the batched sampling kernel -- TEST INFRASTRUCTURE ONLY.

The reference samples the next token of a rollout with ``torch.multinomial`` over
``exp(log_softmax(logits / T))`` (engine/base.py:180-193), or takes the argmax when greedy.
The device kernel draws from the same distribution by the Gumbel-max rule,

    token = argmax_v  x_v / T + G_v,   G_v = -log(-log(U_v)),

with the uniforms U_v taken from a Philox4x32-10 stream (Salmon, Moraes, Dror, Shaw,
"Parallel random numbers: as easy as 1, 2, 3", SC 2011): key = the 64-bit seed, counter =
(v // 4, row, offset low word, offset high word), word v % 4 of the output block.  This file
restates that stream and the keys in numpy; the Philox rounds are pinned by the paper's
published known-answer vectors (tests/test_sampling_oracle.py).  Only tests may import it.
"""

from __future__ import annotations

import numpy as np

PHILOX_M0, PHILOX_M1 = 0xD2511F53, 0xCD9E8D57   # round multipliers (SC 2011, Philox4x32)
PHILOX_W0, PHILOX_W1 = 0x9E3779B9, 0xBB67AE85   # key schedule increments (golden ratio, sqrt(3)-1)
_U32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(ctr, key):
    """Philox4x32 with 10 rounds.  ``ctr``: uint32 array [..., 4]; ``key``: uint32 array
    [..., 2] (broadcast).  Returns uint32 [..., 4]."""
    c = [np.asarray(ctr[..., i], dtype=np.uint64) for i in range(4)]
    k0 = np.asarray(key[..., 0], dtype=np.uint64)
    k1 = np.asarray(key[..., 1], dtype=np.uint64)
    for r in range(10):
        if r:
            k0 = (k0 + np.uint64(PHILOX_W0)) & _U32
            k1 = (k1 + np.uint64(PHILOX_W1)) & _U32
        p0 = np.uint64(PHILOX_M0) * c[0]
        p1 = np.uint64(PHILOX_M1) * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & _U32
        hi1, lo1 = p1 >> np.uint64(32), p1 & _U32
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
    return np.stack(c, axis=-1).astype(np.uint32)


def uniforms(row: int, vocab: int, seed: int, offset: int) -> np.ndarray:
    """U_v of one row, float32 in [2^-24, 1 - 2^-24]: ((bits >> 9) + 0.5) * 2^-23."""
    n = (vocab + 3) // 4
    ctr = np.zeros((n, 4), dtype=np.uint32)
    ctr[:, 0] = np.arange(n, dtype=np.uint32)
    ctr[:, 1] = row
    ctr[:, 2] = offset & 0xFFFFFFFF
    ctr[:, 3] = (offset >> 32) & 0xFFFFFFFF
    key = np.array([seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF], dtype=np.uint32)
    bits = philox4x32_10(ctr, key).reshape(-1)[:vocab]
    return (((bits >> 9).astype(np.float32) + np.float32(0.5)) * np.float32(2.0 ** -23)).astype(np.float32)


def sample(logits: np.ndarray, temperature: float, greedy: bool, seed: int, offset: int):
    """(tokens, logp, keys) of each row of ``logits`` [rows, vocab], in float64: the token, its
    log_softmax(x / T) value and the Gumbel keys the argmax ran over (for tie analysis)."""
    x = np.asarray(logits, dtype=np.float64)
    rows, vocab = x.shape
    z = x / temperature
    m = z.max(axis=1, keepdims=True)
    lse = (m + np.log(np.exp(z - m).sum(axis=1, keepdims=True)))[:, 0]
    if greedy:
        keys = x
    else:
        g = np.stack([-np.log(-np.log(uniforms(r, vocab, seed, offset).astype(np.float64))) for r in range(rows)])
        keys = z + g
    tok = keys.argmax(axis=1)
    return tok.astype(np.int64), z[np.arange(rows), tok] - lse, keys
