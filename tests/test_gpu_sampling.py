"""kvs_sample, the rollout's next-token step (engine/base.py:180-193: log_softmax(logits / T),
multinomial or argmax, the token's log-prob), against torch and the sampling oracle:
greedy tokens equal torch.argmax (first maximum) and log-probs equal log_softmax(x / T) at
them (float32 2e-5, float64 1e-12); sampled tokens equal the oracle's Gumbel-max draws from
the same Philox stream on every row whose two largest keys are more than 1e-3 apart (the
kernel's float Gumbel noise is within ~1e-6 of the oracle's float64); a fixed (seed, offset)
repeats, a new offset redraws, and the frequencies follow softmax(x / T)."""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _logits(n, vocab, dtype, seed, scale=4.0, ld=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    full = torch.randn(n, ld or vocab, generator=g, device="cuda", dtype=torch.float64) * scale
    return full.to(dtype)[:, :vocab]


@pytest.mark.parametrize("dtype,n,vocab,temp,tol,ld", [
    (torch.float32, 64, 128256, 1.0, 2e-5, None),
    (torch.float32, 37, 1001, 0.7, 2e-5, None),      # rows not 16-byte aligned: scalar loads
    (torch.float32, 9, 4000, 1.0, 2e-5, 4099),       # a column slice of wider rows
    (torch.float64, 20, 1003, 1.3, 1e-12, None),
])
def test_greedy_matches_torch(dtype, n, vocab, temp, tol, ld):
    from kvstreams import ops

    x = _logits(n, vocab, dtype, vocab, ld=ld)
    top = x[0].max().item() + 1.0
    x[0, 5] = top
    x[0, vocab - 3] = top                            # a tie: the first maximum wins
    tok, lp = ops.sample(x, temp, greedy=True)
    assert tok[0].item() == 5
    assert torch.equal(tok, x.argmax(-1))
    ref = torch.log_softmax(x.double() / temp, dim=-1).gather(-1, tok[:, None]).squeeze(-1)
    assert (lp.double() - ref).abs().max().item() <= tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_sampled_tokens_match_oracle(dtype):
    from kvstreams import ops
    from oracle import sampling as S

    n, vocab, temp = 48, 5003, 0.8
    seed, offset = 0xDEADBEEF12345, (3 << 32) | 17
    x = _logits(n, vocab, dtype, 11, scale=3.0)
    tok, lp = ops.sample(x, temp, False, seed, offset)
    otok, _, keys = S.sample(x.cpu().double().numpy(), temp, False, seed, offset)
    top2 = np.sort(keys, axis=1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 1e-3
    assert clear.sum() >= 0.9 * n
    assert np.array_equal(tok.cpu().numpy()[clear], otok[clear])
    ref = torch.log_softmax(x.double() / temp, dim=-1).gather(-1, tok[:, None]).squeeze(-1)
    assert (lp.double() - ref).abs().max().item() <= (2e-5 if dtype == torch.float32 else 1e-12)
    again, lp2 = ops.sample(x, temp, False, seed, offset)
    assert torch.equal(again, tok) and torch.equal(lp2, lp)
    other, _ = ops.sample(x, temp, False, seed, offset + 1)
    assert (other != tok).sum().item() >= n // 2


def test_sampled_frequencies_follow_softmax():
    from kvstreams import ops

    base = torch.tensor([1.0, 0.0, -0.5, 2.0, 0.3, -2.0, 0.7, 1.5, -1.0, 0.1, 0.9, -0.2, 0.4, 1.1, -3.0, 0.0],
                        device="cuda")
    temp, rows = 0.9, 1 << 16
    tok, _ = ops.sample(base.expand(rows, -1).contiguous(), temp, False, seed=7, offset=0)
    p = torch.softmax(base.double() / temp, -1).cpu().numpy()
    counts = np.bincount(tok.cpu().numpy(), minlength=16)
    chi2 = float((((counts - rows * p) ** 2) / (rows * p)).sum())
    assert chi2 < 60.0, (counts, rows * p)   # 15 degrees of freedom: p-value ~1e-7 at 60


def test_masked_entries_and_empty_rows():
    from kvstreams import ops

    x = _logits(6, 300, torch.float32, 3)
    x[:, ::2] = -math.inf                    # masked vocabulary entries are never drawn
    x[4] = -math.inf                         # a row with nothing to draw
    for greedy in (True, False):
        tok, lp = ops.sample(x, 1.0, greedy, seed=1, offset=2)
        t = tok.cpu().tolist()
        assert t[4] == -1 and math.isnan(lp[4].item())
        assert all(v % 2 == 1 for i, v in enumerate(t) if i != 4)
        keep = [0, 1, 2, 3, 5]
        ref = torch.log_softmax(x[keep].double(), -1).gather(-1, tok[keep][:, None]).squeeze(-1)
        assert (lp[keep].double() - ref).abs().max().item() <= 2e-5
