"""Binary rollout files: lossless round trip of engine rollouts (token streams, loss masks,
log-probs, compaction events, segments, stats) and, on the GPU, the replay batch built from
a file equals the one collated from the rollouts."""

import json

import numpy as np
import pytest
import torch

from kvstreams.chat import CharTokenizer
from kvstreams.compaction.policies import build_policy
from kvstreams.config import CacheConfig, RolloutConfig, SamplingConfig
from kvstreams.engine import KVStreamEngine
from kvstreams.envs import build_env
from kvstreams.logfmt import read_replay_batch, read_rollouts, write_rollouts

from test_host_logic import _ConstantModel, _OracleBackedCache


def _rollouts():
    """Teacher-forced rollouts with compactions, on the oracle-backed cache double (CPU)."""
    tok = CharTokenizer()
    out = []
    for bs, policy, kw in [(16, "keep_recent", {"keep_last": 2}), (8, "markovian", {"keep_last": 1})]:
        cache = _OracleBackedCache(bs, 1024)
        eng = KVStreamEngine(_ConstantModel(tok.vocab_size), tok, build_policy(policy, **kw),
                             CacheConfig(block_size=bs, num_blocks=1024, pad_to_block=True),
                             RolloutConfig(context_budget=160), SamplingConfig(max_new_tokens=12), cache=cache)
        for i in range(2):
            r = eng.rollout(build_env("recall", seed=i, num_distractors=6), teacher_forcing=True)
            rng = np.random.default_rng(i)
            r.inf_logprobs = (-rng.random(len(r.tokens)) * np.asarray(r.loss_mask)).tolist()
            out.append(r)
    return out


def test_roundtrip_lossless_f64(tmp_path):
    rolls = _rollouts()
    assert sum(len(r.log) for r in rolls) > 0
    p = tmp_path / "r.kvsr"
    size = write_rollouts(p, rolls, logprob_dtype=np.float64)
    back = read_rollouts(p)
    assert [r.to_dict() for r in back] == [r.to_dict() for r in rolls]
    assert size < len(json.dumps([r.to_dict() for r in rolls]))


def test_roundtrip_f32_logprobs(tmp_path):
    rolls = _rollouts()
    p = tmp_path / "r.kvsr"
    write_rollouts(p, rolls)
    back = read_rollouts(p)
    for a, b in zip(rolls, back):
        assert a.tokens == b.tokens and a.loss_mask == b.loss_mask
        assert [e.to_dict() for e in a.log] == [e.to_dict() for e in b.log]
        np.testing.assert_allclose(b.inf_logprobs, a.inf_logprobs, rtol=1e-7, atol=0)


def test_empty_and_bad_files(tmp_path):
    p = tmp_path / "e.kvsr"
    write_rollouts(p, [])
    assert read_rollouts(p) == []
    (tmp_path / "bad").write_bytes(b"not a rollout file at all........................................")
    with pytest.raises(ValueError):
        read_rollouts(tmp_path / "bad")


@pytest.mark.gpu
def test_replay_batch_from_file_equals_collate(tmp_path):
    from kvstreams.training.replay import build_sequences, collate

    rolls = _rollouts()
    p = tmp_path / "r.kvsr"
    write_rollouts(p, rolls, logprob_dtype=np.float64)
    got = read_replay_batch(p, device="cuda")
    want = collate([build_sequences(r)[0] for r in rolls], device="cuda")
    for f in ("tokens", "positions", "loss_mask", "inf_logprobs", "lengths", "evicted_at"):
        a, b = getattr(got, f), getattr(want, f)
        assert torch.equal(a.cpu(), b.cpu()), f
