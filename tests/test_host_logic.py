"""Host-side logic that needs no GPU: spans, policies, compaction log, tokenizer, chat,
envs, and the rollout loop driven with an oracle-backed cache double and a constant
model -- under teacher forcing the token stream and the compaction decisions do not
depend on the model, so they must equal the reference's golden rollouts."""

import json

import numpy as np
import pytest
import torch

from kvstreams.compaction import CompactionEvent, CompactionLog, build_policy
from kvstreams.compaction.segments import Segment
from kvstreams.config import CacheConfig, ModelConfig, RolloutConfig, SamplingConfig
from kvstreams.engine import KVStreamEngine
from kvstreams.envs import build_env
from kvstreams.tokenizer import CharTokenizer
from kvstreams.utils.spans import merge_spans, positions_to_spans
from oracle import kvs_oracle as O


def test_spans_match_oracle():
    rng = np.random.default_rng(0)
    for _ in range(200):
        spans = [(int(a), int(a + rng.integers(-2, 9))) for a in rng.integers(0, 50, rng.integers(0, 8))]
        assert merge_spans(spans) == O.merge_spans(spans)
        pos = sorted(set(rng.integers(0, 60, rng.integers(0, 20)).tolist()))
        assert positions_to_spans(pos) == O.positions_to_spans(pos)


def test_policies_pick_oldest_turns():
    segs = [Segment(0, "prompt", 0, 48, protected=True)] + [Segment(i, "turn", 48 * i, 48 * (i + 1)) for i in range(1, 6)]
    p = build_policy("keep_recent", keep_last=2).plan(segs, 288, 256, 300)
    assert p.spans == [(48, 96)] and p.segments == [1]
    p = build_policy("markovian", keep_last=1).plan(segs, 288, 256, 300)
    assert p.spans == [(48, 240)]
    with pytest.raises(ValueError):
        build_policy("keep_recent", keep_last=0)


def test_log_json_roundtrip():
    log = CompactionLog([CompactionEvent(10, [(0, 4)], [(0, 5)]), CompactionEvent(20, [(6, 8), (9, 12)])])
    log2 = CompactionLog.from_json(log.to_json())
    assert [e.evicted for e in log2] == [e.evicted for e in log]
    np.testing.assert_array_equal(log2.span_triples(), log.span_triples())
    with pytest.raises(ValueError):
        log.append(CompactionEvent(5, []))


def test_tokenizer_and_template():
    tok = CharTokenizer()
    assert tok.vocab_size == 104
    assert tok.decode(tok.encode("hello, world\n")) == "hello, world\n"
    assert tok.encode("é") == [tok.unk_id]


class _OracleBackedCache:
    """Test double with the PagedKVCache host interface, state kept by the oracle."""

    def __init__(self, bs, nb):
        self.c = O.OracleCache(nb, bs)

    def add_sequence(self, s):
        self.c.add_sequence(s)

    def free_sequence(self, s):
        self.c.free_sequence(s)

    def num_tokens(self, s):
        return self.c.lengths[s]

    def append(self, s, positions):
        self.c.append_slots(s, positions)

    def evict_positions(self, s, spans, check=False):
        evicted = self.c.evict_positions(s, spans)
        if check:
            self.check_invariants(s)
        return evicted

    def check_invariants(self, s):
        msg = self.c.check_invariants(s)
        if msg:
            raise AssertionError(msg)

    def truncate(self, s, n):
        self.c.truncate(s, n)


class _ConstantModel:
    """Uniform logits; forward_cached records the appends in the cache double."""

    def __init__(self, vocab):
        self.cfg = ModelConfig(vocab_size=vocab)
        self.device = torch.device("cpu")
        self.dtype = torch.float64
        self.training = False

    def eval(self):
        return self

    def train(self, mode=True):
        return self

    def forward_cached(self, toks, pos, cache, seq_id):
        cache.append(seq_id, pos.tolist())
        return torch.zeros(toks.numel(), self.cfg.vocab_size, dtype=torch.float64)


ENGINE_CASES = [
    # tag, engine, block size, pad to block, commit partial blocks, policy, policy kwargs
    ("f64_bs16", "kvstream", 16, True, True, "keep_recent", {"keep_last": 2}),
    ("f64_bs1", "kvstream", 1, False, True, "keep_recent", {"keep_last": 2}),
    ("f64_bs8_markov", "kvstream", 8, True, True, "markovian", {"keep_last": 1}),
    ("f64_reprefill_bs16", "reprefill", 16, True, True, "keep_recent", {"keep_last": 2}),
    ("f64_reprefill_bs4_recompute", "reprefill", 4, False, False, "keep_recent", {"keep_last": 1}),
    ("f64_bs16_recompute", "kvstream", 16, False, False, "keep_recent", {"keep_last": 2}),
    ("f64_bs8_summary", "kvstream", 8, True, True, "summary", {"keep_last": 1}),
]


@pytest.mark.parametrize("tag,engine,bs,pad,commit,policy,kw", ENGINE_CASES)
def test_teacher_forced_stream_and_events_match_reference(golden_rollouts, tag, engine, bs, pad, commit, policy, kw):
    """Token streams, loss masks, compaction events, stats, segments and completions of the
    rollout loop (both engines, padded / unpadded, committed / recomputed partial blocks, three
    policies) equal the reference's, with the model replaced by uniform logits."""
    from kvstreams.engine import build_engine

    arrays, meta = golden_rollouts
    tok = CharTokenizer()
    cache = _OracleBackedCache(bs, 1024)
    eng = build_engine(engine, _ConstantModel(tok.vocab_size), tok, build_policy(policy, **kw),
                       CacheConfig(block_size=bs, num_blocks=1024, pad_to_block=pad, commit_partial_blocks=commit),
                       RolloutConfig(context_budget=160), SamplingConfig(max_new_tokens=12), cache=cache)
    for i in range(2):
        r = eng.rollout(build_env("recall", seed=i, num_distractors=6), teacher_forcing=True)
        key = f"{tag}_{i}"
        assert r.tokens == arrays[key + "_tokens"].tolist()
        assert r.loss_mask == arrays[key + "_loss"].tolist()
        want = meta[key]["events"]
        assert [e.to_dict() for e in r.log] == want
        got_stats = r.stats.to_dict()
        for name, value in meta[key]["stats"].items():
            if name != "wall_time":
                assert got_stats[name] == value, (name, got_stats[name], value)
        assert [s.to_dict() for s in r.segments] == meta[key]["segments"]
        assert r.completions == meta[key]["completions"]
