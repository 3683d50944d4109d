"""Device-side compaction (kvs_compact_plan / kvs_compact, compaction/device.py): the plan
kernel against plans recorded from the reference policies (tests/golden/policy_plans.json),
and batched rollouts whose compaction runs on the device against the same rollouts with the
host policy (tokens, log-probs, compaction events, segment marks and stats identical)."""

import ctypes as C
import json
from collections import defaultdict
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).parent / "golden" / "policy_plans.json"


def test_plan_kernel_matches_reference_plans():
    from kvstreams import _native as N

    cases = json.loads(GOLDEN.read_text())
    groups = defaultdict(list)
    for c in cases:
        groups[(c["policy"], c["param"])].append(c)
    M = 64
    lib = N.lib()
    for (policy, param), cs in groups.items():
        S = len(cs)
        t = {k: torch.zeros(S, M, dtype=torch.int32) for k in ("start", "end", "flags")}
        t["evicted_at"] = torch.full((S, M), -1, dtype=torch.int32)
        count = torch.zeros(S, dtype=torch.int32)
        live = torch.zeros(S, dtype=torch.int32)
        need = torch.zeros(S, dtype=torch.int32)
        for i, c in enumerate(cs):
            for j, (s, e, prot, alive, part) in enumerate(c["segments"]):
                t["start"][i, j], t["end"][i, j] = s, e
                t["flags"][i, j] = (1 if prot else 0) | (2 if part else 0)
                t["evicted_at"][i, j] = -1 if alive else e
            count[i] = len(c["segments"])
            # budget 0: required' = required - budget keeps both the trigger and the overflow
            live[i] = c["live"]
            need[i] = c["required"] - c["budget"] - c["live"]
        d = {k: v.cuda() for k, v in t.items()}
        count, live, need = count.cuda(), live.cuda(), need.cuda()
        seg = N.KvsSegments(start=d["start"].data_ptr(), end=d["end"].data_ptr(), evicted_at=d["evicted_at"].data_ptr(),
                            flags=d["flags"].data_ptr(), count=count.data_ptr(), max_seqs=S, max_segs=M)
        slots = torch.arange(S, dtype=torch.int32, device="cuda")
        b = N.KvsBatch(seq_slots=slots.data_ptr(), cu_tokens=None, num_seqs=S, total_tokens=S)
        spans = torch.zeros(S, M, 2, dtype=torch.long, device="cuda")
        n_spans = torch.zeros(S, dtype=torch.int32, device="cuda")
        chosen = torch.zeros(S, M, dtype=torch.int32, device="cuda")
        n_chosen = torch.zeros(S, dtype=torch.int32, device="cuda")
        cu = torch.zeros(S + 1, dtype=torch.int32, device="cuda")
        ss = torch.zeros(S * M, dtype=torch.long, device="cuda")
        se = torch.zeros(S * M, dtype=torch.long, device="cuda")
        rc = lib.kvs_compact_plan(C.byref(seg), C.byref(b), N.POLICY_CODES[policy], param, 0, live.data_ptr(),
                                  need.data_ptr(), spans.data_ptr(), n_spans.data_ptr(), chosen.data_ptr(),
                                  n_chosen.data_ptr(), cu.data_ptr(), ss.data_ptr(), se.data_ptr(), N.stream_ptr())
        N.check(rc, "kvs_compact_plan")
        spans_h, ns, ch, nc, cu_h = spans.cpu(), n_spans.cpu(), chosen.cpu(), n_chosen.cpu(), cu.cpu()
        ss_h, se_h = ss.cpu(), se.cpu()
        for i, c in enumerate(cs):
            # the engine consults the policy only when required > budget (engine/base.py:264-265)
            over = c["required"] > c["budget"]
            want_spans, want_chosen = (c["spans"], c["chosen"]) if over else ([], [])
            got = spans_h[i, : int(ns[i])].tolist()
            assert got == want_spans, (policy, param, i, got, want_spans)
            assert ch[i, : int(nc[i])].tolist() == want_chosen, (policy, param, i)
            flat = list(zip(ss_h[int(cu_h[i]):int(cu_h[i + 1])].tolist(), se_h[int(cu_h[i]):int(cu_h[i + 1])].tolist()))
            assert [list(x) for x in flat] == want_spans


def _engine(cfg, dtype, n, budget, policy, device_policy, num_blocks=4096, seed=0):
    from kvstreams.engine.batched import BatchedKVStreams
    from kvstreams.model import TinyLM
    from kvstreams.paged_cache import PagedKVCache

    torch.manual_seed(seed)
    with torch.device("cuda"):
        model = TinyLM(cfg).to(dtype)
    cache = PagedKVCache(cfg.n_layers, cfg.n_kv_heads, cfg.head_dim, block_size=16, num_blocks=num_blocks,
                         dtype=dtype, max_seqs=n)
    return model, BatchedKVStreams(model, cache, policy, context_budget=budget, seed=seed, device_policy=device_policy)


@pytest.mark.parametrize("policy_name,kw", [("markovian", {"keep_last": 1}), ("keep_recent", {"keep_last": 2}),
                                            ("token_window", {"window": 96})])
def test_device_compaction_rollouts_equal_host(policy_name, kw):
    from kvstreams.compaction.policies import build_policy
    from kvstreams.config import ModelConfig
    from kvstreams.engine.batched import synthetic_episodes

    cfg = ModelConfig()
    eps = synthetic_episodes(8, turns=7, turn_range=(5, 60), prompt_len=10, vocab=cfg.vocab_size, seed=5)
    model, host = _engine(cfg, torch.float32, 8, 200, build_policy(policy_name, **kw), False)
    a = host.run(eps)
    _, dev = _engine(cfg, torch.float32, 8, 200, build_policy(policy_name, **kw), True)
    dev.model = model
    b = dev.run(eps)
    assert sum(len(r.log.events) for r in a) >= 4, "the budget should force compactions"
    for x, y in zip(a, b):
        assert x.tokens == y.tokens
        assert x.inf_logprobs == y.inf_logprobs
        assert [e.to_dict() for e in x.log] == [e.to_dict() for e in y.log]
        assert [(s.start, s.end, s.evicted_at, s.partially_evicted) for s in x.segments] == \
               [(s.start, s.end, s.evicted_at, s.partially_evicted) for s in y.segments]
        for f in ("compactions", "evicted_tokens", "budget_overflows", "peak_live_tokens"):
            assert getattr(x.stats, f) == getattr(y.stats, f), f
