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


def test_plan_kernel_many_sequences_matches_oracle():
    """More sequences than one round of the plan kernel's block scan (1024): random tables
    against the oracle's single-pass restatement, cu_spans carried across rounds."""
    import random

    from kvstreams import _native as N
    from oracle.compaction_plan import plan_table

    rng = random.Random(7)
    S, M = 1500, 24
    tabs, lives, needs = [], [], []
    for _ in range(S):
        n = rng.randint(1, M)
        segs, pos = [], 0
        for j in range(n):
            ln = rng.randint(0, 300)
            prot = int(j == 0)
            r = rng.random()
            alive, part = (0, 0) if (not prot and r < 0.2) else (1, int(not prot and r < 0.3))
            segs.append([pos, pos + ln, prot, alive, part])
            pos += ln
        tabs.append(segs)
        lives.append(rng.randint(0, 4000))
        needs.append(rng.randint(-500, 3000))
    lib = N.lib()
    for policy, param in (("keep_recent", 2), ("token_window", 200)):
        t = {k: torch.zeros(S, M, dtype=torch.int32) for k in ("start", "end", "flags")}
        t["evicted_at"] = torch.full((S, M), -1, dtype=torch.int32)
        count = torch.tensor([len(x) for x in tabs], dtype=torch.int32)
        for i, segs in enumerate(tabs):
            for j, (s, e, prot, alive, part) in enumerate(segs):
                t["start"][i, j], t["end"][i, j] = s, e
                t["flags"][i, j] = prot | (2 * part)
                t["evicted_at"][i, j] = -1 if alive else e
        d = {k: v.cuda() for k, v in t.items()}
        cnt, live, need = count.cuda(), torch.tensor(lives, dtype=torch.int32).cuda(), \
            torch.tensor(needs, dtype=torch.int32).cuda()
        seg = N.KvsSegments(start=d["start"].data_ptr(), end=d["end"].data_ptr(), evicted_at=d["evicted_at"].data_ptr(),
                            flags=d["flags"].data_ptr(), count=cnt.data_ptr(), max_seqs=S, max_segs=M)
        order = torch.randperm(S, generator=torch.Generator().manual_seed(1)).to(torch.int32)  # any slot order
        slots = order.cuda()
        b = N.KvsBatch(seq_slots=slots.data_ptr(), cu_tokens=None, num_seqs=S, total_tokens=S)
        out = {k: torch.zeros(S, M, 2, dtype=torch.long, device="cuda") for k in ("spans",)}
        ns, ch, nc = (torch.zeros(S, dtype=torch.int32, device="cuda"), torch.zeros(S, M, dtype=torch.int32, device="cuda"),
                      torch.zeros(S, dtype=torch.int32, device="cuda"))
        cu = torch.zeros(S + 1, dtype=torch.int32, device="cuda")
        ss, se = torch.zeros(S * M, dtype=torch.long, device="cuda"), torch.zeros(S * M, dtype=torch.long, device="cuda")
        # live / need are indexed by batch position
        live_b, need_b = live[slots.long()].contiguous(), need[slots.long()].contiguous()
        N.check(lib.kvs_compact_plan(C.byref(seg), C.byref(b), N.POLICY_CODES[policy], param, 1000,
                                     live_b.data_ptr(), need_b.data_ptr(), out["spans"].data_ptr(), ns.data_ptr(),
                                     ch.data_ptr(), nc.data_ptr(), cu.data_ptr(), ss.data_ptr(), se.data_ptr(),
                                     N.stream_ptr()), "kvs_compact_plan")
        sp_h, ns_h, cu_h, ss_h, se_h = out["spans"].cpu(), ns.cpu(), cu.cpu(), ss.cpu(), se.cpu()
        ch_h, nc_h = ch.cpu(), nc.cpu()
        assert int(cu_h[0]) == 0
        for i in range(S):
            slot = int(order[i])
            required = lives[slot] + needs[slot]
            want_sp, want_ch = plan_table(policy, param, tabs[slot], lives[slot], 1000, required) \
                if required > 1000 else ([], [])
            assert sp_h[i, : int(ns_h[i])].tolist() == want_sp, (policy, i)
            assert ch_h[i, : int(nc_h[i])].tolist() == want_ch, (policy, i)
            assert int(cu_h[i + 1]) - int(cu_h[i]) == len(want_sp)
            flat = list(zip(ss_h[int(cu_h[i]):int(cu_h[i + 1])].tolist(), se_h[int(cu_h[i]):int(cu_h[i + 1])].tolist()))
            assert [list(x) for x in flat] == want_sp


def test_event_log_capacity_is_reported():
    """A compaction whose event does not fit the slot's log raises (status LOG_CAPACITY)
    when the results are read, instead of dropping the event silently."""
    from kvstreams.compaction.device import DeviceCompaction
    from kvstreams.compaction.policies import MarkovianPolicy
    from kvstreams.compaction.segments import Segment
    from kvstreams.paged_cache import PagedKVCache

    cache = PagedKVCache(1, 1, 2, block_size=16, num_blocks=256, dtype=torch.bfloat16, device="cuda", max_seqs=2)
    cache.add_sequence(0)
    cache.append_slots_batch([0], torch.arange(640, dtype=torch.long), [640])
    dc = DeviceCompaction(cache, MarkovianPolicy(keep_last=1), budget=100, max_events=1)
    slot = cache.slot(0)
    dc.reset_slot(slot)
    segs = [Segment(0, "prompt", 0, 64, protected=True)] + [Segment(i, "turn", 64 + 96 * (i - 1), 64 + 96 * i)
                                                           for i in range(1, 7)]
    for s in segs[:4]:
        dc.add_segment(slot, s)
    dc.compact([slot], [0], [50], [640])  # evicts turns 1-2: first event
    for s in segs[4:]:
        dc.add_segment(slot, s)
    dc.compact([slot], [0], [50], [640])  # evicts turns 3-5: no room for a second event
    with pytest.raises(RuntimeError, match="compaction log"):
        dc.read([slot])


def test_stale_mirror_refreshes_instead_of_raising():
    """After a device-side eviction the host mirror overstates the live blocks; an append
    that only fits thanks to the eviction must go through (the check re-reads the device)."""
    from kvstreams.compaction.device import DeviceCompaction
    from kvstreams.compaction.policies import MarkovianPolicy
    from kvstreams.compaction.segments import Segment
    from kvstreams.paged_cache import PagedKVCache

    cache = PagedKVCache(1, 1, 2, block_size=16, num_blocks=40, dtype=torch.bfloat16, device="cuda", max_seqs=1)
    cache.add_sequence(0)
    cache.append_slots_batch([0], torch.arange(576, dtype=torch.long), [576])  # 36 of 40 blocks
    dc = DeviceCompaction(cache, MarkovianPolicy(keep_last=1), budget=200)
    slot = cache.slot(0)
    dc.reset_slot(slot)
    for s in [Segment(0, "prompt", 0, 64, protected=True), Segment(1, "turn", 64, 320), Segment(2, "turn", 320, 576)]:
        dc.add_segment(slot, s)
    dc.compact([slot], [0], [64], [576])  # evicts turn 1: 16 blocks freed on the device only
    cache.append_slots_batch([0], torch.arange(576, 576 + 256, dtype=torch.long), [256])  # needs 16 blocks
    assert cache.num_tokens(0) == 576 - 256 + 256
    d = dc.read([slot])[0]
    assert d["evicted_at"] == [-1, 576, -1] and d["stats"]["compactions"] == 1
