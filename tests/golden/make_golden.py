"""Generate golden fixtures by running the reference implementation itself.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py [--ref /root/reference]

Imports the reference package ``kvstreams`` from the reference checkout (read
only) in a process of its own and records, for seeded inputs:

* cache_traces.json.gz -- op traces on the reference PagedKVCache (bs 4 / 16 / 8 / 1)
  with the full metadata state after every op (tables, lengths, free list, stats,
  a digest of slot_pos, return values, raised exception types);
* evicted_at.npz       -- CompactionLog.evicted_at for random logs;
* rope.npz             -- RotaryEmbedding + apply_rope outputs (fp32 and fp64);
* tinylm.npz           -- TinyLM.forward logits for a small fp64 model under a
                          KV-streams mask (state dict included);
* rollouts.npz/json    -- teacher-forced KV-streams rollouts (fp64 test model and
                          the fp32 default model at the repo's CPU bench config),
                          with their inference and replay log-probs;
* policy_plans.json    -- CompactionPolicy.plan (keep_recent, markovian, summary,
                          token_window) on random segment lists: spans and segments.

The fixtures are committed; this script is only needed to regenerate them.
"""

from __future__ import annotations

import argparse
import gzip
import json
import random
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _snapshot(cache, res, err):
    import hashlib

    return {
        "result": res,
        "error": err,
        "tables": {str(k): list(v) for k, v in sorted(cache._tables.items())},
        "lengths": {str(k): int(v) for k, v in sorted(cache._lengths.items())},
        "free": list(cache.allocator._free),
        "stats": [cache.stats.written_tokens, cache.stats.evicted_tokens, cache.stats.evicted_blocks,
                  cache.stats.truncated_tokens, cache.stats.peak_blocks, cache.stats.eviction_calls,
                  cache.stats.shrunk_tokens],
        "slot_pos_hash": hashlib.sha256(cache.slot_pos.numpy().astype(np.int64).tobytes()).hexdigest()[:24],
    }


def _run_op(cache, op):
    import torch

    from kvstreams.paged_cache import OutOfBlocksError

    kind = op[0]
    res, err = None, None
    try:
        if kind == "add":
            cache.add_sequence(op[1])
        elif kind == "append":
            cache.append_slots(op[1], torch.tensor(op[2], dtype=torch.long))
        elif kind == "evict_positions":
            res = [list(s) for s in cache.evict_positions(op[1], [tuple(s) for s in op[2]])]
        elif kind == "evict_blocks":
            res = cache.evict_blocks(op[1], op[2])
        elif kind == "truncate":
            cache.truncate(op[1], op[2])
        elif kind == "free":
            cache.free_sequence(op[1])
    except (ValueError, OutOfBlocksError) as exc:
        err = type(exc).__name__
    return res, err


def random_trace(seed: int, num_blocks: int, bs: int, n_ops: int, max_seqs: int = 4):
    """Seeded op trace in the style of the engines: turns appended with increasing logical
    positions, whole-turn and unaligned evictions, truncation of partial tails, frees."""
    import torch

    from kvstreams.paged_cache import PagedKVCache

    rng = random.Random(seed)
    cache = PagedKVCache(1, 1, 2, block_size=bs, num_blocks=num_blocks, dtype=torch.float64)
    next_pos: dict[int, int] = {}
    turns: dict[int, list] = {}
    ops, obs = [], []
    next_id = 0

    def record(op):
        res, err = _run_op(cache, op)
        ops.append(op)
        obs.append(_snapshot(cache, res, err))
        return res, err

    for _ in range(n_ops):
        live = list(next_pos)
        r = rng.random()
        if not live or (r < 0.08 and len(live) < max_seqs):
            sid = next_id
            next_id += 1
            record(["add", sid])
            next_pos[sid] = 0
            turns[sid] = []
            continue
        sid = rng.choice(live)
        if r < 0.55:
            n = max(1, int(rng.expovariate(1 / 24)))
            if rng.random() < 0.5:  # pad the turn to the block size like pad_to_block
                n += (-(next_pos[sid] + n)) % bs
            gap = rng.choice([0, 0, 0, rng.randint(1, 5)])  # re-prefill style renumbering gaps
            start = next_pos[sid] + gap
            pos = list(range(start, start + n))
            _, err = record(["append", sid, pos])
            if err is None:
                turns[sid].append((start, start + n))
                next_pos[sid] = start + n
        elif r < 0.80:
            ts = turns[sid]
            if not ts:
                continue
            k = rng.randint(1, max(1, len(ts) - 1))
            picked = rng.sample(ts[:-1] or ts, min(k, len(ts[:-1] or ts)))
            spans = [list(s) for s in picked]
            if rng.random() < 0.3:  # unaligned request, shrunk to whole blocks
                a, b = spans[0]
                spans[0] = [a + rng.randint(0, 3), b + rng.randint(-3, 3)]
            record(["evict_positions", sid, spans])
        elif r < 0.86:
            n = cache.num_tokens(sid)
            nfull = n // bs
            idxs = rng.sample(range(nfull), min(nfull, rng.randint(0, 3))) if nfull else []
            if rng.random() < 0.15:
                idxs = idxs + [nfull + rng.randint(0, 2)]  # invalid: not a full block
            record(["evict_blocks", sid, idxs])
        elif r < 0.93:
            n = cache.num_tokens(sid)
            t = rng.randint(0, max(0, min(n, bs + 2)))
            if rng.random() < 0.1:
                t = n + 1  # invalid: more than live
            _, err = record(["truncate", sid, t])
            if err is None and t > 0:
                next_pos[sid] = next_pos[sid] - t if t <= next_pos[sid] else 0
                turns[sid] = [(a, min(b, next_pos[sid])) for a, b in turns[sid] if a < next_pos[sid]]
        else:
            record(["free", sid])
            next_pos.pop(sid)
            turns.pop(sid)
    return {"num_blocks": num_blocks, "block_size": bs, "ops": ops, "obs": obs}


def scripted_trace():
    """The reference's own cache test scenarios (tests/test_paged_cache.py:34-104) as one trace."""
    import torch

    from kvstreams.paged_cache import PagedKVCache

    cache = PagedKVCache(1, 1, 2, block_size=4, num_blocks=16, dtype=torch.float64)
    ops = [
        ["add", 0], ["append", 0, list(range(14))], ["evict_blocks", 0, [1]],
        ["append", 0, [14, 15]], ["evict_positions", 0, [[2, 12]]],
        ["add", 1], ["append", 1, list(range(6))], ["evict_blocks", 1, [1]],
        ["truncate", 1, 2], ["append", 1, [4, 5]], ["truncate", 1, 7],
        ["add", 2], ["append", 2, list(range(8))], ["evict_positions", 2, [[0, 4]]],
        ["append", 2, [8, 9]], ["free", 1], ["add", 1], ["free", 0], ["free", 2],
        ["add", 3], ["append", 3, list(range(64))], ["append", 3, [64]], ["free", 3],
    ]
    obs = []
    for op in ops:
        res, err = _run_op(cache, op)
        obs.append(_snapshot(cache, res, err))
    return {"num_blocks": 16, "block_size": 4, "ops": ops, "obs": obs}


def make_traces():
    traces = {"scripted_bs4": scripted_trace()}
    traces["random_bs16"] = random_trace(1, 256, 16, 160)
    traces["random_bs8"] = random_trace(2, 160, 8, 160)
    traces["random_bs1"] = random_trace(3, 600, 1, 160)
    traces["random_bs16_tight"] = random_trace(4, 24, 16, 120)  # pool exhaustion
    with gzip.open(HERE / "cache_traces.json.gz", "wt") as f:
        json.dump(traces, f, separators=(",", ":"))


def make_evicted_at():
    import torch

    from kvstreams.compaction.events import CompactionEvent, CompactionLog

    rng = random.Random(7)
    cases = {}
    for i in range(12):
        T = rng.choice([1, 7, 64, 300, 1000])
        events = []
        t = 0
        for _ in range(rng.randint(0, 6)):
            t += rng.randint(0, T // 2 + 1)
            spans = []
            for _ in range(rng.randint(0, 3)):
                a = rng.randint(0, T + 10)
                spans.append((a, a + rng.randint(0, T // 3 + 2)))
            events.append(CompactionEvent(time=t, evicted=spans))
        log = CompactionLog(events)
        trip = np.asarray([(s, e, ev.time) for ev in events for s, e in ev.evicted], dtype=np.int64).reshape(-1, 3)
        cases[f"c{i}_triples"] = trip
        cases[f"c{i}_len"] = np.asarray([T])
        cases[f"c{i}_out"] = log.evicted_at(T).numpy()
    np.savez_compressed(HERE / "evicted_at.npz", **cases)


def make_rope():
    import torch

    from kvstreams.rope import RotaryEmbedding, apply_rope

    g = torch.Generator().manual_seed(11)
    out = {}
    for D, theta in ((16, 1e4), (128, 5e5)):
        pos = torch.tensor([0, 1, 7, 123, 1000, 4097, 65535, 131071, 200003], dtype=torch.long)
        x = torch.randn(pos.numel(), 3, D, generator=g, dtype=torch.float64)
        for name, dt in (("f32", torch.float32), ("f64", torch.float64)):
            rope = RotaryEmbedding(D, theta).to(dt)
            cos, sin = rope(pos)
            y = apply_rope(x.to(dt), cos, sin)
            out[f"D{D}_{name}_x"] = x.to(dt).numpy()
            out[f"D{D}_{name}_y"] = y.numpy()
            out[f"D{D}_{name}_pos"] = pos.numpy()
            out[f"D{D}_{name}_theta"] = np.asarray([theta])
    np.savez_compressed(HERE / "rope.npz", **out)


def make_tinylm():
    import torch

    from kvstreams.config import ModelConfig
    from kvstreams.model import TinyLM, causal_mask

    torch.manual_seed(0)
    model = TinyLM(ModelConfig(vocab_size=104, init_std=0.1)).double()
    g = torch.Generator().manual_seed(5)
    T = 40
    tokens = torch.randint(0, 104, (T,), generator=g)
    mask = causal_mask(T).clone()
    mask[24:, 4:12] = False  # KV-streams mask: keys 4..11 evicted at time 24
    mask[32:, 16:20] = False
    with torch.no_grad():
        logits = model(tokens[None], torch.arange(T)[None], mask[None])[0]
    sd = {f"p::{k}": v.numpy() for k, v in model.state_dict().items()}
    np.savez_compressed(HERE / "tinylm.npz", tokens=tokens.numpy(), mask=mask.numpy(), logits=logits.numpy(),
                        **sd)


def make_rollouts():
    import torch

    from kvstreams.compaction import build_policy
    from kvstreams.config import CacheConfig, ModelConfig, RolloutConfig, SamplingConfig
    from kvstreams.engine import build_engine
    from kvstreams.envs import build_env
    from kvstreams.factory import build_stack
    from kvstreams.model import TinyLM
    from kvstreams.tokenizer import CharTokenizer
    from kvstreams.training import build_sequences, collate, token_logprobs

    tok = CharTokenizer()
    arrays, meta = {}, {}

    def dump(tag, model, rollouts, mode="kvstream"):
        for i, r in enumerate(rollouts):
            key = f"{tag}_{i}"
            arrays[key + "_tokens"] = np.asarray(r.tokens, dtype=np.int64)
            arrays[key + "_loss"] = np.asarray(r.loss_mask, dtype=bool)
            arrays[key + "_inf"] = np.asarray(r.inf_logprobs, dtype=np.float64)
            arrays[key + "_evicted_at"] = r.log.evicted_at(r.length).numpy()
            if mode == "kvstream":
                seq = build_sequences(r, "kvstream")[0]
                batch = collate([seq])
                with torch.no_grad():
                    lp = token_logprobs(model, batch, r.temperature)[0]
                arrays[key + "_replay"] = lp.double().numpy()
            meta[key] = {"events": [e.to_dict() for e in r.log], "stats": r.stats.to_dict(), "reward": r.reward,
                         "completions": r.completions, "segments": [s.to_dict() for s in r.segments]}

    # fp64 test model (tests/conftest.py:16-19) with the reference's engine fixture settings.
    torch.manual_seed(0)
    m64 = TinyLM(ModelConfig(vocab_size=tok.vocab_size, init_std=0.1)).double()
    for tag, bs, pad, commit, policy, kw in (
        ("f64_bs16", 16, True, True, "keep_recent", {"keep_last": 2}),
        ("f64_bs1", 1, False, True, "keep_recent", {"keep_last": 2}),
        ("f64_bs8_markov", 8, True, True, "markovian", {"keep_last": 1}),
    ):
        eng = build_engine("kvstream", m64, tok, build_policy(policy, **kw),
                           CacheConfig(block_size=bs, num_blocks=1024, pad_to_block=pad, commit_partial_blocks=commit),
                           RolloutConfig(context_budget=160), SamplingConfig(max_new_tokens=12))
        rs = [eng.rollout(build_env("recall", seed=i, num_distractors=6), teacher_forcing=True) for i in range(2)]
        dump(tag, m64, rs)
    # the other engine paths: re-prefill, uncommitted partial blocks recomputed, summary turns
    for tag, engine, bs, pad, commit, policy, kw in (
        ("f64_reprefill_bs16", "reprefill", 16, True, True, "keep_recent", {"keep_last": 2}),
        ("f64_reprefill_bs4_recompute", "reprefill", 4, False, False, "keep_recent", {"keep_last": 1}),
        ("f64_bs16_recompute", "kvstream", 16, False, False, "keep_recent", {"keep_last": 2}),
        ("f64_bs8_summary", "kvstream", 8, True, True, "summary", {"keep_last": 1}),
    ):
        eng = build_engine(engine, m64, tok, build_policy(policy, **kw),
                           CacheConfig(block_size=bs, num_blocks=1024, pad_to_block=pad, commit_partial_blocks=commit),
                           RolloutConfig(context_budget=160), SamplingConfig(max_new_tokens=12))
        rs = [eng.rollout(build_env("recall", seed=i, num_distractors=6), teacher_forcing=True) for i in range(2)]
        dump(tag, m64, rs, mode="auto")
    arrays.update({f"m64::{k}": v.numpy() for k, v in m64.state_dict().items()})

    # fp32 default model at the repo's CPU bench config (keep_recent 2, bs 16 padded, budget 256).
    st = build_stack(policy="keep_recent", policy_kwargs={"keep_last": 2},
                     cache_cfg=CacheConfig(16, pad_to_block=True),
                     rollout_cfg=RolloutConfig(context_budget=256, max_turns=128), dtype="float32", seed=0)
    rs = [st.engine.rollout(build_env("recall", seed=0, num_distractors=24, filler_len=64), teacher_forcing=True)]
    dump("f32_c1", st.model, rs)
    # the same episode through the re-prefill engine (the comparison arm of this configuration)
    rp = build_stack(engine="reprefill", policy="keep_recent", policy_kwargs={"keep_last": 2},
                     cache_cfg=CacheConfig(16, pad_to_block=True),
                     rollout_cfg=RolloutConfig(context_budget=256, max_turns=128), model=st.model,
                     dtype="float32", seed=0)
    rs = [rp.engine.rollout(build_env("recall", seed=0, num_distractors=24, filler_len=64), teacher_forcing=True)]
    dump("f32_c1_reprefill", st.model, rs, mode="auto")
    arrays.update({f"m32::{k}": v.numpy() for k, v in st.model.state_dict().items()})
    np.savez_compressed(HERE / "rollouts.npz", **arrays)
    (HERE / "rollouts.json").write_text(json.dumps(meta))


def make_policies():
    from kvstreams.compaction.policies import build_policy
    from kvstreams.compaction.segments import Segment

    rng = random.Random(11)
    cases = []
    for c in range(400):
        n = rng.randint(1, 40)
        segs, pos = [], 0
        for i in range(n):
            prompt = i == 0 and rng.random() < 0.9
            length = rng.choice([0, 16, 32]) if rng.random() < 0.1 else rng.randint(1, 400)
            seg = Segment(i, "prompt" if prompt else "turn", pos, pos + length, protected=prompt)
            pos += length
            r = rng.random()
            if not prompt and i < n - 1 and r < 0.25:
                seg.evicted_at = pos + rng.randint(0, 500)
            elif not prompt and i < n - 1 and r < 0.35:
                seg.partially_evicted = True
            segs.append(seg)
        live = sum(s.length for s in segs if s.alive) + rng.randint(0, 64)
        incoming, reserve = rng.randint(0, 600), rng.randint(1, 400)
        required = live + incoming + reserve
        budget = rng.randint(max(1, required // 4), required + 200)
        name = ["keep_recent", "markovian", "summary", "token_window"][c % 4]
        param = rng.randint(16, 1024) if name == "token_window" else rng.randint(1, 4)
        pol = build_policy(name, **({"window": param} if name == "token_window" else {"keep_last": param}))
        plan = pol.plan(segs, live, budget, required)
        cases.append({
            "policy": name, "param": param, "live": live, "budget": budget, "required": required,
            "segments": [[s.start, s.end, int(s.protected), int(s.alive), int(s.partially_evicted)] for s in segs],
            "spans": [list(x) for x in plan.spans], "chosen": list(plan.segments),
        })
    (HERE / "policy_plans.json").write_text(json.dumps(cases))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--only", default="", help="comma-separated subset: traces,evicted_at,rope,tinylm,rollouts,policies")
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    import kvstreams  # noqa: F401  (the reference package)

    assert Path(kvstreams.__file__).resolve().is_relative_to(Path(a.ref).resolve()), kvstreams.__file__
    steps = {"traces": make_traces, "evicted_at": make_evicted_at, "rope": make_rope, "tinylm": make_tinylm,
             "rollouts": make_rollouts, "policies": make_policies}
    for name, fn in steps.items():
        if not a.only or name in a.only.split(","):
            fn()
    for p in sorted(HERE.glob("*.*")):
        print(f"{p.name:28s} {p.stat().st_size:>9d} B")


if __name__ == "__main__":
    main()
