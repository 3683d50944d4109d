"""Benchmark of the KV-streams paged decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (one GPU; weak scaling: every rank runs its own copy, seeded by rank):
paged decode + append, bf16, 32 query / 8 KV heads, head_dim 128, block_size 16,
64 concurrent streams with live context ~U[1024, 16384] drawn from a pool of
131072 blocks (random permutation), 1-6 evicted whole-block spans per stream
(logical positions with gaps), RoPE theta 5e5, Q/K/V ~ N(0, 1).
One step = batched slot allocation + one layer of fused RoPE / K-V append /
split-K paged GQA attention for one new token per stream.  The per-step KV read
(~2.3 GB) is far larger than L2, so no flush is needed between steps.

Also reported (same line, `secondary`): the batched whole-block compaction kernel
on 256 streams x 512-block tables (pool 200000).

`--impl reference` times the reference's own CPU implementation (the package installed
in baseline/_ref) on the host cores, on bounded samples of the same workloads: the decode
step through its PagedKVCache (append_slots, write, gather; paged_cache.py:145-182) and
RoPE (rope.py:21-46) with the attention math of model.py:67-74, its evict_positions on
the 256-stream compaction trace, and its KV-streams and re-prefill rollouts at the CPU
bench configuration.  Without baseline/_ref the oracle port stands in (kind "port").
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
PKG_DIR = REPO / "faster-rl-training_b200"
REF_DIR = REPO / "baseline" / "_ref"  # the reference package, installed there unmodified


def _use_package() -> None:
    """This library's ``kvstreams`` (and the oracle) on the import path."""
    for p in (str(PKG_DIR), str(REPO)):
        if p not in sys.path:
            sys.path.insert(0, p)


def _use_reference() -> bool:
    """The reference's own ``kvstreams`` on the import path (a process that runs it never
    imports this library's package of the same name).  False when it is not installed."""
    if not (REF_DIR / "kvstreams" / "__init__.py").exists():
        return False
    sys.path.insert(0, str(REF_DIR))
    return True


def _workloads():
    """The seeded workload generators (kvstreams/workloads.py of this package, numpy only),
    loaded by path, so that a process running the reference's package uses the same streams."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("kvs_b200_workloads", PKG_DIR / "kvstreams" / "workloads.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclasses resolve their module by name
    spec.loader.exec_module(mod)
    return mod

METRIC = "rollout decode tok/s/GPU + replay tok/s; paged-attn HBM GB/s; replay TC util"
S, HQ, HKV, D, BS, NB = 64, 32, 8, 128, 16, 131072
THETA = 5e5
CTX = (1024, 16384)


def _peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "of measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "of fallback"}


def _traffic() -> dict:
    p = REPO / "profiles" / "traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


class ClockSampler:
    """SM clock and throttle reasons of one GPU, read through NVML (what nvidia-smi reads)
    every 5 ms on a background thread while the timed region runs.  Read-only."""

    REASONS = {  # NVML clocks-event reason bits
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4,
    }

    def __init__(self, gpu_index: int, interval: float = 0.005):
        self.idx = gpu_index
        self.interval = interval
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = None
        self._thread = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[self.idx]) if vis and vis.split(",")[self.idx].isdigit() else self.idx
            h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: report no samples rather than guess
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((float(mhz), int(rs)))
                except Exception:
                    pass
                self._stop.wait(self.interval)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self) -> dict:
        sm = [m for m, _ in self.samples]
        reasons = sorted(n for n, bit in self.REASONS.items() if any(r & bit for _, r in self.samples))
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(sm), "source": "NVML, 5 ms"}


# ---------------------------------------------------------------------- workload
def build_decode(dev, seed: int, value_seed: int, bs: int = BS):
    """Same stream shapes on every rank (weak scaling: identical work per GPU); the K/V,
    q, k, v values are drawn with a per-rank seed.  ``bs`` = 1 keeps the pool's bytes
    (NB * 16 one-token blocks)."""
    import torch

    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.rope import RotaryEmbedding
    from kvstreams.workloads import decode_state

    nb = NB * (BS // bs)
    st = decode_state(num_streams=S, ctx_range=CTX, block_size=bs, num_blocks=nb, seed=seed)
    cache = PagedKVCache(1, HKV, D, block_size=bs, num_blocks=nb, dtype=torch.bfloat16, device=dev, max_seqs=S,
                         max_blocks_per_seq=(CTX[1] + 4096) // bs)
    cache.load_state(range(S), st.tables, st.positions, st.free_list)
    g = torch.Generator(device=dev).manual_seed(value_seed)
    for t in (cache.k, cache.v):
        t.view(-1)[:] = torch.randn(t.numel(), generator=g, device=dev, dtype=torch.float32).bfloat16()
    q = torch.randn(S, HQ, D, generator=g, device=dev).bfloat16()
    k = torch.randn(S, HKV, D, generator=g, device=dev).bfloat16()
    v = torch.randn(S, HKV, D, generator=g, device=dev).bfloat16()
    rope = RotaryEmbedding(D, THETA)
    return st, cache, q, k, v, rope


def decode_bytes(lengths: np.ndarray, bs: int = BS) -> int:
    """Algorithmic HBM bytes of one decode launch: every live K and V row read once
    (4096 B per context token), the new K/V read + written, Q read, O written, tables."""
    kv_read = int(lengths.sum()) * HKV * D * 2 * 2
    per_stream = HQ * D * 2 * 2 + HKV * D * 2 * 2 * 2
    tables = int(sum(-(-int(n) // bs) for n in lengths)) * 4
    return kv_read + S * per_stream + tables


def decode_bs1_bench(dev, args, rank: int) -> dict:
    """The headline decode step with one-token blocks (SGLang-style): same streams, contexts,
    evicted spans and pool bytes (NB * 16 blocks of one token), one layer of fused RoPE /
    append / split-K paged attention per step, CUDA events around each kvs_paged_decode."""
    import torch

    from kvstreams import ops
    from kvstreams.distributed import reduce_max

    st, cache, q, k, v, rope = build_decode(dev, seed=1000, value_seed=1000 + rank, bs=1)
    inv = rope.table(dev, torch.bfloat16)
    seqs = list(range(S))
    pos = torch.as_tensor(st.next_positions, device=dev)
    out = torch.empty_like(q)
    path = []
    times = []
    for i in range(args.warmup + args.steps):
        p = pos + i
        mapping = cache.append_slots_batch(seqs, p)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ops.paged_forward(cache, seqs, None, 0, q, k, v, p, mapping, inv, D ** -0.5, out=out,
                          report_path=path if i == 0 else None)
        b.record()
        if i >= args.warmup:
            times.append((a, b))
    torch.cuda.synchronize(dev)
    ms = reduce_max(statistics.mean(x.elapsed_time(y) for x, y in times), dev)
    alg = decode_bytes(st.lengths + args.warmup + args.steps // 2 + 1, bs=1)
    gbs = alg / (ms * 1e-3) / 1e9
    peaks = _peaks()
    del cache, q, k, v, out
    _release_device_memory()
    return {"ms": ms, "gbs": gbs, "hbm_frac": gbs / peaks["hbm_gbs"], "kv_bytes": int(alg),
            "decode_tok_s": S / (ms * 1e-3), "fused_kernel": path == [1]}


def _release_device_memory() -> None:
    """Return the freed blocks of the legs before to the device.  A leg's engine, CUDA graphs and
    model can sit in reference cycles that only Python's cycle collector frees; without a
    collection here, whether a rank still held the previous leg's tens of GB when the next leg
    allocated depended on when each rank's collector last ran."""
    import gc

    import torch

    gc.collect()
    torch.cuda.empty_cache()


def decode_short_bench(dev, args, rank: int) -> dict:
    """The paged decode at rollout contexts: 64 streams of ~U[300, 500] live tokens (16-token
    blocks, 1-6 evicted spans), 32 layers per step sharing one batch descriptor, as one
    decode iteration of the rollout engine issues them; CUDA events around each step's 32
    kvs_paged_decode calls.  Per-launch fixed costs (batch scan, table gather, first blocks in
    flight, combine) weigh here, where each layer streams only ~105 MB."""
    import torch

    from kvstreams import ops
    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.rope import RotaryEmbedding
    from kvstreams.workloads import decode_state

    layers, ctx, nb = 32, (300, 500), 4096
    st = decode_state(num_streams=S, ctx_range=ctx, block_size=BS, num_blocks=nb, seed=7)
    cache = PagedKVCache(layers, HKV, D, block_size=BS, num_blocks=nb, dtype=torch.bfloat16, device=dev,
                         max_seqs=S, max_blocks_per_seq=64)
    cache.load_state(range(S), st.tables, st.positions, st.free_list)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    for t in (cache.k, cache.v):
        t.view(-1)[:] = torch.randn(t.numel(), generator=g, device=dev, dtype=torch.float32).bfloat16()
    q = torch.randn(S, HQ, D, generator=g, device=dev).bfloat16()
    k = torch.randn(S, HKV, D, generator=g, device=dev).bfloat16()
    v = torch.randn(S, HKV, D, generator=g, device=dev).bfloat16()
    inv = RotaryEmbedding(D, THETA).table(dev, torch.bfloat16)
    seqs = list(range(S))
    pos = torch.as_tensor(st.next_positions, device=dev)
    out = torch.empty_like(q)
    batch = cache._batch(seqs)
    steps, warm = 8, 3
    from kvstreams import _native as N

    def run(step0: int, planned: bool) -> float:
        times = []
        for i in range(warm + steps):
            p = pos + step0 + i
            mapping = cache.append_slots_batch(seqs, p)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for layer in range(layers):
                plan = (N.PLAN_BUILD if layer == 0 else N.PLAN_REUSE) if planned else N.PLAN_NONE
                ops.paged_forward(cache, seqs, None, layer, q, k, v, p, mapping, inv, D ** -0.5, out=out, batch=batch,
                                  plan=plan)
            b.record()
            if i >= warm:
                times.append((a, b))
        torch.cuda.synchronize(dev)
        return statistics.mean(x.elapsed_time(y) for x, y in times) / layers

    ms_noplan = run(0, False)
    ms = run(warm + steps, True)  # as the engine runs a step: the first layer stores the plan
    alg = decode_bytes(st.lengths + 2 * (warm + steps) - steps // 2)
    gbs = alg / (ms * 1e-3) / 1e9
    peaks = _peaks()
    del cache, q, k, v, out
    _release_device_memory()
    return {"workload": f"{S} streams, ctx U[{ctx[0]},{ctx[1]}] (mean {st.lengths.mean():.0f}), {layers} layers per "
                        "step, bs16", "us_per_layer": ms * 1e3, "gbs": gbs, "hbm_frac": gbs / peaks["hbm_gbs"],
            "us_per_layer_without_plan": ms_noplan * 1e3, "kv_bytes_per_layer": int(alg),
            "ideal_us": alg / (peaks["hbm_gbs"] * 1e9) * 1e6}


# ---------------------------------------------------------------------- cpu baseline
CPU_STREAMS = 4  # decode streams of the 64-stream workload per CPU step


def _cpu_threads() -> int:
    import torch

    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(n)
    return torch.get_num_threads()


def _ref_attend(q, k, v):
    """The attention of the reference's Attention.forward (model.py:67-74) for one decode
    query: GQA heads expanded by repeat_interleave, scaled scores, the (all-visible) mask,
    softmax, weighted values.  q [1, 1, Hq, D], k/v [1, n, Hkv, D]."""
    import torch

    rep = q.shape[2] // k.shape[2]
    k = k.repeat_interleave(rep, dim=2)
    v = v.repeat_interleave(rep, dim=2)
    mask = torch.ones(1, q.shape[1], k.shape[1], dtype=torch.bool)
    scores = torch.einsum("bqhd,bkhd->bhqk", q, k) * (q.shape[-1] ** -0.5)
    scores = scores.masked_fill(~mask[:, None, :, :], float("-inf"))
    return torch.einsum("bhqk,bkhd->bqhd", scores.softmax(dim=-1), v)


def ref_decode_leg(seed: int):
    """The decode step of the first CPU_STREAMS streams of the headline workload through the
    reference's own code, bf16 as the GPU arm: its RotaryEmbedding / apply_rope on the new q
    and k (rope.py:21-46), PagedKVCache.append_slots + write + gather (paged_cache.py:145-182),
    then the model.py:67-74 attention.  Returns (step, context tokens in the sample)."""
    import torch
    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.rope import RotaryEmbedding, apply_rope

    st = _workloads().decode_state(num_streams=S, ctx_range=CTX, block_size=BS, num_blocks=NB, seed=seed)
    sample = list(range(CPU_STREAMS))
    cache = PagedKVCache(1, HKV, D, block_size=BS, num_blocks=sum(len(st.tables[s]) + 8 for s in sample),
                         dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(seed)
    for s in sample:
        cache.add_sequence(s)
        pos = torch.from_numpy(st.positions[s])
        slots = cache.append_slots(s, pos)
        n = pos.numel()
        cache.write(0, slots, torch.randn(n, HKV, D, generator=g).bfloat16(),
                    torch.randn(n, HKV, D, generator=g).bfloat16())
    rope = RotaryEmbedding(D, THETA)
    q = torch.randn(len(sample), 1, 1, HQ, D, generator=g).bfloat16()
    k = torch.randn(len(sample), 1, 1, HKV, D, generator=g).bfloat16()
    v = torch.randn(len(sample), 1, HKV, D, generator=g).bfloat16()
    nxt = [int(st.next_positions[s]) for s in sample]

    def step() -> int:
        for i, s in enumerate(sample):
            p = torch.tensor([[nxt[i]]])
            nxt[i] += 1
            cos, sin = rope(p)
            qr, kr = apply_rope(q[i], cos, sin), apply_rope(k[i], cos, sin)
            slots = cache.append_slots(s, p[0])
            cache.write(0, slots, kr[0], v[i])
            kk, vv = cache.gather(s, 0)
            _ref_attend(qr, kk[None], vv[None])
        return len(sample)

    return step, int(sum(st.positions[s].size for s in sample))


def port_decode_leg(seed: int):
    """The same sample through the oracle port (numpy float32), when the reference package is
    not installed."""
    from oracle import kvs_oracle as O

    st = _workloads().decode_state(num_streams=S, ctx_range=CTX, block_size=BS, num_blocks=NB, seed=seed)
    rng = np.random.default_rng(seed)
    sample = list(range(CPU_STREAMS))
    pools = {s: (rng.standard_normal((st.positions[s].size, HKV, D), dtype=np.float32),
                 rng.standard_normal((st.positions[s].size, HKV, D), dtype=np.float32)) for s in sample}
    q = rng.standard_normal((len(sample), HQ, D), dtype=np.float32)
    knew = rng.standard_normal((len(sample), HKV, D), dtype=np.float32)
    vnew = rng.standard_normal((len(sample), HKV, D), dtype=np.float32)

    def step() -> int:
        for i, s in enumerate(sample):
            kp, vp = pools[s]
            pos = np.asarray([st.next_positions[s]])
            qr = O.rope_apply(q[i:i + 1], pos, THETA, np.float32)
            keys = np.concatenate([kp, O.rope_apply(knew[i:i + 1], pos, THETA, np.float32)])
            vals = np.concatenate([vp, vnew[i:i + 1]])
            O.gqa_attention(qr, keys, vals, np.ones((1, keys.shape[0]), bool), D ** -0.5, np.float32)
        return len(sample)

    return step, int(sum(st.positions[s].size for s in sample))


def ref_compaction_leg(bs: int, n_streams: int, seed: int) -> dict:
    """The compaction workload (256 streams x 512-block tables, pool 200000, 1-8 keep-recent
    events) through the reference's PagedKVCache: the first ``n_streams`` streams filled by its
    append_slots, then its evict_positions for their first eviction round, timed per stream."""
    import torch
    from kvstreams.paged_cache import PagedKVCache

    rounds = _workloads().compaction_plan(num_streams=256, blocks_per_stream=512, block_size=bs,
                                          num_events_range=(1, 8), seed=seed)
    cache = PagedKVCache(1, 1, 2, block_size=bs, num_blocks=200000)
    keep = set(range(n_streams))
    for s in sorted(keep):
        cache.add_sequence(s)
    for s, pos in zip(rounds[0].append_seqs, rounds[0].append_positions):
        if s in keep:
            cache.append_slots(s, torch.from_numpy(pos))
    ev = rounds[1]
    work = [(s, spans) for s, spans in zip(ev.evict_seqs, ev.evict_spans) if s in keep]
    t0 = time.perf_counter()
    for s, spans in work:
        cache.evict_positions(s, spans)
    sec = time.perf_counter() - t0
    per = sec / max(len(work), 1)
    return {"streams": len(work), "ms_per_stream": per * 1e3, "ms_per_256_streams": per * 256e3}


def ref_rollout_leg() -> dict:
    """The CPU bench configuration through the reference's own engines (fp32 default TinyLM,
    keep_recent keep_last=2, 16-token blocks padded, budget 256, recall env with 24
    distractors x filler 64, seeds 0-7, teacher-forced): KV-streams and re-prefill, 8
    rollouts each; tokens forwarded, wall time and the KV-streams replay mismatch."""
    from kvstreams.config import CacheConfig, RolloutConfig
    from kvstreams.envs import build_env
    from kvstreams.factory import build_stack
    from kvstreams.training import measure_mismatch

    out = {}
    for engine in ("kvstream", "reprefill"):
        st = build_stack(engine=engine, policy="keep_recent", policy_kwargs={"keep_last": 2},
                         cache_cfg=CacheConfig(16, pad_to_block=True),
                         rollout_cfg=RolloutConfig(context_budget=256, max_turns=128), dtype="float32", seed=0)
        t0 = time.perf_counter()
        rs = [st.engine.rollout(build_env("recall", seed=i, num_distractors=24, filler_len=64), teacher_forcing=True)
              for i in range(8)]
        out[f"{engine}_s"] = time.perf_counter() - t0
        out[f"{engine}_tokens_forwarded"] = sum(r.stats.tokens_forwarded for r in rs)
        if engine == "kvstream":
            out["kvstream_replay_max_dlogp"] = measure_mismatch(st.model, rs, "kvstream").max_abs_logprob_diff
    return out


def cpu_legs(args) -> dict:
    """Every CPU measurement of this run in one process: the reference's own code when it is
    installed (kind "reference"), else the oracle port for the decode step."""
    reference = _use_reference()
    if not reference:
        _use_package()  # the oracle port and its workloads
    cores = _cpu_threads()
    step, ctx = ref_decode_leg(0) if reference else port_decode_leg(0)
    for _ in range(args.warmup):
        step()
    rates = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        n = step()
        rates.append(n / (time.perf_counter() - t0))
    value = statistics.median(rates)
    out = {"kind": "reference" if reference else "port", "cores": cores, "decode_tok_s": value,
           "decode_sample": f"{CPU_STREAMS} of the {S} streams ({ctx} context tokens) per step, "
                            + ("the reference's PagedKVCache + RoPE + model.py:67-74 attention in bf16 (torch CPU)"
                               if reference else "oracle port, numpy float32")}
    if reference:
        out["compaction_bs16"] = ref_compaction_leg(16, 32, 0)
        out["compaction_bs1"] = ref_compaction_leg(1, 256, 0)
        out["config1"] = ref_rollout_leg()
    return out


def workload_config() -> dict:
    """The ``config`` of both arms' lines (the same workload)."""
    return {"workload": f"paged decode+append (one layer), 32q/8kv heads, D128, bs16, {S} streams/GPU, "
                        f"ctx U[{CTX[0]},{CTX[1]}], pool {NB} blocks, 1-6 evicted spans/stream, theta 5e5",
            "streams_per_gpu": S, "l2": "per-step KV read ~2.3 GB > 126 MB L2 (no flush needed)"}


# ---------------------------------------------------------------------- main arms
def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: rank 0 alone times the CPU path (the other ranks exit)."""
    if rank != 0:
        return
    cpu = cpu_legs(args)
    value = cpu["decode_tok_s"]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "decode tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * CPU_STREAMS / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if cpu["kind"] == "reference" else "f32", "data": "synthetic",
        "config": workload_config(),
        "cpu_baseline": {"value": value, "unit": "decode tok/s", "cores": cpu["cores"], "kind": cpu["kind"],
                         "sample": cpu["decode_sample"]},
        "e2e": {"value": value, "unit": "decode tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if "compaction_bs16" in cpu:
        line["secondary"] = {"compaction_bs16_ms_per_256_streams": cpu["compaction_bs16"]["ms_per_256_streams"],
                             "compaction_bs1_ms_per_256_streams": cpu["compaction_bs1"]["ms_per_256_streams"],
                             **{f"config1_{k}": v for k, v in cpu["config1"].items()}}
    if args.cpu_json:
        print(json.dumps(cpu), flush=True)
    else:
        print(json.dumps(line), flush=True)


def cpu_baseline_subprocess(args) -> dict:
    """cpu_legs in a process of its own (it imports the reference's package, whose name is
    this library's), on the same steps and warm-up."""
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR",
                                                            "MASTER_PORT", "LOCAL_WORLD_SIZE")}
    cmd = [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--cpu-json", "--steps", str(args.steps),
           "--warmup", str(args.warmup), "--streams", str(S), "--pool-blocks", str(NB), "--ctx-max", str(CTX[1])]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=900)
    if r.returncode != 0:
        raise RuntimeError(f"CPU baseline process failed:\n{r.stderr[-2000:]}")
    return json.loads(r.stdout.strip().splitlines()[-1])


def run_b200(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    from kvstreams import _native as N
    from kvstreams import ops
    from kvstreams.distributed import reduce_max

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = N.lib()
    st, cache, q, k, v, rope = build_decode(dev, seed=1000, value_seed=1000 + rank)
    inv = rope.table(dev, torch.bfloat16)
    seqs = list(range(S))
    steps_all = max(args.warmup, args.steps)
    # every step's positions, resident before the timed region (an input like q/k/v)
    pos_steps = torch.as_tensor(st.next_positions, device=dev)[None, :] + torch.arange(steps_all, device=dev)[:, None]
    out = torch.empty_like(q)
    snap = cache.snapshot_state()

    def step(i: int, ev=None):
        p = pos_steps[i]
        mapping = cache.append_slots_batch(seqs, p)
        if ev is not None:
            ev[0].record()
        ops.paged_forward(cache, seqs, None, 0, q, k, v, p, mapping, inv, D ** -0.5, out=out)
        if ev is not None:
            ev[1].record()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident timing
    for i in range(args.warmup):
        step(i)
    cache.restore_state(snap)
    barrier()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = lib.kvs_launch_count()
    with ClockSampler(local_rank) as clk:
        t_start.record()
        for i in range(args.steps):
            step(i, kev[i])
        t_end.record()
        barrier()
    launches = lib.kvs_launch_count() - launches0
    ms = t_start.elapsed_time(t_end)
    kernel_ms = [a.elapsed_time(b) for a, b in kev]
    ms = reduce_max(ms, dev)  # slowest rank (weak scaling: every rank times its own streams)
    clocks = clk.summary()
    lengths_mid = st.lengths + args.steps // 2 + 1
    alg_bytes = decode_bytes(lengths_mid)
    attn_ms = statistics.mean(kernel_ms)
    achieved_gbs = alg_bytes / (attn_ms * 1e-3) / 1e9

    # ---- end-to-end through the public call with host buffers.  Inputs and outputs are double
    # buffered on the device and moved on a copy stream: step i+1's upload and step i-1's download
    # overlap step i's kernels; every copy of every step stays inside the timed region.
    cache.restore_state(snap)
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hpos_steps = pos_steps.cpu().pin_memory()  # row i: step i's positions, uploaded with its q/k/v
    hpos = hpos_steps[0]
    hout = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    bufs = [tuple(torch.empty_like(t, device=dev) for t in (hq, hk, hv, hpos)) for _ in range(2)]
    outs = [out, torch.empty_like(out)]
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(args.steps + 1)]
    done = [torch.cuda.Event() for _ in range(args.steps)]
    fetched = [torch.cuda.Event() for _ in range(args.steps)]

    def upload(i):
        with torch.cuda.stream(copy):
            if i >= 2:
                copy.wait_event(done[i - 2])  # step i-2 has read this buffer
            for d_t, h_t in zip(bufs[i % 2], (hq, hk, hv, hpos_steps[i])):
                d_t.copy_(h_t, non_blocking=True)
            in_ready[i].record(copy)

    for i in range(args.warmup):
        bufs[0][0].copy_(hq, non_blocking=True)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    copy.wait_event(e0)
    upload(0)
    for i in range(args.steps):
        if i + 1 < args.steps:
            upload(i + 1)
        comp.wait_event(in_ready[i])
        if i >= 2:
            comp.wait_event(fetched[i - 2])  # the output buffer of step i-2 is on the host
        dq, dk, dv, dpos = bufs[i % 2]
        mapping = cache.append_slots_batch(seqs, dpos)
        ops.paged_forward(cache, seqs, None, 0, dq, dk, dv, dpos, mapping, inv, D ** -0.5, out=outs[i % 2])
        done[i].record(comp)
        with torch.cuda.stream(copy):
            copy.wait_event(done[i])
            hout[i % 2].copy_(outs[i % 2], non_blocking=True)
            fetched[i].record(copy)
    comp.wait_event(fetched[args.steps - 1])
    e1.record(comp)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    e2e_ms = reduce_max(e2e_ms, dev)
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hpos))
    d2h = hout[0].numel() * hout[0].element_size()

    detail = {}
    if not args.skip_secondary:
        del hq, hk, hv, hout
        detail = compaction_bench(dev, args, rank)
        detail["decode_bs1"] = decode_bs1_bench(dev, args, rank)
        detail["decode_short"] = decode_short_bench(dev, args, rank)
        detail["replay_attention"] = replay_bench(dev, args, rank)
        detail["replay_backward"] = replay_backward_bench(dev, args, rank)
        detail["compaction_policy"] = compaction_policy_bench(dev, args, rank)
        detail["lm_head_logprobs"] = lm_head_logprobs_bench(dev, args, rank)
        detail["config1"] = config1_bench(dev, args, rank)
        detail["rollout"] = rollout_bench(dev, args, rank, world)
        detail["prefill"] = prefill_bench(dev, args, rank)
        detail["replay_model"] = replay_model_bench(dev, args, rank)
        detail["replay_train"] = replay_train_bench(dev, args, rank)

    if rank != 0:
        return
    peaks = _peaks()
    # the CPU baseline: rank 0 at one GPU only
    cpu = cpu_baseline_subprocess(args) if world == 1 and not args.skip_cpu else None
    if cpu is not None:
        detail["cpu"] = cpu
    # DRAM bytes of one decode launch: ncu-measured traffic/algorithmic ratio (small-case
    # capture, profiles/) scaled by this launch's algorithmic bytes
    ratio = _traffic().get("paged_decode", {}).get("traffic_over_algorithmic")
    traffic = int(ratio * alg_bytes) if ratio else None
    line = {
        "metric": METRIC,
        "value": world * S * args.steps / (ms * 1e-3),
        "unit": "decode tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": workload_config(),
        "e2e": {"value": world * S * args.steps / (e2e_ms * 1e-3), "unit": "decode tok/s",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "ms_per_step": e2e_ms / args.steps,
                "copies": "pinned host q/k/v/positions uploaded and the output read back every step on a "
                          "second stream (double-buffered device buffers): step i+1's upload and step i-1's "
                          "download overlap step i's kernels, all inside the timed region"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved_gbs / peaks["hbm_gbs"], "peak_src": peaks["src"],
                     "frac_of_8tbs_spec": achieved_gbs / 8000.0, "bytes_per_launch": int(alg_bytes),
                     "traffic": traffic, "kernel": "decode_bf16_kernel (kvs_paged_decode)", "kernel_ms": attn_ms},
        "clocks": clocks,
    }
    if cpu is not None:
        line["cpu_baseline"] = {"value": cpu["decode_tok_s"], "unit": "decode tok/s", "cores": cpu["cores"],
                                "kind": cpu["kind"], "sample": cpu["decode_sample"]}
    if "rollout" in detail:
        r = detail["rollout"]
        line["rollout_decode_tok_s"] = r["rollout_decode_tok_s_total"]
        line["rollout_decode_tok_s_per_gpu"] = r["rollout_decode_tok_s_total"] / world
        line["rollout_ms_per_iteration"] = r["ms_per_iteration"]
    if detail:
        line["secondary"] = flat_secondary(detail)
    if args.detail:
        Path(args.detail).write_text(json.dumps(detail, indent=1))
    print(json.dumps(line), flush=True)


def flat_secondary(d: dict) -> dict:
    """The measurements beside the headline as one short flat dict of numbers (4 significant
    digits), last on the line so that a reader of the line's tail sees them; the nested
    ``--detail`` file holds everything.  Keys: *_tc / *_hbm = fraction of the measured bf16 /
    HBM peak; c1_* = the CPU bench configuration (8 rollouts, KV-streams vs re-prefill) on the
    GPU and through the reference on the host cores; *_cpu_ref_* = the reference on the host."""
    out = {}

    def put(key, *path):
        v = d
        for k in path:
            if not isinstance(v, dict) or k not in v:
                return
            v = v[k]
        out[key] = float(f"{v:.4g}") if isinstance(v, float) else v

    put("bs1_decode_hbm", "decode_bs1", "hbm_frac")
    put("rollout_ctx_decode_hbm", "decode_short", "hbm_frac")
    put("rollout_ctx_decode_us", "decode_short", "us_per_layer")
    put("prefill_tc", "prefill", "tc_frac")
    put("replay_tc", "replay_attention", "tc_frac")
    put("replay_bwd_tc", "replay_backward", "tc_frac")
    put("lse_gather_hbm", "lm_head_logprobs", "lse_gather_hbm_frac")
    put("bs1_decode_ms", "decode_bs1", "ms")
    put("prefill_ms", "prefill", "ms")
    put("replay_ms", "replay_attention", "ms")
    put("replay_bwd_ms", "replay_backward", "ms")
    put("compact16_ms", "compaction_bs16", "ms_per_call")
    put("compact1_ms", "compaction_bs1", "ms_per_call")
    put("compact16_cpu_ref_ms", "cpu", "compaction_bs16", "ms_per_256_streams")
    put("compact1_cpu_ref_ms", "cpu", "compaction_bs1", "ms_per_256_streams")
    put("round_host_ms", "compaction_policy", "host_policy_ms_per_round")
    put("round_dev_ms", "compaction_policy", "device_policy_gpu_ms_per_round")
    put("lmhead_epilogue_ms", "lm_head_logprobs", "epilogue_kernel_ms")
    put("lmhead_epilogue_tc", "lm_head_logprobs", "epilogue_kernel_tc_frac")
    put("lmhead_gemm_lse_ms", "lm_head_logprobs", "fused_fwd_ms")
    put("lmhead_torch_ms", "lm_head_logprobs", "torch_fwd_ms")
    put("sample_ms", "lm_head_logprobs", "sampling", "kvs_sample_kernel_ms")
    put("rollout_prefill_tok_s", "rollout", "prefill_tok_s_per_gpu")
    put("replay_model_tok_s", "replay_model", "replay_tok_s_per_gpu")
    put("train_tok_s", "replay_train", "train_tok_s_per_gpu")
    put("train_flop_frac", "replay_train", "model_flop_frac")
    put("c1_tok_kvs", "config1", "kvstream_tokens_forwarded")
    put("c1_tok_reprefill", "config1", "reprefill_tokens_forwarded")
    put("c1_gpu_kvs_s", "config1", "kvstream_s")
    put("c1_gpu_reprefill_s", "config1", "reprefill_s")
    put("c1_gpu_dlogp", "config1", "kvstream_replay_max_dlogp")
    put("c1_cpu_ref_kvs_s", "cpu", "config1", "kvstream_s")
    put("c1_cpu_ref_reprefill_s", "cpu", "config1", "reprefill_s")
    put("c1_cpu_ref_dlogp", "cpu", "config1", "kvstream_replay_max_dlogp")
    return out


def compaction_bench(dev, args, rank: int) -> dict:
    """256 streams x 512-block tables (pool 200000), 1-8 keep-recent events per stream: the
    first eviction round (every stream evicts its turn spans) as one batched evict_positions
    per step, state restored between steps."""
    import torch

    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.workloads import compaction_plan

    out = {}
    for bs, blocks in ((16, 512), (1, 512)):
        rounds = compaction_plan(num_streams=256, blocks_per_stream=blocks, block_size=bs, seed=rank,
                                 num_events_range=(1, 8))
        nb = 200000
        cache = PagedKVCache(1, 1, 2, block_size=bs, num_blocks=nb, dtype=torch.bfloat16, device=dev,
                             max_seqs=256, max_blocks_per_seq=blocks + 64)
        for s in range(256):
            cache.add_sequence(s)
        r0 = rounds[0]
        seqs, poss = r0.append_seqs, r0.append_positions
        start = 0
        while start < len(seqs):
            seen, end = set(), start
            while end < len(seqs) and seqs[end] not in seen:
                seen.add(seqs[end])
                end += 1
            cache.append_slots_batch(seqs[start:end], torch.as_tensor(np.concatenate(poss[start:end])),
                                     [p.size for p in poss[start:end]])
            start = end
        ev = rounds[1]
        snap = cache.snapshot_state()
        times = []
        for i in range(args.warmup + args.steps):
            cache.restore_state(snap)
            req = cache.prepare_evict(ev.evict_seqs, ev.evict_spans, span_cap=64)  # upload outside timing
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            cache.evict_prepared(req)
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                times.append(a.elapsed_time(b))
        ms = statistics.median(times)
        out[f"compaction_bs{bs}"] = {"streams": len(ev.evict_seqs), "ms_per_call": ms,
                                     "streams_per_s": len(ev.evict_seqs) / (ms * 1e-3),
                                     "live_tokens": int(blocks * bs * 256)}
    return out


def compaction_policy_bench(dev, args, rank: int) -> dict:
    """One compaction round of config 5 (64 rollouts over the 8192-token budget, Markovian
    keep_last=1, 16-token blocks): decide and evict for every rollout.  Host path as the
    engine's default (the reference policy in Python per rollout, one batched eviction, the
    evicted spans read back, events and segment marks updated): wall time per round.  Device
    path (kvs_compact: plan, eviction and bookkeeping kernels, no round trip): host time to
    launch and GPU time by CUDA events.  Cache state restored between rounds."""
    import torch

    from kvstreams.compaction.device import DeviceCompaction
    from kvstreams.compaction.policies import MarkovianPolicy
    from kvstreams.compaction.segments import Segment
    from kvstreams.paged_cache import PagedKVCache

    rng = np.random.default_rng(rank)
    n, budget, bs = 64, 8192, 16
    cache = PagedKVCache(1, 1, 2, block_size=bs, num_blocks=n * 1024, dtype=torch.bfloat16, device=dev,
                         max_seqs=n, max_blocks_per_seq=1024)
    policy = MarkovianPolicy(keep_last=1)
    segs, lens, needs = [], [], []
    for s in range(n):
        cache.add_sequence(s)
        seg = [Segment(0, "prompt", 0, 64, protected=True)]
        pos = 64
        while pos < budget - 256:
            ln = int(rng.integers(128, 1024)) // bs * bs
            seg.append(Segment(len(seg), "turn", pos, pos + ln))
            pos += ln
        cache.append_slots_batch([s], torch.arange(pos, dtype=torch.long), [pos])
        segs.append(seg)
        lens.append(pos)
        needs.append(int(rng.integers(512, 1024)))
    dc = DeviceCompaction(cache, policy, budget)
    snap = cache.snapshot_state()
    host_ms, launch_ms, gpu_ms, evicted = [], [], [], 0
    for i in range(args.warmup + args.steps):
        # host path
        cache.restore_state(snap)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        todo, plans = [], []
        for s in range(n):
            required = lens[s] + needs[s]
            if required > budget:
                plan = policy.plan(segs[s], lens[s], budget, required)
                if plan.spans:
                    todo.append(s)
                    plans.append(plan)
        ev = cache.evict_positions_batch(todo, [pl.spans for pl in plans])
        for s, e in zip(todo, ev):  # the engine's per-rollout bookkeeping
            for seg in segs[s]:
                covered = sum(max(0, min(seg.end, b) - max(seg.start, a)) for a, b in e)
                _ = covered >= seg.length
        t1 = time.perf_counter()
        evicted = sum(b - a for e in ev for a, b in e)
        # device path (segment tables uploaded before the timed call)
        cache.restore_state(snap)
        for s in range(n):
            dc.reset_slot(cache.slot(s))
            for seg in segs[s]:
                dc.add_segment(cache.slot(s), seg)
        dc._flush()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t2 = time.perf_counter()
        a.record()
        dc.compact([cache.slot(s) for s in range(n)], [0] * n, needs, lens)
        b.record()
        t3 = time.perf_counter()
        torch.cuda.synchronize()
        if i >= args.warmup:
            host_ms.append((t1 - t0) * 1e3)
            launch_ms.append((t3 - t2) * 1e3)
            gpu_ms.append(a.elapsed_time(b))
    dev_evicted = sum(sum(e.num_evicted for e in d["events"]) for d in dc.read([cache.slot(s) for s in range(n)]))
    return {"workload": "64 rollouts over an 8192-token budget, ~12 turns each, Markovian keep_last=1, bs 16",
            "host_policy_ms_per_round": statistics.median(host_ms),
            "device_policy_launch_ms_per_round": statistics.median(launch_ms),
            "device_policy_gpu_ms_per_round": statistics.median(gpu_ms),
            "evicted_tokens_per_round": evicted, "device_evicted_tokens_per_round": dev_evicted,
            "kernels": "compact_live + compact_plan + evict_mark + evict_apply + compact_commit"}


def lm_head_logprobs_bench(dev, args, rank: int) -> dict:
    """token_logprobs' lm_head stage for one chunk of config 4 (8192 tokens, d 4096, vocab
    128256, bf16 weight, float32 logits): forward and forward + backward, the torch chunk
    (GEMM, logits / T, log_softmax, gather; autograd keeps the log-softmax rows) against the
    fused chunk (GEMM + kvs_lse_gather; backward recomputes the logits, kvs_lse_gather_backward,
    two GEMMs).  The torch forward + backward uses bf16 logits cast to float32 (the float32-result
    GEMM has no autograd derivative).  The kvs_lse_gather kernel alone against the measured HBM bandwidth: it reads
    each float32 logit once (algorithmic bytes = rows x vocab x 4 + 16 B per row).  And the lm_head GEMM with
    the log-sum-exp in its epilogue (kvs_lm_head_logprobs, 2 x rows x vocab x d FLOP) against the
    measured bf16 peak; the fused forward + backward takes it for its forward."""
    import torch

    from kvstreams import ops
    from kvstreams.training.logprobs import _LmHeadLogprob

    n, d, V, temp = 8192, 4096, 128256, 1.0
    g = torch.Generator(device=dev).manual_seed(rank)
    w = (torch.randn(V, d, generator=g, device=dev) * 0.02).bfloat16()
    h = torch.randn(n, d, generator=g, device=dev).bfloat16()
    tgt = torch.randint(0, V, (n,), generator=g, device=dev)

    class _Head:  # the model's lm_head.logits for a standalone weight
        def logits(self, x):
            return torch.mm(x, w.t(), out_dtype=torch.float32)

    head = _Head()

    def ev_time(fn, reps=3):
        ts = []
        for i in range(2 + reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            if i >= 2:
                ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    def torch_fwd():
        with torch.no_grad():
            lp = torch.log_softmax(head.logits(h) / temp, dim=-1)
            return lp.gather(-1, tgt[:, None]).squeeze(-1)

    def fused_fwd():
        with torch.no_grad():
            return ops.lse_gather(head.logits(h), tgt, temp)[0]

    def torch_fb():  # differentiable torch form: bf16 GEMM, float32 log-softmax
        hh = h.detach().requires_grad_()
        ww = w.detach().requires_grad_()
        lp = torch.log_softmax(torch.nn.functional.linear(hh, ww).float() / temp, dim=-1)
        lp.gather(-1, tgt[:, None]).sum().backward()

    class _HeadW:
        def __init__(self, ww):
            self.ww = ww

        def logits(self, x):
            return torch.mm(x, self.ww.t(), out_dtype=torch.float32)

    def fused_fb():
        hh = h.detach().requires_grad_()
        ww = w.detach().requires_grad_()
        _LmHeadLogprob.apply(hh, ww, tgt, temp, _HeadW(ww)).sum().backward()

    logits = head.logits(h)
    k_ms = ev_time(lambda: ops.lse_gather(logits, tgt, temp))
    peaks = _peaks()
    gbs = (n * V * 4 + n * 16) / (k_ms * 1e-3) / 1e9
    out = {"workload": "8192 tokens x d 4096 x vocab 128256, bf16 weight, float32 logits",
           "torch_fwd_ms": ev_time(torch_fwd), "fused_fwd_ms": ev_time(fused_fwd),
           "lse_gather_kernel_ms": k_ms, "lse_gather_gbs": gbs, "lse_gather_hbm_frac": gbs / peaks["hbm_gbs"],
           "peak_src": peaks["src"]}
    del logits
    # the GEMM with the log-sum-exp in its epilogue (the logits never stored)
    if ops.lm_head_logprobs_supported(h, w):
        e_ms = ev_time(lambda: ops.lm_head_logprobs(h, w, tgt, temp))
        tf = 2.0 * n * V * d / (e_ms * 1e-3) / 1e12
        out.update({"epilogue_kernel_ms": e_ms, "epilogue_kernel_tflops": tf,
                    "epilogue_kernel_tc_frac": tf / peaks["bf16_tflops"],
                    "epilogue_kernel_max_abs_diff": float((ops.lm_head_logprobs(h, w, tgt, temp)[0]
                                                           - fused_fwd()).abs().max())})
    _release_device_memory()
    torch.cuda.reset_peak_memory_stats(dev)
    out["torch_fwd_bwd_ms"] = ev_time(torch_fb, reps=2)
    out["torch_fwd_bwd_peak_gb"] = torch.cuda.max_memory_allocated(dev) / 1e9
    _release_device_memory()
    torch.cuda.reset_peak_memory_stats(dev)
    out["fused_fwd_bwd_ms"] = ev_time(fused_fb, reps=2)
    out["fused_fwd_bwd_peak_gb"] = torch.cuda.max_memory_allocated(dev) / 1e9
    # the same outputs
    a, b = torch_fwd(), fused_fwd()
    out["max_abs_diff_vs_torch"] = float((a - b).abs().max())
    del w, h
    _release_device_memory()
    # the rollout's next-token step for 64 rollouts (engine/base.py:180-193): torch's
    # log_softmax + exp + multinomial + gather against one kvs_sample launch
    rows = 64
    x = torch.randn(rows, V, generator=g, device=dev) * 4
    tgen = torch.Generator(device=dev).manual_seed(rank)

    def torch_sample():
        lp = torch.log_softmax(x / temp, dim=-1)
        tok = torch.multinomial(lp.exp(), 1, generator=tgen).squeeze(1)
        return tok, lp.gather(1, tok[:, None]).squeeze(1)

    draws = iter(range(1 << 30))

    def graphed_ms(greedy, n=20):  # kernel time: n launches replayed as one CUDA graph
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            ops.sample(x, temp, greedy, seed=rank, offset=0)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(n):
                ops.sample(x, temp, greedy, seed=rank, offset=i)
        return ev_time(graph.replay, reps=5) / n

    s_ms = graphed_ms(False)
    sgbs = rows * V * 4 / (s_ms * 1e-3) / 1e9
    out["sampling"] = {"workload": "64 rows x vocab 128256 float32 logits, temperature 1",
                       "torch_call_ms": ev_time(torch_sample, reps=20),
                       "kvs_sample_call_ms": ev_time(lambda: ops.sample(x, temp, False, seed=rank,
                                                                        offset=next(draws)), reps=20),
                       "kvs_sample_kernel_ms": s_ms, "kvs_sample_gbs": sgbs,
                       "kvs_sample_hbm_frac": sgbs / peaks["hbm_gbs"], "greedy_kernel_ms": graphed_ms(True)}
    return out


def config1_bench(dev, args, rank: int) -> dict:
    """The CPU bench configuration on the GPU (fp32 default TinyLM, keep_recent keep_last=2,
    16-token blocks padded, budget 256, recall env with 24 distractors x filler 64, seeds 0-7,
    teacher-forced): 8 rollouts per engine in one rollout_batch call (KV-streams, re-prefill),
    tokens forwarded, wall time, and the KV-streams replay mismatch (gate 1e-5)."""
    import torch

    from kvstreams.config import CacheConfig, RolloutConfig
    from kvstreams.envs import build_env
    from kvstreams.factory import build_stack
    from kvstreams.training import measure_mismatch

    out = {}
    for engine in ("kvstream", "reprefill"):
        st = build_stack(engine=engine, policy="keep_recent", policy_kwargs={"keep_last": 2},
                         cache_cfg=CacheConfig(16, pad_to_block=True),
                         rollout_cfg=RolloutConfig(context_budget=256, max_turns=128), dtype="float32",
                         device=str(dev), seed=0)
        envs = [build_env("recall", seed=i, num_distractors=24, filler_len=64) for i in range(8)]
        st.engine.rollout_batch(envs[:1], teacher_forcing=True)  # warm-up
        torch.cuda.synchronize(dev)
        envs = [build_env("recall", seed=i, num_distractors=24, filler_len=64) for i in range(8)]
        t0 = time.perf_counter()
        rs = st.engine.rollout_batch(envs, teacher_forcing=True)
        torch.cuda.synchronize(dev)
        out[f"{engine}_s"] = time.perf_counter() - t0
        out[f"{engine}_tokens_forwarded"] = sum(r.stats.tokens_forwarded for r in rs)
        if engine == "kvstream":
            out["kvstream_replay_max_dlogp"] = measure_mismatch(st.model, rs, "kvstream").max_abs_logprob_diff
        del st
    return out


def lmhead_bench(dev, args, rank: int) -> dict:
    """The lm_head GEMM with the log-sum-exp epilogue alone: ``--lmhead-rows`` rows x d 4096 x
    vocab 128256 (bf16), CUDA events around kvs_lm_head_logprobs (2 x rows x vocab x d FLOP)."""
    import torch

    from kvstreams import ops

    n, d, V = args.lmhead_rows, 4096, 128256
    g = torch.Generator(device=dev).manual_seed(rank)
    w = (torch.randn(V, d, generator=g, device=dev) * 0.02).bfloat16()
    h = torch.randn(n, d, generator=g, device=dev).bfloat16()
    tgt = torch.randint(0, V, (n,), generator=g, device=dev)
    ts = []
    for i in range(args.warmup + args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ops.lm_head_logprobs(h, w, tgt, 1.0)
        b.record()
        torch.cuda.synchronize(dev)
        if i >= args.warmup:
            ts.append(a.elapsed_time(b))
    ms = statistics.median(ts)
    tf = 2.0 * n * V * d / (ms * 1e-3) / 1e12
    return {"rows": n, "ms": ms, "tflops": tf, "tc_frac": tf / _peaks()["bf16_tflops"]}


def rollout_bench(dev, args, rank: int, world: int = 1) -> dict:
    """Config 5 on one GPU: batched KV-streams rollouts of the Llama-3-8B architecture
    (random init, bf16; 32 layers, d 4096, 32/8 heads, FFN 14336, vocab 128256), 64 rollouts
    of 24 turns with observation and reply lengths ~U[64, 512] (uniform random ids), Markovian
    keep_last=1, context budget 8192, 16-token blocks padded.  Timed: ``--rollout-iters`` engine
    iterations (each one decode step of the generating rollouts plus one batched chunk call
    for turn starts and reply ends) after ``--rollout-warmup`` iterations, by CUDA events,
    preceded by an untimed run of ``--rollout-warmup-run`` iterations on other episodes."""
    import torch

    from kvstreams.compaction.policies import MarkovianPolicy
    from kvstreams.config import ModelConfig
    from kvstreams.distributed import reduce_max
    from kvstreams.engine.batched import BatchedKVStreams, synthetic_episodes
    from kvstreams.model import TinyLM
    from kvstreams.paged_cache import PagedKVCache

    _release_device_memory()
    n, budget, turns = args.rollout_streams, 8192, 24
    cfg = ModelConfig(vocab_size=128256, d_model=4096, n_layers=args.rollout_layers, n_heads=32, n_kv_heads=8,
                      d_ff=14336, rope_theta=5e5)
    torch.manual_seed(rank)
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with dev:
            model = TinyLM(cfg)
    finally:
        torch.set_default_dtype(old)
    model.eval()
    # budget + the largest turn reserve (reply 512 + 1 + 15 padding) + a block, per rollout
    blocks = n * ((budget + 512 + 16 + 16) // 16 + 1)
    cache = PagedKVCache(cfg.n_layers, cfg.n_kv_heads, cfg.head_dim, block_size=16, num_blocks=blocks,
                         dtype=torch.bfloat16, device=dev, max_seqs=n)
    def engine():
        return BatchedKVStreams(model, cache, MarkovianPolicy(keep_last=1), context_budget=budget, seed=rank,
                                cuda_graphs=not args.rollout_eager, device_policy=args.rollout_device_policy)

    # untimed warm-up on other episodes: the first use of each GEMM shape family loads and
    # selects its cuBLAS kernels (milliseconds per call), a one-time cost of the process that a
    # long run amortises and a 100-iteration window would otherwise carry
    if args.rollout_warmup_run > 0:
        engine().run(synthetic_episodes(n, turns=turns, turn_range=(64, 512), prompt_len=64, vocab=cfg.vocab_size,
                                        seed=7000 + rank), max_iterations=args.rollout_warmup_run)
        torch.cuda.synchronize(dev)
    eng = engine()
    eps = synthetic_episodes(n, turns=turns, turn_range=(64, 512), prompt_len=64, vocab=cfg.vocab_size,
                             seed=1000 + rank)
    W, K = args.rollout_warmup, args.rollout_iters
    ev = [torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
    tally = {"decode": 0, "prefill": 0}
    clk = ClockSampler(dev.index or 0)  # seconds of GEMM-heavy work: the power cap may lower the clock
    host_t = [0.0, 0.0]  # host wall clock at the first and last timed iteration

    prof = args.rollout_profile_iter

    def hook(i, n_dec, n_pre):
        # iterations [prof, prof + 3) inside cudaProfilerStart/Stop, for an ncu launch list
        # taken with --profile-from-start off (no work is skipped)
        if prof > 0 and i == prof - 1:
            torch.cuda.synchronize(dev)
            torch.cuda.profiler.start()
        elif prof > 0 and i == prof + 2:
            torch.cuda.synchronize(dev)
            torch.cuda.profiler.stop()
        if i == W:
            ev[0].record()
            host_t[0] = time.perf_counter()
            clk.__enter__()
        elif W < i <= W + K:
            tally["decode"] += n_dec
            tally["prefill"] += n_pre
            if i == W + K:
                ev[1].record()
                host_t[1] = time.perf_counter()
                clk.__exit__(None, None, None)

    from kvstreams import _native as N

    launches0 = N.lib().kvs_launch_count()
    rolls = eng.run(eps, max_iterations=None if args.rollout_full else W + K, on_iteration=hook)
    torch.cuda.synchronize(dev)
    ms = ev[0].elapsed_time(ev[1])
    ms = reduce_max(ms, dev)
    from kvstreams.distributed import reduce_sum

    total_decode = reduce_sum(tally["decode"], dev)  # every rank's rollouts over the slowest rank's time
    out = {
        "workload": f"{n} rollouts/GPU x {turns} turns, obs/reply ~U[64,512], Llama-3-8B arch "
                    f"({cfg.n_layers} layers) bf16 random init, Markovian keep_last=1, budget {budget}, bs16",
        "iterations_timed": K, "ms": ms,
        "decode_tokens": tally["decode"], "prefill_tokens": tally["prefill"],
        "rollout_decode_tok_s_per_gpu": tally["decode"] / (ms * 1e-3),
        "rollout_decode_tok_s_total": total_decode / (ms * 1e-3), "ranks": world,
        "prefill_tok_s_per_gpu": tally["prefill"] / (ms * 1e-3),
        "ms_per_iteration": ms / K,
        # the engine loop never waits on the GPU: the host's time per iteration, against the
        # device's, says whether the host kept the launch queue full
        "host_ms_per_iteration": (host_t[1] - host_t[0]) * 1e3 / K,
        "library_launches": N.lib().kvs_launch_count() - launches0,
        "engine_iterations": eng.last_iterations,
        "cuda_graphs": not args.rollout_eager,
        "device_policy": bool(args.rollout_device_policy),
        "clocks": clk.summary(),
    }
    if args.rollout_full:
        out["compactions"] = sum(r.stats.compactions for r in rolls)
        out["episode_wall_s"] = eng.last_wall
        out["decode_tokens_total"] = sum(r.stats.decode_tokens for r in rolls)
        out["rollout_decode_tok_s_per_gpu_whole_episode"] = out["decode_tokens_total"] / eng.last_wall
    del model, cache, eng, rolls
    _release_device_memory()
    return out


def prefill_bench(dev, args, rank: int) -> dict:
    """Tensor-core paged prefill, one layer: ``--prefill-streams`` sequences each appending a
    chunk of ~U[64,512] new tokens (the config-5 observation) onto live contexts ~U[1024,8192]
    with evicted gaps, 32q/8kv heads, D 128, bs 16, bf16.  Algorithmic work: 4 * Hq * D FLOP per
    (new token, visible entry) pair; timed by CUDA events around the kvs_paged_decode call
    (RoPE + append + attention), after warm-up, on fresh appends each step."""
    import numpy as np
    import torch

    from kvstreams import ops
    from kvstreams.distributed import reduce_max
    from kvstreams.paged_cache import PagedKVCache
    from kvstreams.rope import RotaryEmbedding
    from kvstreams.workloads import decode_state

    n, steps = args.prefill_streams, 3
    rng = np.random.default_rng(7 + rank)
    chunk = [int(x) for x in rng.integers(64, 513, size=n)]
    st = decode_state(num_streams=n, ctx_range=(1024, 8192), block_size=16,
                      num_blocks=n * ((8192 + (steps + 4) * 512) // 16 + 8), evicted_spans_range=(1, 6), seed=3 + rank)
    cache = PagedKVCache(1, 8, 128, block_size=16, num_blocks=st.num_blocks, dtype=torch.bfloat16, device=dev,
                         max_seqs=n)
    cache.load_state(range(n), st.tables, st.positions, st.free_list)
    g = torch.Generator(device=dev).manual_seed(rank)
    cache.k.normal_(generator=g)
    cache.v.normal_(generator=g)
    inv = RotaryEmbedding(128, 5e5).table(dev, torch.bfloat16)
    N = sum(chunk)
    q = torch.randn(N, 32, 128, generator=g, device=dev).bfloat16()
    kn = torch.randn(N, 8, 128, generator=g, device=dev).bfloat16()
    vn = torch.randn(N, 8, 128, generator=g, device=dev).bfloat16()
    nxt = [int(x) for x in st.next_positions]
    seqs = list(range(n))
    ms_all, flops_all = [], []
    for it in range(steps + 2):
        lens = [cache.num_tokens(s) for s in seqs]
        pos = torch.from_numpy(np.concatenate([np.arange(p, p + c) for p, c in zip(nxt, chunk)])).to(dev)
        mapping = cache.append_slots_batch(seqs, pos, chunk)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.paged_forward(cache, seqs, chunk, 0, q, kn, vn, pos, mapping, inv, 128 ** -0.5)
        e1.record()
        torch.cuda.synchronize(dev)
        if it >= 2:
            ms_all.append(e0.elapsed_time(e1))
            # visible pairs: token i of a chunk of c over n_old entries sees n_old + i + 1
            flops_all.append(sum(4 * 32 * 128 * (c * L + c * (c + 1) / 2) for c, L in zip(chunk, lens)))
        nxt = [p + c for p, c in zip(nxt, chunk)]
    cache.sync()
    ms = reduce_max(float(np.mean(ms_all)), dev)
    tf = float(np.mean(flops_all)) / (ms * 1e-3) / 1e12
    peaks = _peaks()
    del cache, q, kn, vn
    _release_device_memory()
    return {"workload": f"{n} sequences x chunk U[64,512] ({N} new tokens) onto contexts U[1024,8192], 32q/8kv D128 "
                        "bs16 bf16, one layer", "ms": ms, "tflops": tf, "tc_frac": tf / peaks["bf16_tflops"],
            "peak_src": peaks["src"], "prefill_tok_s": N / (ms * 1e-3),
            "kernel": "pair_attn_kernel<true> (tcgen05/TMEM paged prefill)"}


def replay_train_bench(dev, args, rank: int) -> dict:
    """A replay training step of config 4's model (Llama-3-8B architecture, random init, bf16):
    loss = sum(advantage * token_logprobs) and its backward through the whole model -- the
    masked replay forward and backward kernels in every layer, the lm_head chunks with their
    fused log-softmax + gather and its recomputing backward.  One stream of
    ``--replay-train-t`` tokens (3-8 keep-recent events); one untimed step, then one timed
    by CUDA events.  Model FLOP: 6 per parameter per token for the dense layers (forward +
    backward) + 14·Hq·D per visible pair per layer for attention (4 forward, 10 backward)."""
    import torch

    from kvstreams.config import ModelConfig
    from kvstreams.distributed import reduce_max
    from kvstreams.model import TinyLM
    from kvstreams.training.logprobs import token_logprobs
    from kvstreams.training.replay import Batch
    from kvstreams.workloads import replay_evicted_at, visible_pairs

    _release_device_memory()
    B, T = 1, args.replay_train_t
    cfg = ModelConfig(vocab_size=128256, d_model=4096, n_layers=args.rollout_layers, n_heads=32, n_kv_heads=8,
                      d_ff=14336, rope_theta=5e5)
    torch.manual_seed(rank)
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with dev:
            model = TinyLM(cfg)
    finally:
        torch.set_default_dtype(old)
    model.train()
    ev, _ = replay_evicted_at(batch=B, seq_len=T, seed=rank)
    pairs = visible_pairs(ev)
    g = torch.Generator(device=dev).manual_seed(rank)
    tokens = torch.randint(1, cfg.vocab_size, (B, T), generator=g, device=dev)
    adv = torch.randn(B, T, generator=g, device=dev)
    batch = Batch(tokens, torch.arange(T, device=dev).expand(B, T), torch.from_numpy(ev).to(dev),
                  torch.ones(B, T, dtype=torch.bool, device=dev), torch.zeros(B, T, device=dev),
                  torch.full((B,), T, dtype=torch.long, device=dev))

    def step():
        model.zero_grad(set_to_none=True)
        (token_logprobs(model, batch) * adv).sum().backward()

    step()
    torch.cuda.synchronize(dev)
    torch.cuda.reset_peak_memory_stats(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    step()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = reduce_max(e0.elapsed_time(e1), dev)
    finite = all(bool(torch.isfinite(p.grad).all()) for p in model.parameters() if p.grad is not None)
    n_dense = sum(p.numel() for n, p in model.named_parameters() if "embed" not in n and p.dim() == 2)
    flops = 6.0 * n_dense * B * T + 14.0 * cfg.n_heads * (cfg.d_model // cfg.n_heads) * pairs * cfg.n_layers
    peaks = _peaks()
    tf = flops / (ms * 1e-3) / 1e12
    peak_gb = torch.cuda.max_memory_allocated(dev) / 1e9
    del model, batch, tokens, adv
    _release_device_memory()
    return {"workload": f"B={B} T={T}, Llama-3-8B arch ({cfg.n_layers} layers) bf16 random init, 3-8 keep-recent "
                        "events: forward + backward of sum(advantage * token_logprobs)",
            "ms": ms, "train_tok_s_per_gpu": B * T / (ms * 1e-3), "model_tflops": tf,
            "model_flop_frac": tf / peaks["bf16_tflops"], "peak_src": peaks["src"], "peak_mem_gb": peak_gb,
            "grads_finite": finite}


def replay_model_bench(dev, args, rank: int) -> dict:
    """Config 4 end to end: the trainer's replay of KV-streams rollouts through the whole
    Llama-3-8B architecture (random init, bf16): token_logprobs = masked full-sequence forward
    (32 layers; attention in the tcgen05 replay kernel with the evicted_at mask) + lm_head +
    log-softmax + gather of every next token.  ``--replay-model-b`` streams of
    ``--replay-model-t`` tokens with 3-8 keep-recent events each; timed by CUDA events."""
    import torch

    from kvstreams.config import ModelConfig
    from kvstreams.model import TinyLM
    from kvstreams.ops import ReplayMask
    from kvstreams.training.logprobs import token_logprobs
    from kvstreams.training.replay import Batch
    from kvstreams.workloads import replay_evicted_at
    from kvstreams.distributed import reduce_max

    _release_device_memory()
    B, T = args.replay_model_b, args.replay_model_t
    cfg = ModelConfig(vocab_size=128256, d_model=4096, n_layers=args.rollout_layers, n_heads=32, n_kv_heads=8,
                      d_ff=14336, rope_theta=5e5)
    torch.manual_seed(rank)
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with dev:
            model = TinyLM(cfg)
    finally:
        torch.set_default_dtype(old)
    model.eval()
    ev, _ = replay_evicted_at(batch=B, seq_len=T, seed=rank)
    g = torch.Generator(device=dev).manual_seed(rank)
    tokens = torch.randint(1, cfg.vocab_size, (B, T), generator=g, device=dev)
    batch = Batch(tokens, torch.arange(T, device=dev).expand(B, T), torch.from_numpy(ev).to(dev),
                  torch.ones(B, T, dtype=torch.bool, device=dev), torch.zeros(B, T, device=dev),
                  torch.full((B,), T, dtype=torch.long, device=dev))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.no_grad():
        token_logprobs(model, batch)  # warm-up
        torch.cuda.synchronize(dev)
        e0.record()
        lp = token_logprobs(model, batch)
        e1.record()
    torch.cuda.synchronize(dev)
    ms = reduce_max(e0.elapsed_time(e1), dev)
    finite = bool(torch.isfinite(lp).all())
    del model, lp, batch, tokens
    _release_device_memory()
    return {"workload": f"B={B} T={T}, Llama-3-8B arch ({cfg.n_layers} layers) bf16 random init, 3-8 keep-recent "
                        f"events/stream: token_logprobs (masked forward + lm_head + log-softmax + gather)",
            "ms": ms, "replay_tok_s_per_gpu": B * T / (ms * 1e-3), "logprobs_finite": finite}


def replay_bench(dev, args, rank: int) -> dict:
    """Masked replay attention, one layer of the Llama-3-8B geometry (32 q / 8 kv heads,
    D 128, bf16): B streams x T tokens with 3-8 keep-recent compaction events each.
    Algorithmic work = 4 * Hq * D FLOP per visible (query, key) pair."""
    import torch

    from kvstreams import _native as N
    from kvstreams import ops
    from kvstreams.workloads import replay_evicted_at, visible_pairs

    B, T = args.replay_b, args.replay_t
    ev, _ = replay_evicted_at(batch=B, seq_len=T, seed=rank)
    pairs = visible_pairs(ev)
    causal = B * T * (T + 1) // 2
    g = torch.Generator(device=dev).manual_seed(rank)
    q = torch.randn(B, T, HQ, D, generator=g, device=dev).bfloat16()
    k = torch.randn(B, T, HKV, D, generator=g, device=dev).bfloat16()
    v = torch.randn(B, T, HKV, D, generator=g, device=dev).bfloat16()
    ev_t = torch.from_numpy(ev).to(dev)
    ln_t = torch.full((B,), T, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    lib = N.lib()
    times = []
    for i in range(2 + args.replay_steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ops.replay_attention(q, k, v, ev_t, ln_t, D ** -0.5, out=out)
        b.record()
        torch.cuda.synchronize()
        if i >= 2:
            times.append(a.elapsed_time(b))
    ms = statistics.median(times)
    flops = 4.0 * HQ * D * pairs
    peaks = _peaks()
    tf = flops / (ms * 1e-3) / 1e12
    del q, k, v, out
    return {"workload": f"B={B} T={T} 32q/8kv D128 bf16, 3-8 keep-recent events/stream (one layer)",
            "ms": ms, "visible_pairs": pairs, "visible_frac_of_causal": pairs / causal,
            "tflops": tf, "tc_frac": tf / peaks["bf16_tflops"], "peak_src": peaks["src"],
            "replay_attn_tok_s": B * T / (ms * 1e-3),
            "kernel": "pair_attn_kernel (tcgen05/TMEM, two query heads of a GQA group per CTA)"}


def replay_backward_bench(dev, args, rank: int) -> dict:
    """Backward of the masked replay attention, one layer of the Llama-3-8B geometry (bf16):
    the tcgen05 kernels (row statistics from the forward).  Algorithmic work = 10 * Hq * D
    FLOP per visible (query, key) pair (dV, dP, dS^T Q, dS K and the S recompute counted
    once, the standard 2.5x of the forward); the dK/dV kernel's second S/dP product is
    overhead, not work."""
    import torch

    from kvstreams import ops
    from kvstreams.workloads import replay_evicted_at, visible_pairs

    B, T = args.replay_bwd_b, args.replay_t
    ev, _ = replay_evicted_at(batch=B, seq_len=T, seed=rank)
    pairs = visible_pairs(ev)
    g = torch.Generator(device=dev).manual_seed(rank)
    q = torch.randn(B, T, HQ, D, generator=g, device=dev).bfloat16()
    k = torch.randn(B, T, HKV, D, generator=g, device=dev).bfloat16()
    v = torch.randn(B, T, HKV, D, generator=g, device=dev).bfloat16()
    go = torch.randn(B, T, HQ, D, generator=g, device=dev).bfloat16()
    ev_t = torch.from_numpy(ev).to(dev)
    ln_t = torch.full((B,), T, dtype=torch.int32, device=dev)
    lse = ops.row_lse_buffer(B, HQ, T, dev)
    out = ops.replay_attention(q, k, v, ev_t, ln_t, D ** -0.5, row_lse=lse)
    times = []
    for i in range(2):
        grads = ops.replay_attention_backward(q, k, v, ev_t, ln_t, D ** -0.5, out, go, row_lse=lse)
        del grads
    torch.cuda.synchronize()
    with ClockSampler(dev.index or 0) as clk:
        for i in range(args.replay_steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            grads = ops.replay_attention_backward(q, k, v, ev_t, ln_t, D ** -0.5, out, go, row_lse=lse)
            b.record()
            torch.cuda.synchronize()
            del grads
            times.append(a.elapsed_time(b))
    ms = statistics.median(times)
    flops = 10.0 * HQ * D * pairs
    peaks = _peaks()
    tf = flops / (ms * 1e-3) / 1e12
    del q, k, v, go, out, lse
    return {"workload": f"B={B} T={T} 32q/8kv D128 bf16, 3-8 keep-recent events/stream (one layer)",
            "ms": ms, "visible_pairs": pairs, "tflops": tf, "tc_frac": tf / peaks["bf16_tflops"],
            "tc_frac_sustained": tf / peaks["bf16_tflops_sustained"],
            "peak_src": peaks["src"], "replay_bwd_tok_s": B * T / (ms * 1e-3), "clocks": clk.summary(),
            "kernels": "replay_rowdot_kernel + replay_dkdv_kernel + replay_dq_kernel (tcgen05/TMEM)"}


def main() -> int:
    global S, NB, CTX
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-json", action="store_true", help=argparse.SUPPRESS)  # the CPU legs' process
    ap.add_argument("--skip-cpu", action="store_true", help="no CPU baseline leg")
    ap.add_argument("--detail", default="", help="write every measurement, nested, to this JSON file")
    ap.add_argument("--skip-secondary", action="store_true")
    ap.add_argument("--streams", type=int, default=S, help="decode streams per GPU (profiling: smaller case)")
    ap.add_argument("--pool-blocks", type=int, default=NB)
    ap.add_argument("--ctx-max", type=int, default=CTX[1])
    ap.add_argument("--replay-b", type=int, default=16)
    ap.add_argument("--replay-t", type=int, default=32768)
    ap.add_argument("--replay-steps", type=int, default=2)
    ap.add_argument("--replay-only", action="store_true", help="only the replay attention measurement")
    ap.add_argument("--replay-bwd-b", type=int, default=4)
    ap.add_argument("--replay-bwd-only", action="store_true", help="only the replay backward measurement")
    ap.add_argument("--compaction-policy-only", action="store_true",
                    help="only the host vs device compaction-round measurement")
    ap.add_argument("--logprobs-only", action="store_true", help="only the lm_head log-prob stage measurement")
    ap.add_argument("--rollout-streams", type=int, default=64)
    ap.add_argument("--rollout-layers", type=int, default=32)
    ap.add_argument("--rollout-warmup", type=int, default=20)
    ap.add_argument("--rollout-warmup-run", type=int, default=300,
                    help="engine iterations of an untimed warm-up run on other episodes first")
    ap.add_argument("--rollout-iters", type=int, default=100)
    ap.add_argument("--rollout-full", action="store_true", help="play the whole episodes (minutes)")
    ap.add_argument("--rollout-eager", action="store_true", help="decode steps without CUDA graphs")
    ap.add_argument("--rollout-profile-iter", type=int, default=0,
                    help="bracket engine iterations [N, N+3) with cudaProfilerStart/Stop")
    ap.add_argument("--rollout-device-policy", action="store_true",
                    help="compaction decided and applied on the device (kvs_compact)")
    ap.add_argument("--rollout-only", action="store_true", help="only the batched rollout measurement")
    ap.add_argument("--replay-model-b", type=int, default=2, help="config 4 uses 16")
    ap.add_argument("--replay-model-t", type=int, default=32768)
    ap.add_argument("--replay-model-only", action="store_true", help="only the whole-model replay measurement")
    ap.add_argument("--replay-train-t", type=int, default=16384)
    ap.add_argument("--replay-train-only", action="store_true", help="only the replay training step measurement")
    ap.add_argument("--prefill-streams", type=int, default=64)
    ap.add_argument("--prefill-only", action="store_true", help="only the paged prefill measurement")
    ap.add_argument("--decode-bs1-only", action="store_true", help="only the one-token-block decode measurement")
    ap.add_argument("--decode-short-only", action="store_true",
                    help="only the paged decode at rollout contexts (~400 tokens, 32 layers per step)")
    ap.add_argument("--lmhead-only", action="store_true", help="only the lm_head log-sum-exp GEMM")
    ap.add_argument("--lmhead-rows", type=int, default=8192)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    S, NB, CTX = args.streams, args.pool_blocks, (min(CTX[0], args.ctx_max), args.ctx_max)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return 0
    _use_package()
    import datetime

    import torch
    import torch.distributed as dist

    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    if local_world > 1 and hasattr(os, "sched_setaffinity"):
        # one rank per GPU on a shared host: each rank's engine loop and launches get their own
        # slice of the host cores instead of all ranks' threads competing for every core
        cores = sorted(os.sched_getaffinity(0))
        per = len(cores) // local_world
        if per >= 2:
            mine = cores[local_rank * per:(local_rank + 1) * per]
            os.sched_setaffinity(0, mine)
            torch.set_num_threads(len(mine))

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.replay_only:
            torch.cuda.set_device(local_rank)
            r = replay_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"replay_attention": r}), flush=True)
        elif args.logprobs_only:
            torch.cuda.set_device(local_rank)
            r = lm_head_logprobs_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"lm_head_logprobs": r}), flush=True)
        elif args.compaction_policy_only:
            torch.cuda.set_device(local_rank)
            r = compaction_policy_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"compaction_policy": r}), flush=True)
        elif args.replay_bwd_only:
            torch.cuda.set_device(local_rank)
            r = replay_backward_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"replay_backward": r}), flush=True)
        elif args.lmhead_only:
            torch.cuda.set_device(local_rank)
            r = lmhead_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"lmhead": r}), flush=True)
        elif args.decode_short_only:
            torch.cuda.set_device(local_rank)
            r = decode_short_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"decode_short": r}), flush=True)
        elif args.decode_bs1_only:
            torch.cuda.set_device(local_rank)
            r = decode_bs1_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"decode_bs1": r}), flush=True)
        elif args.prefill_only:
            torch.cuda.set_device(local_rank)
            r = prefill_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"prefill": r}), flush=True)
        elif args.replay_train_only:
            torch.cuda.set_device(local_rank)
            r = replay_train_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"replay_train": r}), flush=True)
        elif args.replay_model_only:
            torch.cuda.set_device(local_rank)
            r = replay_model_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"replay_model": r}), flush=True)
        elif args.rollout_only:
            torch.cuda.set_device(local_rank)
            r = rollout_bench(torch.device("cuda", local_rank), args, rank)
            if rank == 0:
                print(json.dumps({"rollout": r}), flush=True)
        else:
            run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
