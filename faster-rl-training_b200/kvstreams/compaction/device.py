"""Compaction decided and applied on the device (the ``kvs_compact`` entry point).

The reference decides compaction on the host, per rollout, before each turn
(engine/base.py:260-308: ``_maybe_compact`` / ``_compact`` with a ``CompactionPolicy.plan``
over the rollout's segments, compaction/policies.py:34-170).  :class:`DeviceCompaction` keeps
the segments, the compaction log and the stats of every sequence of a
:class:`~kvstreams.paged_cache.PagedKVCache` in device arrays, so that one call runs the
policy, the in-place eviction and the bookkeeping for a whole batch of rollouts without a
device round trip.  The host appends segments as turns end and reads the results back once
(:meth:`read`), when the rollouts are done.

Supported policies: ``keep_recent``, ``markovian``, ``summary`` (its spans; generating the
summary turn stays with the caller) and ``token_window``.
"""

from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np
import torch

from .. import _native as N
from .events import CompactionEvent
from .policies import CompactionPolicy
from .segments import Segment

_FLAG_PROTECTED, _FLAG_PARTIAL = 1, 2


def policy_code(policy: CompactionPolicy) -> tuple[int, int]:
    """(kvs_policy_code, param) of a policy instance."""
    code = getattr(policy, "device_code", None)
    if code is None or N.POLICY_CODES.get(policy.name) != code:
        raise ValueError(f"policy {policy.name!r} has no device implementation")
    return int(code), int(policy.device_param)


class DeviceCompaction:
    def __init__(self, cache, policy: CompactionPolicy, budget: int, max_segs: int = 256, max_events: int = 256,
                 span_pool: int = 4096, seg_pool: int = 4096) -> None:
        self.cache = cache
        self.policy = policy
        self.code, self.param = policy_code(policy)
        self.budget = int(budget)
        self.max_segs, self.max_events = int(max_segs), int(max_events)
        self.span_pool, self.seg_pool = int(span_pool), int(seg_pool)
        self._queued: list[tuple[int, int, int, int, int]] = []  # (slot, index, start, end, flags)
        self._count = np.zeros(0, dtype=np.int64)                  # host copy of the segment counts
        self._alloc(cache.max_seqs)
        self._scratch = None

    # ------------------------------------------------------------------ storage
    def _alloc(self, max_seqs: int) -> None:
        dev = self.cache.device
        S, M = max_seqs, self.max_segs
        old = getattr(self, "_t", None)
        i32 = dict(dtype=torch.int32, device=dev)
        t = {
            "start": torch.zeros(S, M, **i32), "end": torch.zeros(S, M, **i32),
            "evicted_at": torch.full((S, M), -1, **i32), "flags": torch.zeros(S, M, **i32),
            "count": torch.zeros(S, **i32), "ev_count": torch.zeros(S, **i32),
            "ev_meta": torch.zeros(S, self.max_events, N.EV_FIELDS, **i32),
            "ev_spans": torch.zeros(S, self.span_pool, 2, dtype=torch.long, device=dev),
            "ev_segs": torch.zeros(S, self.seg_pool, **i32), "ev_fill": torch.zeros(S, 2, **i32),
            "stats": torch.zeros(S, 4, **i32),
        }
        count = np.zeros(S, dtype=np.int64)
        if old is not None:
            n = old["count"].shape[0]
            for k in t:
                t[k][:n].copy_(old[k])
            count[:n] = self._count
        self._t, self._count, self.max_seqs = t, count, S
        self.struct = N.KvsSegments(
            start=t["start"].data_ptr(), end=t["end"].data_ptr(), evicted_at=t["evicted_at"].data_ptr(),
            flags=t["flags"].data_ptr(), count=t["count"].data_ptr(), ev_count=t["ev_count"].data_ptr(),
            ev_meta=t["ev_meta"].data_ptr(), ev_spans=t["ev_spans"].data_ptr(), ev_segs=t["ev_segs"].data_ptr(),
            ev_fill=t["ev_fill"].data_ptr(), stats=t["stats"].data_ptr(), max_seqs=S, max_segs=M,
            max_events=self.max_events, span_pool=self.span_pool, seg_pool=self.seg_pool, reserved=0)

    def _ensure(self, slot: int) -> None:
        if slot >= self.max_seqs:
            self._alloc(max(slot + 1, 2 * self.max_seqs))

    # ------------------------------------------------------------------ host updates
    def reset_slot(self, slot: int) -> None:
        """Forget everything recorded for a sequence slot (a new rollout takes it)."""
        self._ensure(slot)
        self._queued = [q for q in self._queued if q[0] != slot]
        t = self._t
        for k in ("count", "ev_count"):
            t[k][slot] = 0
        t["ev_fill"][slot] = 0
        t["stats"][slot] = 0
        t["evicted_at"][slot] = -1
        t["flags"][slot] = 0
        self._count[slot] = 0

    def add_segment(self, slot: int, seg: Segment) -> None:
        """Record a finished segment (engine/base.py:255, segments are appended in stream order)."""
        self._ensure(slot)
        idx = int(self._count[slot])
        if idx != seg.index:
            raise ValueError(f"segment {seg.index} of slot {slot} arrives out of order (expected {idx})")
        if idx >= self.max_segs:
            raise ValueError(f"more than max_segs={self.max_segs} segments in one rollout")
        self._queued.append((slot, idx, int(seg.start), int(seg.end), _FLAG_PROTECTED if seg.protected else 0))
        self._count[slot] = idx + 1

    def _flush(self) -> None:
        if not self._queued:
            return
        q = torch.tensor(self._queued, dtype=torch.int32).pin_memory().to(self.cache.device, non_blocking=True)
        slot, idx = q[:, 0].long(), q[:, 1].long()
        t = self._t
        t["start"][slot, idx] = q[:, 2]
        t["end"][slot, idx] = q[:, 3]
        t["flags"][slot, idx] = q[:, 4]
        t["evicted_at"][slot, idx] = -1
        slots = sorted({s for s, *_ in self._queued})
        cnt = torch.tensor([int(self._count[s]) for s in slots], dtype=torch.int32).pin_memory()
        t["count"][torch.tensor(slots, dtype=torch.long).pin_memory().to(self.cache.device, non_blocking=True)] = \
            cnt.to(self.cache.device, non_blocking=True)
        self._queued = []

    # ------------------------------------------------------------------ the call
    def compact(self, slots: Sequence[int], pending: Sequence[int], need: Sequence[int],
                now: Sequence[int]) -> None:
        """engine/base.py:260-308 for each slot (in the given order): pending tokens not yet in
        the cache, need = incoming + reserve, now = stream length.  Launches and returns."""
        n = len(slots)
        if n == 0:
            return
        if len(set(slots)) != n:
            raise ValueError("a sequence appears twice in one compaction call")
        for s in slots:
            self._ensure(s)
        self._flush()
        dev = self.cache.device
        step = torch.tensor(np.stack([np.asarray(pending), np.asarray(need), np.asarray(now)], axis=1),
                            dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        slot_t = torch.tensor(list(slots), dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        b = N.KvsBatch(seq_slots=slot_t.data_ptr(), cu_tokens=None, num_seqs=n, total_tokens=n)
        lib = N.lib()
        nbytes = int(lib.kvs_compact_scratch_bytes(C.byref(self.cache.struct), C.byref(self.struct), n))
        if self._scratch is None or self._scratch.numel() < nbytes:
            self._scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        rc = lib.kvs_compact(C.byref(self.cache.struct), C.byref(b), C.byref(self.struct), self.code, self.param,
                             self.budget, step.data_ptr(), self._scratch.data_ptr(), self._scratch.numel(),
                             N.stream_ptr(dev))
        N.check(rc, "kvs_compact")
        self.cache.mark_mirror_stale(slots)
        self._keep = (step, slot_t)  # alive until the kernels have read them

    # ------------------------------------------------------------------ results
    def read(self, slots: Sequence[int]) -> list[dict]:
        """Segments marks, events and stats of each slot (one device round trip).  Each entry:
        ``evicted_at`` / ``partial`` lists per segment, ``events`` (CompactionEvent objects
        without the policy name filled in), ``stats`` (compactions, evicted tokens, budget
        overflows) and ``peak_cached`` (the largest cache live count seen before an event)."""
        self._flush()
        t = self._t
        idx = torch.tensor(list(slots), dtype=torch.long, device=self.cache.device)
        host = {k: t[k].index_select(0, idx).cpu().numpy() for k in
                ("evicted_at", "flags", "count", "ev_count", "ev_meta", "ev_spans", "ev_segs", "stats")}
        self.cache._raise_status()
        out = []
        for r, slot in enumerate(slots):
            n = int(host["count"][r])
            evs = []
            peak = 0
            for e in range(int(host["ev_count"][r])):
                m = host["ev_meta"][r, e]
                so, nr, ne = int(m[7]), int(m[4]), int(m[5])
                sp = host["ev_spans"][r]
                requested = [(int(a), int(b)) for a, b in sp[so:so + nr]]
                evicted = [(int(a), int(b)) for a, b in sp[so + nr:so + nr + ne]]
                sg = host["ev_segs"][r, int(m[8]):int(m[8]) + int(m[6])]
                evs.append(CompactionEvent(time=int(m[0]), evicted=evicted, requested=requested,
                                           live_before=int(m[1]), live_after=int(m[2]), policy=self.policy.name,
                                           segments=[int(x) for x in sg]))
                peak = max(peak, int(m[3]))
            st = host["stats"][r]
            out.append({
                "evicted_at": [int(x) for x in host["evicted_at"][r, :n]],
                "partial": [bool(int(f) & _FLAG_PARTIAL) for f in host["flags"][r, :n]],
                "events": evs,
                "stats": {"compactions": int(st[0]), "evicted_tokens": int(st[1]), "budget_overflows": int(st[2])},
                "peak_cached": peak,
            })
        return out
