"""CPU oracle of the device compaction policies -- TEST INFRASTRUCTURE ONLY.

Restates, as the single pass over a sequence's segment table that the device plan kernel
makes, the reference's CompactionPolicy.plan (compaction/policies.py:34-170) with
merge_spans (utils/spans.py:10-18), and the bookkeeping after an eviction
(engine/base.py:287-308).  Pinned against plans recorded from the reference
(tests/golden/policy_plans.json, tests/test_policy_golden.py).  Only tests may import it.

A segment is ``[start, end, protected, alive, partially_evicted]``.
"""

from __future__ import annotations

POLICY_CODES = {"keep_recent": 0, "markovian": 1, "summary": 2, "token_window": 3}


def plan_table(policy: str, param: int, segments, live: int, budget: int, required: int):
    """(merged spans, chosen segment indices) of ``policy`` (policies.py:34-170)."""
    spans: list[list[int]] = []
    chosen: list[int] = []

    def add(s: int, e: int) -> None:  # merge_spans on spans that arrive in stream order
        if e <= s:
            return
        if spans and s <= spans[-1][1]:
            spans[-1][1] = max(spans[-1][1], e)
        else:
            spans.append([s, e])

    if policy == "token_window":
        if not segments:
            return spans, chosen
        prompt_end = max((seg[1] for seg in segments if seg[2]), default=0)
        cut = min(segments[-1][1] - param, segments[-1][0])
        if cut <= prompt_end:
            return spans, chosen
        chosen = [i for i, seg in enumerate(segments) if seg[0] < cut and seg[1] > prompt_end and seg[3]]
        add(prompt_end, cut)
        return spans, chosen
    # keep_recent / markovian / summary: alive, not partially evicted, not protected, and not
    # among the keep_last most recent alive-and-whole segments (policies.py:34-38)
    n_whole = sum(1 for seg in segments if seg[3] and not seg[4])
    overflow = required - budget
    freed = 0
    rank = 0
    for i, (s, e, prot, alive, part) in enumerate(segments):
        if not alive or part:
            continue
        recent = rank >= n_whole - param
        rank += 1
        if recent or prot:
            continue
        if policy == "keep_recent" and freed >= overflow:
            break
        chosen.append(i)
        freed += e - s
        add(s, e)
    return spans, chosen


def commit(segments, evicted, now: int):
    """engine/base.py:300-308: a segment wholly covered by the evicted spans gets
    evicted_at = now, a partly covered one is marked partially evicted.  Returns the new
    segment list (entries ``[start, end, protected, evicted_at (-1 alive), partial]``)."""
    out = []
    for s, e, prot, ev_at, part in segments:
        if ev_at < 0:
            covered = sum(max(0, min(e, b) - max(s, a)) for a, b in evicted)
            if covered >= e - s:
                ev_at, part = now, 0
            elif covered:
                part = 1
        out.append([s, e, prot, ev_at, part])
    return out
