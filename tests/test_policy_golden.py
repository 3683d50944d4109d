"""Compaction policies (compaction/policies.py:34-170) against plans recorded from the
reference on random segment lists (tests/golden/policy_plans.json, make_golden.py): the
host policies here, and the oracle restatement of the device plan kernel's loop."""

import json
from pathlib import Path

import pytest

GOLDEN = Path(__file__).parent / "golden" / "policy_plans.json"


def _cases():
    return json.loads(GOLDEN.read_text())


def _segments(case):
    from kvstreams.compaction.segments import Segment

    out = []
    for i, (s, e, prot, alive, part) in enumerate(case["segments"]):
        seg = Segment(i, "prompt" if prot else "turn", s, e, protected=bool(prot))
        if not alive:
            seg.evicted_at = e
        seg.partially_evicted = bool(part)
        out.append(seg)
    return out


def test_host_policies_match_reference_plans():
    from kvstreams.compaction.policies import build_policy

    for case in _cases():
        name, param = case["policy"], case["param"]
        pol = build_policy(name, **({"window": param} if name == "token_window" else {"keep_last": param}))
        plan = pol.plan(_segments(case), case["live"], case["budget"], case["required"])
        assert [list(x) for x in plan.spans] == case["spans"], case
        assert list(plan.segments) == case["chosen"], case


def test_oracle_plan_loop_matches_reference_plans():
    """oracle/compaction_plan.py restates the device kernel's single pass over a segment
    table (rank among alive segments for keep_last, running merge of adjacent spans)."""
    from oracle.compaction_plan import plan_table

    for case in _cases():
        spans, chosen = plan_table(case["policy"], case["param"], case["segments"], case["live"],
                                   case["budget"], case["required"])
        assert spans == case["spans"], case
        assert chosen == case["chosen"], case
