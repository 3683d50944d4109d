from .events import NEVER, CompactionEvent, CompactionLog
from .policies import (
    CompactionPlan,
    CompactionPolicy,
    KeepRecentTurns,
    MarkovianPolicy,
    SummaryPolicy,
    TokenSlidingWindow,
    build_policy,
)
from .segments import Segment

__all__ = [
    "NEVER",
    "CompactionEvent",
    "CompactionLog",
    "CompactionPlan",
    "CompactionPolicy",
    "KeepRecentTurns",
    "MarkovianPolicy",
    "Segment",
    "SummaryPolicy",
    "TokenSlidingWindow",
    "build_policy",
]
