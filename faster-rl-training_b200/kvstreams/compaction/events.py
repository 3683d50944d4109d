"""Compaction log: when (stream length) each compaction happened and what it removed.

A token with stream index >= ``time`` was forwarded after the event and never saw
the evicted spans; earlier tokens did.  ``evicted_at`` turns the log into the
per-token eviction time that defines the replay mask (events.py:1-84).
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field

import numpy as np
import torch

from ..utils.spans import Span, span_length

NEVER = torch.iinfo(torch.long).max


@dataclass
class CompactionEvent:
    time: int
    evicted: list[Span]
    requested: list[Span] = field(default_factory=list)
    live_before: int = 0
    live_after: int = 0
    policy: str = ""
    segments: list[int] = field(default_factory=list)

    @property
    def num_evicted(self) -> int:
        return span_length(self.evicted)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["evicted"] = [list(s) for s in self.evicted]
        d["requested"] = [list(s) for s in self.requested]
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "CompactionEvent":
        d = dict(d)
        d["evicted"] = [tuple(s) for s in d["evicted"]]
        d["requested"] = [tuple(s) for s in d.get("requested", [])]
        return cls(**d)


class CompactionLog:
    def __init__(self, events: list[CompactionEvent] | None = None) -> None:
        self.events: list[CompactionEvent] = list(events or [])

    def append(self, event: CompactionEvent) -> None:
        if self.events and event.time < self.events[-1].time:
            raise ValueError("compaction events must be appended in time order")
        self.events.append(event)

    def __iter__(self):
        return iter(self.events)

    def __len__(self) -> int:
        return len(self.events)

    def span_triples(self) -> np.ndarray:
        """``[n, 3]`` int64 rows (start, end, time): the device evicted_at kernel's input."""
        rows = [(s, e, ev.time) for ev in self.events for s, e in ev.evicted]
        return np.asarray(rows, dtype=np.int64).reshape(-1, 3)

    def evicted_at(self, length: int, device=None) -> torch.Tensor:
        """``[length]`` int64: stream time at which each token was evicted, NEVER if kept.

        Computed by the device evicted_at kernel (events.py:66-74 semantics); with a
        non-CUDA ``device`` the result is copied there afterwards.
        """
        from ..ops import evicted_at_device

        dev = torch.device(device) if device is not None else None
        run_on = dev if dev is not None and dev.type == "cuda" else torch.device("cuda")
        out = evicted_at_device([self], [length], run_on)[0, :length]
        return out if dev is None or dev.type == "cuda" else out.to(dev)

    def total_evicted(self) -> int:
        return sum(ev.num_evicted for ev in self.events)

    def to_json(self) -> str:
        return json.dumps([ev.to_dict() for ev in self.events])

    @classmethod
    def from_json(cls, text: str) -> "CompactionLog":
        return cls([CompactionEvent.from_dict(d) for d in json.loads(text)])
