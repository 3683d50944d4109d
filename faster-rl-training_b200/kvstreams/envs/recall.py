"""Assignment recall (envs/recall.py:1-60): a task is assigned in turn 1, filler notes
follow, the last turn asks who owns the task.

The order of random draws (name, task, then one filler string per note turn, one
character at a time from lowercase letters plus three spaces) is part of the
episode definition: it fixes the token stream for a seed.
"""

from __future__ import annotations

import string

from .base import Env, EnvStart, EnvStep

NAMES = ["ana", "bob", "cai", "dev", "eli", "fay", "gus", "hal"]
TASKS = ["t%d" % i for i in range(10)]
_FILLER_ALPHABET = string.ascii_lowercase + "   "


class AssignmentRecallEnv(Env):
    def __init__(self, seed: int = 0, num_distractors: int = 4, filler_len: int = 24) -> None:
        super().__init__(seed)
        self.num_distractors = num_distractors
        self.filler_len = filler_len
        self.name = ""
        self.task = ""
        self.turn = 0

    @property
    def _last_turn(self) -> int:
        return self.num_distractors + 1

    def _filler(self) -> str:
        text = "".join(self.rng.choice(_FILLER_ALPHABET) for _ in range(self.filler_len))
        return text.strip() or "x"

    def reset(self) -> EnvStart:
        self.name = self.rng.choice(NAMES)
        self.task = self.rng.choice(TASKS)
        self.turn = 0
        return EnvStart(system="track task owners. reply ok to notes.", user=f"assign {self.task} to {self.name}")

    def oracle(self) -> str:
        return self.name if self.turn == self._last_turn else "ok"

    def summary_oracle(self) -> str:
        return f"{self.task}={self.name}"

    def step(self, completion: str) -> EnvStep:
        if self.turn == self._last_turn:
            ok = completion.strip() == self.name
            return EnvStep(user=None, reward=1.0 if ok else 0.0, done=True, info={"answer": self.name})
        self.turn += 1
        if self.turn == self._last_turn:
            return EnvStep(user=f"who has {self.task}?")
        return EnvStep(user=f"note: {self._filler()}")
