"""Multi-turn text environments (envs/base.py:1-41)."""

from __future__ import annotations

import random
from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from typing import Optional


@dataclass
class EnvStart:
    system: str
    user: str


@dataclass
class EnvStep:
    user: Optional[str]
    reward: float = 0.0
    done: bool = False
    info: dict = field(default_factory=dict)


class Env(ABC):
    def __init__(self, seed: int = 0) -> None:
        self.seed = seed
        self.rng = random.Random(seed)

    @abstractmethod
    def reset(self) -> EnvStart: ...

    @abstractmethod
    def step(self, completion: str) -> EnvStep: ...

    @abstractmethod
    def oracle(self) -> str:
        """The ideal assistant completion for the current turn (teacher forcing)."""

    def summary_oracle(self) -> str:
        return ""
