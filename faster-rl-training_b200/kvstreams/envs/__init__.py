from .base import Env, EnvStart, EnvStep
from .chain_sum import ChainSumEnv
from .recall import AssignmentRecallEnv

ENVS = {"recall": AssignmentRecallEnv, "chainsum": ChainSumEnv}


def build_env(name: str, seed: int = 0, **kwargs) -> Env:
    if name not in ENVS:
        raise ValueError(f"unknown env {name!r}; choose from {sorted(ENVS)}")
    return ENVS[name](seed=seed, **kwargs)


__all__ = ["AssignmentRecallEnv", "ChainSumEnv", "ENVS", "Env", "EnvStart", "EnvStep", "build_env"]
