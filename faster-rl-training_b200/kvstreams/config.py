"""Configuration dataclasses (same fields and defaults as kvstreams/config.py:9-87)."""

from __future__ import annotations

from dataclasses import asdict, dataclass


@dataclass
class ModelConfig:
    """Llama-style decoder geometry: RMSNorm, RoPE, GQA, SwiGLU (config.py:9-35)."""

    vocab_size: int = 104
    d_model: int = 64
    n_layers: int = 2
    n_heads: int = 4
    n_kv_heads: int = 2
    d_ff: int = 128
    rope_theta: float = 10000.0
    norm_eps: float = 1e-6
    init_std: float = 0.02
    # Optional explicit head size (Llama-3-8B: d_model 4096 / 32 heads = 128 anyway).
    head_dim_override: int = 0

    def __post_init__(self) -> None:
        if not self.head_dim_override and self.d_model % self.n_heads:
            raise ValueError("d_model must be divisible by n_heads")
        if self.n_heads % self.n_kv_heads:
            raise ValueError("n_heads must be divisible by n_kv_heads")
        if self.head_dim % 2:
            raise ValueError("head_dim must be even for RoPE")

    @property
    def head_dim(self) -> int:
        return self.head_dim_override or self.d_model // self.n_heads

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass
class CacheConfig:
    """Paged cache layout (config.py:39-65).

    block_size: tokens per physical block (16 like vLLM, 1 like SGLang).
    num_blocks: blocks in the shared pool.
    pad_to_block: pad prompt and completions to whole blocks so turns map to blocks.
    commit_partial_blocks: if False, a trailing partial block is re-forwarded next turn.
    max_seqs / max_blocks_per_seq: device table capacity (0 = num_blocks entries per sequence).
    """

    block_size: int = 16
    num_blocks: int = 4096
    pad_to_block: bool = True
    commit_partial_blocks: bool = True
    max_seqs: int = 16
    max_blocks_per_seq: int = 0

    def __post_init__(self) -> None:
        if self.block_size < 1:
            raise ValueError("block_size must be >= 1")


@dataclass
class SamplingConfig:
    temperature: float = 1.0
    max_new_tokens: int = 24
    greedy: bool = False


@dataclass
class RolloutConfig:
    """Soft live-KV budget checked before every turn (config.py:76-87)."""

    context_budget: int = 256
    max_turns: int = 32
    record_full_logprobs: bool = False
