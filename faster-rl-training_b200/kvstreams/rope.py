"""Rotary position embeddings at explicit *logical* positions (rope.py:1-46).

Keys are rotated with their logical position when they are appended and never
re-rotated; after a compaction a key keeps its original rotation and new tokens
continue the original position counter.  The rotation itself runs inside the
kernels (``kvs_rope`` / the decode and replay kernels); this module owns the
frequency table they share, computed exactly like the reference: in float64,
then rounded to float32 (``rope.py:26-28``).  float64 models use that float32
table widened to double (the reference's ``.double()`` buffer conversion).

Unlike the reference, a bfloat16 model keeps the float32 table and float32 angles:
the reference casts the table and the positions to bfloat16, which destroys the
rotation at large positions.
"""

from __future__ import annotations

import numpy as np
import torch
from torch import nn

from . import ops


def inv_freq_table(head_dim: int, theta: float) -> np.ndarray:
    """float32 ``1 / theta**(2i/D)``, computed in float64 (rope.py:26-28)."""
    exponent = np.arange(0, head_dim, 2, dtype=np.float64) / head_dim
    return (1.0 / (theta ** exponent)).astype(np.float32)


class RotaryEmbedding(nn.Module):
    def __init__(self, head_dim: int, theta: float = 10000.0) -> None:
        super().__init__()
        if head_dim % 2:
            raise ValueError("head_dim must be even")
        self.head_dim = head_dim
        self.theta = theta
        self._f32 = inv_freq_table(head_dim, theta)
        self._tables: dict[tuple, torch.Tensor] = {}

    def table(self, device: torch.device, dtype: torch.dtype) -> torch.Tensor:
        """Device frequency table for activations of ``dtype`` (double for float64)."""
        want = torch.float64 if dtype == torch.float64 else torch.float32
        key = (str(device), want)
        t = self._tables.get(key)
        if t is None:
            t = torch.from_numpy(self._f32.astype(np.float64) if want == torch.float64 else self._f32).to(device)
            self._tables[key] = t
        return t

    def rotate_(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """Rotate ``x [..., H, D]`` in place at ``positions`` with the rope kernel."""
        return ops.rope_(x, positions, self.table(x.device, x.dtype))


def apply_rope_at(x: torch.Tensor, positions: torch.Tensor, theta: float = 10000.0) -> torch.Tensor:
    """Rotated copy of ``x [..., T, H, D]`` at ``positions [..., T]`` (rope.py:42-46 semantics)."""
    rope = RotaryEmbedding(x.shape[-1], theta)
    return rope.rotate_(x.contiguous().clone(), positions)
