"""CUDA graphs of the decode step: one token for each of ``n`` rollouts through the whole model.

A decode step of the 8B architecture is ~300 kernel launches (per layer: RMSNorm, the fused
q/k/v GEMM, the fused paged decode kernel, output projection + residual, RMSNorm, gate/up
GEMM, SiLU, product, down projection + residual) whose host-side cost exceeds their device
time.  :class:`DecodeGraphs` records that sequence once per batch size ``n`` and replays it:

* inputs live in static device buffers (token ids, positions, cache slots); the slot append
  runs inside the graph on them (``PagedKVCache.append_slots_device``), its host half
  (``reserve_slots``: pool check, host-mirror lengths) runs before each replay;
* the paged-decode scratch is sized once for the largest batch, so no replay reallocates it;
* the first decode step runs eagerly (it also warms cuBLAS and the library's one-time kernel
  attributes); right after it the graphs of every batch size 1..max_batch are recorded
  (recording executes nothing), so that no later step pays for a capture -- a rollout batch
  changes size whenever a rollout starts or ends a turn, and capturing a size on its first
  appearance spread ~0.1 s captures over the run.  All graphs share one memory pool (each
  graph's output stays referenced, and one graph's intermediates are dead before the next
  replays).
"""

from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np
import torch

from .. import _native as N
from ..paged_cache import SlotMapping


class DecodeGraphs:
    def __init__(self, model, cache, max_batch: int) -> None:
        self.model, self.cache = model, cache
        dev = model.device
        self.max_batch = int(max_batch)
        self.tok = torch.zeros(self.max_batch, dtype=torch.long, device=dev)
        self.pos = torch.zeros(self.max_batch, dtype=torch.long, device=dev)
        self.slots = torch.zeros(self.max_batch, dtype=torch.int32, device=dev)
        self.blocks = torch.zeros(self.max_batch, dtype=torch.int32, device=dev)
        self.offsets = torch.zeros(self.max_batch, dtype=torch.int32, device=dev)
        # pinned staging for the per-step inputs, a ring so that the host never rewrites a
        # buffer whose asynchronous copy has not run yet (each slot waits on its own event)
        self._ring = [(torch.zeros(self.max_batch, dtype=torch.int32).pin_memory(),
                       torch.zeros(self.max_batch, dtype=torch.long).pin_memory(), torch.cuda.Event())
                      for _ in range(4)]
        self._ri = 0
        nbytes = int(N.lib().kvs_decode_scratch_bytes(C.byref(cache.struct), self.max_batch, model.cfg.n_heads, 0))
        if nbytes:
            cache._decode_scratch(nbytes)
        self.graphs: dict[int, tuple] = {}
        self.pool = None
        self.replays = 0

    def _body(self, n: int) -> torch.Tensor:
        b = N.KvsBatch(seq_slots=self.slots.data_ptr(), cu_tokens=None, num_seqs=n, total_tokens=n)
        pos, blocks, offsets = self.pos[:n], self.blocks[:n], self.offsets[:n]
        self.cache.append_slots_device(b, pos, blocks, offsets)
        return self.model.forward_layers(self.tok[:n], pos, self.cache, (b, [self.slots]), SlotMapping(blocks, offsets))

    def _record(self, n: int) -> None:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool):
            out = self._body(n)
        self.pool = g.pool()
        self.graphs[n] = (g, out)

    @torch.no_grad()
    def step(self, seq_ids: Sequence[int], tokens: torch.Tensor, positions: Sequence[int]) -> torch.Tensor:
        """Logits ``[n, vocab]`` of one new token per sequence (same effect on the cache as
        ``model.forward_cached_batch(tokens, positions, cache, seq_ids)``)."""
        n = len(seq_ids)
        if n > self.max_batch:
            raise ValueError(f"{n} sequences exceed the graph batch capacity {self.max_batch}")
        if n not in self.graphs:
            pos_t = N.to_device(np.asarray(positions, dtype=np.int64), torch.long, self.model.device)
            logits = self.model.forward_cached_batch(tokens, pos_t, self.cache, seq_ids)
            torch.cuda.current_stream().synchronize()
            for m in ([n] if self.graphs else range(1, self.max_batch + 1)):
                self._record(m)
            return logits
        self.cache.reserve_slots(seq_ids)
        cache = self.cache
        h_slots, h_pos, ev = self._ring[self._ri]
        self._ri = (self._ri + 1) % len(self._ring)
        ev.synchronize()
        h_slots[:n] = torch.as_tensor([cache.slot(s) for s in seq_ids], dtype=torch.int32)
        h_pos[:n] = torch.as_tensor(np.asarray(positions, dtype=np.int64))
        self.slots[:n].copy_(h_slots[:n], non_blocking=True)
        self.pos[:n].copy_(h_pos[:n], non_blocking=True)
        ev.record()
        self.tok[:n].copy_(tokens)
        g, out = self.graphs[n]
        g.replay()
        self.replays += 1
        return out
