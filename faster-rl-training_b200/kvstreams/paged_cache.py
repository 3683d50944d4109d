"""Device-resident paged KV cache with block tables (kvstreams/paged_cache.py:81-273).

Storage is a pool of fixed-size blocks, ``k, v = [n_layers, num_blocks, block_size,
n_kv_heads, head_dim]`` (the reference layout), plus ``slot_pos[num_blocks,
block_size]``: the logical (RoPE) position stored in every slot, -1 when empty.

Everything the reference keeps in Python lists lives on the GPU here:

* block tables ``[max_seqs, max_blocks]`` int32 and their lengths,
* the LIFO free list (``free_stack`` + ``free_top``; the next block handed out is
  ``free_stack[free_top - 1]``, exactly the end of the reference's ``_free`` list),
* per-block owner (the reference's ``_used`` set) and the CacheStats counters.

Allocation, whole-block eviction + table join (a stream-compaction kernel),
truncation, freeing and the invariant check run as kernels of libkvs_b200.so.
The host keeps an exact mirror of the per-sequence token/block counts and of the
number of free blocks, so that ``num_tokens`` and out-of-blocks checks need no
device round trip; after an eviction (whose outcome depends on device data) the
mirror is refreshed from the device.

Batched calls (``append_slots_batch``, ``evict_positions_batch``, ...) process
sequences in the given order and reproduce, bit for bit, the state reached by
calling the single-sequence method once per sequence in that order.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, fields
from typing import Iterable, Optional, Sequence

import numpy as np
import torch

from . import _native as N
from .config import CacheConfig, ModelConfig
from .utils.spans import Span, merge_spans


class OutOfBlocksError(RuntimeError):
    pass


@dataclass
class SlotMapping:
    """Physical (block, offset) of every token written by one forward call (paged_cache.py:62-67)."""

    blocks: torch.Tensor
    offsets: torch.Tensor


@dataclass
class CacheStats:
    written_tokens: int = 0
    evicted_tokens: int = 0
    evicted_blocks: int = 0
    truncated_tokens: int = 0
    peak_blocks: int = 0
    eviction_calls: int = 0
    shrunk_tokens: int = 0  # requested for eviction but kept because the block was shared


@dataclass
class EvictRequest:
    """An evict_positions batch already uploaded to the device (see PagedKVCache.prepare_evict)."""

    slots: list
    batch: object
    keep: list
    cu: torch.Tensor
    starts: torch.Tensor
    ends: torch.Tensor
    out: torch.Tensor
    counts: torch.Tensor
    cap: int


class BlockAllocator:
    """View of a cache's device free list (paged_cache.py:32-59): LIFO over ``num_blocks``."""

    def __init__(self, cache: "PagedKVCache") -> None:
        self._cache = cache
        self.num_blocks = cache.num_blocks

    @property
    def num_free(self) -> int:
        return self._cache._h_top

    @property
    def num_used(self) -> int:
        return self.num_blocks - self._cache._h_top

    def free_list(self) -> list[int]:
        """The free list bottom-to-top (the reference's ``_free``); reads the device."""
        c = self._cache
        top = int(c._free_top.item())
        return c._free_stack[:top].tolist()


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype not in N.DTYPE_CODE:
        raise ValueError(f"unsupported cache dtype {dtype}")
    return N.DTYPE_CODE[dtype]


class PagedKVCache:
    def __init__(
        self,
        n_layers: int,
        n_kv_heads: int,
        head_dim: int,
        block_size: int = 16,
        num_blocks: int = 4096,
        device: Optional[torch.device | str] = None,
        dtype: torch.dtype = torch.float32,
        max_seqs: int = 16,
        max_blocks_per_seq: int = 0,
    ) -> None:
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        if self.device.type != "cuda":
            raise RuntimeError(
                f"PagedKVCache lives in GPU memory; device {self.device} is not a CUDA device (no CPU path)"
            )
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self._lib = N.lib()
        self.block_size = int(block_size)
        self.num_blocks = int(num_blocks)
        self.n_layers = int(n_layers)
        self.n_kv_heads = int(n_kv_heads)
        self.head_dim = int(head_dim)
        self.dtype = dtype
        self.max_blocks = int(max_blocks_per_seq) or self.num_blocks
        dev = self.device
        shape = (n_layers, num_blocks, block_size, n_kv_heads, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=dev)
        self.v = torch.zeros(shape, dtype=dtype, device=dev)
        self.slot_pos = torch.empty((num_blocks, block_size), dtype=torch.long, device=dev)
        self._free_stack = torch.empty(num_blocks, dtype=torch.int32, device=dev)
        self._free_top = torch.empty(1, dtype=torch.int32, device=dev)
        self._owner = torch.empty(num_blocks, dtype=torch.int32, device=dev)
        self._stats = torch.zeros(N.STAT_COUNT, dtype=torch.long, device=dev)
        self._status = torch.zeros(N.STATUS_WORDS, dtype=torch.int32, device=dev)
        self._alloc_seq_storage(int(max_seqs))
        self._h_top = self.num_blocks
        self._slot_of: dict[int, int] = {}
        self._stale: set[int] = set()  # slots whose host mirror is a bound (device-side eviction)
        self._scratch = torch.empty(0, dtype=torch.uint8, device=dev)
        self.allocator = BlockAllocator(self)
        with torch.cuda.device(dev):
            N.check(self._lib.kvs_cache_reset(C.byref(self._struct), N.stream_ptr(dev)), "kvs_cache_reset")

    # ------------------------------------------------------------------ storage
    def _alloc_seq_storage(self, max_seqs: int, old: Optional[dict] = None) -> None:
        dev = self.device
        self.max_seqs = max_seqs
        self._tables = torch.full((max_seqs, self.max_blocks), -1, dtype=torch.int32, device=dev)
        self._n_blocks = torch.zeros(max_seqs, dtype=torch.int32, device=dev)
        self._lengths = torch.zeros(max_seqs, dtype=torch.int32, device=dev)
        self._slot_ids = torch.arange(max_seqs, dtype=torch.int32, device=dev)
        h_len = np.zeros(max_seqs, dtype=np.int64)
        h_nb = np.zeros(max_seqs, dtype=np.int64)
        if old is not None:
            n = old["tables"].shape[0]
            self._tables[:n].copy_(old["tables"])
            self._n_blocks[:n].copy_(old["n_blocks"])
            self._lengths[:n].copy_(old["lengths"])
            h_len[:n] = old["h_len"]
            h_nb[:n] = old["h_nb"]
        self._h_len, self._h_nb = h_len, h_nb
        self._free_slots = [s for s in range(max_seqs - 1, -1, -1) if old is None or s >= old["tables"].shape[0]]
        if old is not None:
            self._free_slots = list(range(max_seqs - 1, old["tables"].shape[0] - 1, -1)) + old["free_slots"]
        self._struct = N.KvsCache(
            k=self.k.data_ptr(),
            v=self.v.data_ptr(),
            slot_pos=self.slot_pos.data_ptr(),
            tables=self._tables.data_ptr(),
            n_blocks=self._n_blocks.data_ptr(),
            lengths=self._lengths.data_ptr(),
            free_stack=self._free_stack.data_ptr(),
            free_top=self._free_top.data_ptr(),
            block_owner=self._owner.data_ptr(),
            stats=self._stats.data_ptr(),
            status=self._status.data_ptr(),
            n_layers=self.n_layers,
            num_blocks=self.num_blocks,
            block_size=self.block_size,
            n_kv_heads=self.n_kv_heads,
            head_dim=self.head_dim,
            max_seqs=max_seqs,
            max_blocks=self.max_blocks,
            dtype=_dtype_code(self.dtype),
        )

    def _grow_seqs(self) -> None:
        old = {
            "tables": self._tables,
            "n_blocks": self._n_blocks,
            "lengths": self._lengths,
            "h_len": self._h_len,
            "h_nb": self._h_nb,
            "free_slots": self._free_slots,
        }
        self._alloc_seq_storage(max(2 * self.max_seqs, 1), old)

    def _scratch_buf(self, nbytes: int) -> torch.Tensor:
        if self._scratch.numel() < nbytes:
            self._scratch = torch.empty(max(nbytes, 2 * self._scratch.numel()), dtype=torch.uint8, device=self.device)
        return self._scratch

    def _decode_scratch(self, nbytes: int) -> torch.Tensor:
        """Split-K partials of the decode kernel; its counters must start (and end) at zero,
        so the buffer is zeroed once when (re)allocated and the kernel leaves it zeroed."""
        buf = getattr(self, "_dscratch", None)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._dscratch = buf
        return buf

    @property
    def struct(self) -> N.KvsCache:
        """The C ABI view (kvs_cache) of this cache."""
        return self._struct

    def _stream(self) -> int:
        return N.stream_ptr(self.device)

    @classmethod
    def from_config(cls, model_cfg: ModelConfig, cache_cfg: CacheConfig, device=None, dtype=torch.float32):
        return cls(
            n_layers=model_cfg.n_layers,
            n_kv_heads=model_cfg.n_kv_heads,
            head_dim=model_cfg.head_dim,
            block_size=cache_cfg.block_size,
            num_blocks=cache_cfg.num_blocks,
            device=device,
            dtype=dtype,
            max_seqs=getattr(cache_cfg, "max_seqs", 16),
            max_blocks_per_seq=getattr(cache_cfg, "max_blocks_per_seq", 0),
        )

    # ------------------------------------------------------------------ status
    def _raise_status(self) -> None:
        st = self._status.tolist()
        if st[0] == N.ST_OK:
            return
        self._status.zero_()
        code, a, b, c = st
        if code == N.ST_OUT_OF_BLOCKS:
            raise OutOfBlocksError(f"all {self.num_blocks} KV blocks are in use (needed {a}, free {b})")
        if code == N.ST_DOUBLE_FREE:
            raise ValueError(f"double free of block {a}")
        if code == N.ST_TRUNCATE:
            raise ValueError("cannot truncate more tokens than are live")
        if code == N.ST_SEQ_TOO_LONG:
            raise RuntimeError(f"sequence in slot {a} has {b} live entries, more than the 32768 the "
                               "tensor-core prefill attends over")
        if code == N.ST_LOG_CAPACITY:
            raise RuntimeError(f"device compaction log of slot {a} is full ({b} events, {c} spans): "
                               "raise DeviceCompaction's max_events / span_pool")
        if code == N.ST_KERNEL_TIMEOUT:
            raise RuntimeError(f"a tensor-core attention kernel timed out waiting (site {a}, CTA {b}); "
                               "its outputs are invalid")
        raise RuntimeError(f"kvstreams device status {code} (details {a}, {b}, {c})")

    def sync(self) -> None:
        """Wait for queued cache kernels and raise any device-side error they reported."""
        torch.cuda.current_stream(self.device).synchronize()
        self._raise_status()

    def mark_mirror_stale(self, slots: Sequence[int]) -> None:
        """A device-side eviction ran for these slots without a round trip: their host-mirror
        lengths and table sizes (and the free count) are now upper / lower bounds.  Allocation
        checks that fail on the bounds re-read the device state before raising."""
        self._stale.update(int(s) for s in slots)

    def _refresh(self, slots: Sequence[int]) -> None:
        """Re-read lengths / table sizes / free count after a data-dependent kernel."""
        idx = torch.as_tensor(list(slots), dtype=torch.long, device=self.device)
        packed = torch.cat(
            [self._lengths.index_select(0, idx), self._n_blocks.index_select(0, idx), self._free_top, self._status]
        ).cpu()
        n = len(slots)
        vals = packed.numpy().astype(np.int64)
        self._h_len[list(slots)] = vals[:n]
        self._h_nb[list(slots)] = vals[n : 2 * n]
        self._h_top = int(vals[2 * n])
        self._stale.difference_update(int(s) for s in slots)
        if vals[2 * n + 1] != 0:
            self._raise_status()

    # ------------------------------------------------------------------ sequences
    def add_sequence(self, seq_id: int) -> None:
        if seq_id in self._slot_of:
            raise ValueError(f"sequence {seq_id} already exists")
        if not self._free_slots:
            self._grow_seqs()
        slot = self._free_slots.pop()
        self._slot_of[seq_id] = slot
        self._h_len[slot] = 0
        self._h_nb[slot] = 0

    def free_sequence(self, seq_id: int) -> None:
        """paged_cache.py:129-133: clear and free every block of the table, in table order."""
        slot = self._slot_of.pop(seq_id, None)
        if slot is None:
            return
        self.free_sequences_slots([slot])
        self._free_slots.append(slot)

    def free_sequences_slots(self, slots: Sequence[int]) -> None:
        if not slots:
            return
        stale = [s for s in slots if s in self._stale]
        if stale:  # the free count must not be credited with an upper bound of their blocks
            self._refresh(stale)
        b, keep = self._batch(slots)
        N.check(self._lib.kvs_release(C.byref(self._struct), C.byref(b), None, 1, self._stream()), "kvs_release")
        for s in slots:
            self._h_top += int(self._h_nb[s])
            self._h_len[s] = 0
            self._h_nb[s] = 0

    def has_sequence(self, seq_id: int) -> bool:
        return seq_id in self._slot_of

    def num_tokens(self, seq_id: int) -> int:
        slot = self._slot_of[seq_id]
        if slot in self._stale:
            self._refresh([slot])
        return int(self._h_len[slot])

    def slot(self, seq_id: int) -> int:
        return self._slot_of[seq_id]

    def block_table(self, seq_id: int) -> list[int]:
        slot = self._slot_of[seq_id]
        return self._tables[slot, : int(self._h_nb[slot])].tolist()

    def block_table_tensor(self, seq_id: int) -> torch.Tensor:
        slot = self._slot_of[seq_id]
        return self._tables[slot, : int(self._h_nb[slot])]

    # ------------------------------------------------------------------ batches
    def _batch(self, slots: Sequence[int], counts: Optional[Sequence[int]] = None):
        """kvs_batch over ``slots`` (in order); counts = new tokens per sequence."""
        slots = list(slots)
        if len(set(slots)) != len(slots):
            raise ValueError("a sequence appears twice in one batch")
        contiguous = slots == list(range(slots[0], slots[0] + len(slots))) if slots else True
        if contiguous:
            slot_t = self._slot_ids[slots[0] : slots[0] + len(slots)] if slots else self._slot_ids[:0]
        else:
            slot_t = N.to_device(slots, torch.int32, self.device)
        keep = [slot_t]
        cu_ptr = None
        total = len(slots)
        if counts is not None:
            cu = np.zeros(len(slots) + 1, dtype=np.int32)
            cu[1:] = np.cumsum(np.asarray(counts, dtype=np.int64))
            total = int(cu[-1])
            cu_t = N.to_device(cu, torch.int32, self.device)
            keep.append(cu_t)
            cu_ptr = cu_t.data_ptr()
        b = N.KvsBatch(seq_slots=slot_t.data_ptr(), cu_tokens=cu_ptr, num_seqs=len(slots), total_tokens=total)
        return b, keep

    # ------------------------------------------------------------------ writes
    def _check_alloc(self, slots: Sequence[int], counts: Sequence[int]) -> np.ndarray:
        try:
            return self._check_alloc_mirror(slots, counts)
        except OutOfBlocksError:
            if not self._stale:
                raise
            # the mirror is conservative after device-side evictions: re-read, then decide
            self._refresh(sorted(self._slot_of.values()))
            self._stale.clear()
            return self._check_alloc_mirror(slots, counts)

    def _check_alloc_mirror(self, slots: Sequence[int], counts: Sequence[int]) -> np.ndarray:
        bs = self.block_size
        s = np.asarray(slots, dtype=np.int64)
        n = self._h_len[s]
        nb = self._h_nb[s]
        need = np.maximum(-(-(n + np.asarray(counts, dtype=np.int64)) // bs) - nb, 0)
        total = int(need.sum())
        if total > self._h_top:
            # paged_cache.py:41-42
            raise OutOfBlocksError(f"all {self.num_blocks} KV blocks are in use")
        if np.any(nb + need > self.max_blocks):
            raise OutOfBlocksError(f"a block table would exceed max_blocks_per_seq={self.max_blocks}")
        return need

    def append_slots(self, seq_id: int, positions: torch.Tensor) -> SlotMapping:
        """paged_cache.py:145-165: reserve slots for len(positions) new tokens."""
        slot = self._slot_of[seq_id]
        return self._append([slot], [int(positions.numel())], positions)

    def append_slots_batch(self, seq_ids: Sequence[int], positions: torch.Tensor,
                           counts: Optional[Sequence[int]] = None) -> SlotMapping:
        """Batched append: ``positions`` concatenates each sequence's new positions in order;
        ``counts`` gives tokens per sequence (default one each)."""
        slots = [self._slot_of[s] for s in seq_ids]
        counts = [1] * len(slots) if counts is None else list(counts)
        return self._append(slots, counts, positions, one_each=counts is None or all(c == 1 for c in counts))

    def _append(self, slots, counts, positions, one_each: bool = False) -> SlotMapping:
        total = int(sum(counts))
        pos = positions.to(device=self.device, dtype=torch.long).reshape(-1).contiguous()
        if pos.numel() != total:
            raise ValueError("positions do not match the token counts")
        self._reserve(slots, counts)
        blocks = torch.empty(total, dtype=torch.int32, device=self.device)
        offsets = torch.empty(total, dtype=torch.int32, device=self.device)
        b, keep = self._batch(slots, None if one_each else counts)
        self.append_slots_device(b, pos, blocks, offsets)
        return SlotMapping(blocks, offsets)

    def _reserve(self, slots, counts) -> None:
        """Host half of an append: pool and table checks, then the host mirror's new lengths."""
        need = self._check_alloc(slots, counts)
        for s, c, k in zip(slots, counts, need):
            self._h_len[s] += c
            self._h_nb[s] += int(k)
        self._h_top -= int(need.sum())

    def reserve_slots(self, seq_ids: Sequence[int], counts: Optional[Sequence[int]] = None) -> None:
        """Host half of :meth:`append_slots_batch` for callers that launch the append kernel
        themselves (:meth:`append_slots_device`, e.g. inside a replayed CUDA graph)."""
        slots = [self._slot_of[s] for s in seq_ids]
        self._reserve(slots, [1] * len(slots) if counts is None else list(counts))

    def append_slots_device(self, batch, positions: torch.Tensor, blocks: torch.Tensor,
                            offsets: torch.Tensor) -> None:
        """Device half of an append: the append kernel on caller-provided buffers (``batch`` a
        kvs_batch whose arrays live on the device); no host work, so it can be graph-captured."""
        rc = self._lib.kvs_append_slots(C.byref(self._struct), C.byref(batch), positions.data_ptr(),
                                        blocks.data_ptr(), offsets.data_ptr(), self._stream())
        N.check(rc, "kvs_append_slots")

    def write(self, layer: int, slots: SlotMapping, k: torch.Tensor, v: torch.Tensor) -> None:
        """paged_cache.py:167-171: store already-rotated keys/values ``[T, n_kv_heads, head_dim]``."""
        k = k.to(self.dtype).contiguous()
        v = v.to(self.dtype).contiguous()
        rc = self._lib.kvs_write_kv(C.byref(self._struct), int(layer), slots.blocks.data_ptr(),
                                    slots.offsets.data_ptr(), k.data_ptr(), v.data_ptr(), int(k.shape[0]),
                                    self._stream())
        N.check(rc, "kvs_write_kv")

    # ------------------------------------------------------------------ reads
    def gather(self, seq_id: int, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """paged_cache.py:176-182: live keys/values in block-table order (a copy)."""
        n = self.num_tokens(seq_id)
        table = self.block_table_tensor(seq_id).long()
        k = self.k[layer].index_select(0, table).reshape(-1, self.n_kv_heads, self.head_dim)[:n]
        v = self.v[layer].index_select(0, table).reshape(-1, self.n_kv_heads, self.head_dim)[:n]
        return k, v

    def positions(self, seq_id: int) -> torch.Tensor:
        """paged_cache.py:184-188: logical positions of the live entries, in table order."""
        n = self.num_tokens(seq_id)
        table = self.block_table_tensor(seq_id).long()
        return self.slot_pos.index_select(0, table).reshape(-1)[:n]

    # ------------------------------------------------------------------ eviction
    def evict_blocks(self, seq_id: int, table_indices: Iterable[int]) -> int:
        """paged_cache.py:190-217: remove whole blocks by table index and join the rest."""
        return self.evict_blocks_batch([seq_id], [table_indices])[0]

    def evict_blocks_batch(self, seq_ids: Sequence[int], table_indices: Sequence[Iterable[int]]) -> list[int]:
        slots = [self._slot_of[s] for s in seq_ids]
        bs = self.block_size
        flags = np.zeros((len(slots), self.max_blocks), dtype=np.uint8)
        removed = []
        for r, (slot, idxs) in enumerate(zip(slots, table_indices)):
            idxs = sorted(set(int(i) for i in idxs))
            n_full = int(self._h_len[slot]) // bs
            for i in idxs:
                if not 0 <= i < n_full:
                    raise ValueError(f"block index {i} is not a full block (sequence has {n_full} full blocks)")
            flags[r, idxs] = 1
            removed.append(len(idxs) * bs)
        if not any(removed):
            return removed
        flags_t = torch.from_numpy(flags).to(self.device)
        b, keep = self._batch(slots)
        nbytes = self._lib.kvs_evict_scratch_bytes(len(slots), self.max_blocks)
        scratch = self._scratch_buf(nbytes)
        rc = self._lib.kvs_evict_blocks(C.byref(self._struct), C.byref(b), flags_t.data_ptr(), scratch.data_ptr(),
                                        scratch.numel(), self._stream())
        N.check(rc, "kvs_evict_blocks")
        for slot, rem in zip(slots, removed):
            self._h_len[slot] -= rem
            self._h_nb[slot] -= rem // bs
            self._h_top += rem // bs
        return removed

    def evict_positions(self, seq_id: int, spans: Iterable[Span], check: bool = False) -> list[Span]:
        """paged_cache.py:219-240: evict every full block whose tokens all lie in ``spans``;
        returns the logical spans actually removed.  ``check``: also run
        :meth:`check_invariants` on the sequence, read back with the eviction's results."""
        return self.evict_positions_batch([seq_id], [spans], check=check)[0]

    def evict_positions_batch(self, seq_ids: Sequence[int], spans: Sequence[Iterable[Span]],
                              check: bool = False) -> list[list[Span]]:
        """Batched evict_positions in canonical (given) order.  One device round trip: the
        evicted spans, the sequences' new lengths and table sizes, the free count, the status
        word and (with ``check``) the invariant codes of the evicted sequences come back in one
        read."""
        req = self.prepare_evict(seq_ids, spans)
        if req is None:
            return [[] for _ in seq_ids]
        self.evict_prepared(req)
        slots, n = req.slots, len(req.slots)
        idx = req.keep[0].long()  # the batch's slot ids, already on the device
        parts = [req.counts.long(), req.out.reshape(-1), self._lengths.index_select(0, idx).long(),
                 self._n_blocks.index_select(0, idx).long(), self._free_top.long(), self._status.long()]
        if check:
            parts.append(self._launch_check(req.batch).long())
        vals = torch.cat(parts).cpu().numpy()
        counts = vals[:n]
        spans_h = vals[n : n + n * req.cap * 2].reshape(n, req.cap, 2)
        o = n + n * req.cap * 2
        self._h_len[list(slots)] = vals[o : o + n]
        self._h_nb[list(slots)] = vals[o + n : o + 2 * n]
        self._h_top = int(vals[o + 2 * n])
        self._stale.difference_update(int(sl) for sl in slots)
        if vals[o + 2 * n + 1] != 0:
            self._raise_status()
        if check:
            for code in vals[o + 2 * n + 2 :].tolist():
                if code != N.ST_OK:
                    raise AssertionError(self._INV_MESSAGES.get(code, f"invariant {code} violated"))
        return [[(int(a), int(b)) for a, b in spans_h[i, : counts[i]]] for i in range(n)]

    def evict_positions_async(self, seq_ids: Sequence[int], spans: Sequence[Iterable[Span]],
                              span_cap: int = 0):
        """Launch the compaction kernels without waiting.  Returns (spans [S, cap, 2] int64,
        counts [S] int32, slots) as device tensors; the host mirror is marked stale until
        :meth:`refresh` (or any synchronising call) runs."""
        req = self.prepare_evict(seq_ids, spans, span_cap)
        if req is None:
            return None, None, [self._slot_of[s] for s in seq_ids]
        self.evict_prepared(req)
        return req.out, req.counts, req.slots

    def prepare_evict(self, seq_ids: Sequence[int], spans: Sequence[Iterable[Span]], span_cap: int = 0):
        """Upload an eviction request (merged spans per sequence) and its output buffers;
        :meth:`evict_prepared` then only launches kernels.  None when nothing can be evicted."""
        slots = [self._slot_of[s] for s in seq_ids]
        merged = [merge_spans(sp) for sp in spans]
        if not any(merged) or not any(self._h_len[s] for s in slots):
            return None
        # starts (int64), ends (int64) and the per-sequence prefix (int32) in one upload
        ns = sum(len(m) for m in merged)
        buf = np.zeros(16 * ns + 4 * (len(slots) + 1), dtype=np.uint8)
        flat = np.asarray([x for m in merged for x in m], dtype=np.int64).reshape(-1, 2)
        buf[: 8 * ns].view(np.int64)[:] = flat[:, 0]
        buf[8 * ns : 16 * ns].view(np.int64)[:] = flat[:, 1]
        np.cumsum([len(m) for m in merged], out=buf[16 * ns :].view(np.int32)[1:])
        cap = int(span_cap) or max(1, int(max(self._h_len[s] for s in slots)))
        dev = self.device
        b, keep = self._batch(slots)
        up = torch.from_numpy(buf).to(dev)
        return EvictRequest(
            slots=slots, batch=b, keep=keep + [up],
            cu=up[16 * ns :].view(torch.int32),
            starts=up[: 8 * ns].view(torch.int64),
            ends=up[8 * ns : 16 * ns].view(torch.int64),
            out=torch.empty((len(slots), cap, 2), dtype=torch.long, device=dev),
            counts=torch.empty(len(slots), dtype=torch.int32, device=dev),
            cap=cap,
        )

    def evict_prepared(self, req: "EvictRequest") -> None:
        """Launch the two compaction kernels of an uploaded request (no host work besides the call)."""
        nbytes = self._lib.kvs_evict_scratch_bytes(len(req.slots), self.max_blocks)
        scratch = self._scratch_buf(nbytes)
        rc = self._lib.kvs_evict_positions(C.byref(self._struct), C.byref(req.batch), req.cu.data_ptr(),
                                           req.starts.data_ptr(), req.ends.data_ptr(), req.out.data_ptr(),
                                           req.counts.data_ptr(), req.cap, scratch.data_ptr(), scratch.numel(),
                                           self._stream())
        N.check(rc, "kvs_evict_positions")

    def refresh(self, seq_ids: Optional[Sequence[int]] = None) -> None:
        slots = [self._slot_of[s] for s in (seq_ids if seq_ids is not None else list(self._slot_of))]
        if slots:
            self._refresh(slots)

    def truncate(self, seq_id: int, n_tokens: int) -> None:
        """paged_cache.py:242-260: drop the last ``n_tokens`` live entries."""
        if n_tokens <= 0:
            return
        slot = self._slot_of[seq_id]
        n = int(self._h_len[slot])
        if n_tokens > n:
            raise ValueError("cannot truncate more tokens than are live")
        new_len = n - n_tokens
        b, keep = self._batch([slot])
        nl = torch.tensor([new_len], dtype=torch.int32).to(self.device)
        N.check(self._lib.kvs_release(C.byref(self._struct), C.byref(b), nl.data_ptr(), 0, self._stream()),
                "kvs_release")
        keep_blocks = -(-new_len // self.block_size)
        self._h_top += int(self._h_nb[slot]) - keep_blocks
        self._h_nb[slot] = keep_blocks
        self._h_len[slot] = new_len

    # ------------------------------------------------------------------ checks
    _INV_MESSAGES = {
        N.ST_INV_DUP_BLOCK: "block table references a block twice",
        N.ST_INV_TABLE_LEN: "block table length does not match token count",
        N.ST_INV_HOLE: "live slot without a logical position (hole in block table)",
        N.ST_INV_ORDER: "logical positions are not strictly increasing",
    }

    def check_invariants(self, seq_id: int) -> None:
        """paged_cache.py:262-273, run by the device validation kernel."""
        self.check_invariants_batch([seq_id])

    def _launch_check(self, batch) -> torch.Tensor:
        """Launch the invariant check of ``batch``'s sequences; their codes, on the device."""
        codes = torch.empty(batch.num_seqs, dtype=torch.int32, device=self.device)
        nbytes = self._lib.kvs_check_scratch_bytes(self.num_blocks)
        scratch = self._scratch_buf(nbytes)
        rc = self._lib.kvs_check_invariants(C.byref(self._struct), C.byref(batch), codes.data_ptr(),
                                            scratch.data_ptr(), scratch.numel(), self._stream())
        N.check(rc, "kvs_check_invariants")
        return codes

    def check_invariants_batch(self, seq_ids: Sequence[int]) -> None:
        slots = [self._slot_of[s] for s in seq_ids]
        if not slots:
            return
        b, keep = self._batch(slots)
        codes = self._launch_check(b)
        for code in codes.cpu().tolist():
            if code != N.ST_OK:
                raise AssertionError(self._INV_MESSAGES.get(code, f"invariant {code} violated"))
        self._raise_status()

    # ------------------------------------------------------------------ set-up
    def load_state(self, seq_ids: Sequence[int], tables: Sequence[np.ndarray], positions: Sequence[np.ndarray],
                   free_list: np.ndarray) -> None:
        """Install block tables and logical positions directly (benchmark / test set-up).

        ``tables[i]`` are the block ids of sequence ``seq_ids[i]`` in order, ``positions[i]``
        its live tokens' logical positions; ``free_list`` the remaining blocks bottom to top.
        Every block must appear exactly once across tables and the free list."""
        all_blocks = np.concatenate([np.asarray(t, dtype=np.int64) for t in tables] + [np.asarray(free_list)])
        if all_blocks.size != self.num_blocks or np.unique(all_blocks).size != self.num_blocks:
            raise ValueError("tables and free list must partition the pool")
        dev = self.device
        bs = self.block_size
        for sid, tab, pos in zip(seq_ids, tables, positions):
            self.add_sequence(sid)
            slot = self._slot_of[sid]
            n = int(np.asarray(pos).size)
            if len(tab) != -(-n // bs):
                raise ValueError("table length does not match the token count")
            tt = torch.as_tensor(np.asarray(tab, dtype=np.int32)).to(dev)
            self._tables[slot, : len(tab)] = tt
            self._owner[tt.long()] = slot
            flat = torch.full((len(tab) * bs,), -1, dtype=torch.long)
            flat[:n] = torch.as_tensor(np.asarray(pos, dtype=np.int64))
            self.slot_pos[tt.long()] = flat.view(len(tab), bs).to(dev)
            self._h_len[slot] = n
            self._h_nb[slot] = len(tab)
        slots = [self._slot_of[s] for s in seq_ids]
        idx = torch.as_tensor(slots, dtype=torch.long, device=dev)
        self._lengths[idx] = torch.as_tensor(self._h_len[slots], dtype=torch.int32).to(dev)
        self._n_blocks[idx] = torch.as_tensor(self._h_nb[slots], dtype=torch.int32).to(dev)
        fl = np.asarray(free_list, dtype=np.int32)
        self._free_stack[: fl.size] = torch.as_tensor(fl).to(dev)
        self._free_top.fill_(int(fl.size))
        self._h_top = int(fl.size)
        used = self.num_blocks - int(fl.size)
        self._stats[N.STAT_FIELDS.index("peak_blocks")] = max(int(self._stats[4].item()), used)

    def snapshot_state(self) -> dict:
        """Device copies of every mutable tensor (restore with :meth:`restore_state`)."""
        names = ("slot_pos", "_tables", "_n_blocks", "_lengths", "_free_stack", "_free_top", "_owner", "_stats")
        return {"dev": {n: getattr(self, n).clone() for n in names},
                "host": (self._h_len.copy(), self._h_nb.copy(), self._h_top, set(self._stale))}

    def restore_state(self, snap: dict) -> None:
        for n, t in snap["dev"].items():
            getattr(self, n).copy_(t)
        self._h_len[:], self._h_nb[:], self._h_top = snap["host"][0], snap["host"][1], snap["host"][2]
        self._stale = set(snap["host"][3])

    # ------------------------------------------------------------------ stats
    @property
    def stats(self) -> CacheStats:
        """CacheStats read from the device counters (paged_cache.py:70-78)."""
        vals = self._stats.tolist()
        return CacheStats(**{f.name: int(vals[i]) for i, f in enumerate(fields(CacheStats))})

    def lengths_tensor(self) -> torch.Tensor:
        return self._lengths
