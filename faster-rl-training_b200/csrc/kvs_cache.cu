// Device-resident paged KV cache: allocator, block tables, whole-block eviction
// (stream compaction), truncation, invariant checks and the evicted_at map.
//
// Reference: kvstreams/paged_cache.py (PagedKVCache, BlockAllocator) and
// kvstreams/compaction/events.py (CompactionLog.evicted_at).  Every batched call
// reproduces, bit for bit, the state the reference reaches when its
// single-sequence method is called once per sequence in batch order.
#include "kvs_common.cuh"

#include <algorithm>

using namespace kvs;

namespace {

__device__ __forceinline__ int batch_cu(const kvs_batch& b, int i) {
  return b.cu_tokens ? b.cu_tokens[i] : i;
}

// ------------------------------------------------------------------ reset
__global__ void reset_kernel(kvs_cache c) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t nslots = (int64_t)c.num_blocks * c.block_size;
  for (int64_t i = tid; i < nslots; i += stride) c.slot_pos[i] = -1;
  for (int64_t i = tid; i < c.num_blocks; i += stride) {
    // paged_cache.py:37 -- _free = [NB-1, ..., 0]; the end of the list is popped first.
    c.free_stack[i] = c.num_blocks - 1 - (int32_t)i;
    c.block_owner[i] = -1;
  }
  const int64_t ntab = (int64_t)c.max_seqs * c.max_blocks;
  for (int64_t i = tid; i < ntab; i += stride) c.tables[i] = -1;
  for (int64_t i = tid; i < c.max_seqs; i += stride) {
    c.n_blocks[i] = 0;
    c.lengths[i] = 0;
  }
  if (tid < KVS_STAT_COUNT) c.stats[tid] = 0;
  if (tid < KVS_STATUS_WORDS) c.status[tid] = 0;
  if (tid == 0) *c.free_top = c.num_blocks;
}

// ------------------------------------------------------------------ append_slots
// One CTA: the allocation order is a prefix sum over the batch (canonical order).
constexpr int kAppendThreads = 1024;

// The decode step's append (one new token per sequence, at most kAppendThreads sequences): a
// thread per sequence, every value loaded once and kept in registers, the token's slot taken
// from the table entry it already has or from the block it pops.  Same allocation order,
// checks and status words as append_slots_kernel, in fewer dependent global round trips.
__global__ void __launch_bounds__(kAppendThreads)
append_one_kernel(kvs_cache c, kvs_batch b, const int64_t* __restrict__ positions,
                  int32_t* __restrict__ out_blocks, int32_t* __restrict__ out_offsets) {
  __shared__ int s_scan[33];
  __shared__ long long s_red[32];
  const int tid = threadIdx.x, bs = c.block_size;
  const int top = *c.free_top;  // read by every thread before the first barrier; written last
  const bool valid = tid < b.num_seqs;
  int slot = 0, n = 0, nb = 0, need = 0, tab = -1;
  int64_t pos = 0;
  if (valid) {
    slot = b.seq_slots[tid];
    pos = positions[tid];
    n = c.lengths[slot];
    nb = c.n_blocks[slot];
    need = n / bs + 1 - nb;  // ceil_div(n + 1, bs) - nb
    need = need < 0 ? 0 : need;
    if (need == 0) tab = c.tables[(int64_t)slot * c.max_blocks + n / bs];
  }
  const int over = valid && nb + need > c.max_blocks;
  int total = 0;
  const int off = block_exclusive_scan(need, s_scan, &total);
  // the batch must fit as a whole (no partial state on failure)
  if (total > top) {
    if (tid == 0) set_status(c.status, KVS_ST_OUT_OF_BLOCKS, total, top, 0);
    return;
  }
  if (__syncthreads_or(over)) {
    const long long overflow = block_sum_ll(over, s_red);
    if (tid == 0) set_status(c.status, KVS_ST_TABLE_OVERFLOW, (int)overflow, c.max_blocks, 0);
    return;
  }
  if (valid) {
    // paged_cache.py:152-155 -- a block is taken from the end of the free list whenever the
    // token index reaches a new table entry
    int blk_tok = tab;
    for (int k = 0; k < need; ++k) {
      const int blk = c.free_stack[top - 1 - (off + k)];
      c.tables[(int64_t)slot * c.max_blocks + nb + k] = blk;
      if (c.block_owner[blk] != -1) set_status(c.status, KVS_ST_OWNER, blk, slot, c.block_owner[blk]);
      c.block_owner[blk] = slot;
      if (nb + k == n / bs) blk_tok = blk;
    }
    c.n_blocks[slot] = nb + need;
    // paged_cache.py:152,161 -- slot of token n is (table[n // bs], n % bs)
    const int o = n % bs;
    c.slot_pos[(int64_t)blk_tok * bs + o] = pos;
    out_blocks[tid] = blk_tok;
    out_offsets[tid] = o;
    c.lengths[slot] = n + 1;
  }
  if (tid == 0) {
    const int new_top = top - total;
    *c.free_top = new_top;
    c.stats[KVS_STAT_WRITTEN_TOKENS] += b.total_tokens;
    const long long used = c.num_blocks - new_top;  // paged_cache.py:164
    if (used > c.stats[KVS_STAT_PEAK_BLOCKS]) c.stats[KVS_STAT_PEAK_BLOCKS] = used;
  }
}

__global__ void __launch_bounds__(kAppendThreads)
append_slots_kernel(kvs_cache c, kvs_batch b, const int64_t* __restrict__ positions,
                    int32_t* __restrict__ out_blocks, int32_t* __restrict__ out_offsets) {
  __shared__ int s_scan[33];
  __shared__ int s_n[kAppendThreads], s_slot[kAppendThreads], s_cu[kAppendThreads + 1];
  __shared__ long long s_red[32];
  __shared__ int s_top;
  const int tid = threadIdx.x, bs = c.block_size;
  if (tid == 0) s_top = *c.free_top;
  __syncthreads();
  const int top = s_top;

  // Pass 1: the batch must fit as a whole (no partial state on failure).
  long long need_local = 0, overflow_local = 0;
  for (int i = tid; i < b.num_seqs; i += blockDim.x) {
    const int slot = b.seq_slots[i];
    const int n = c.lengths[slot], nb = c.n_blocks[slot];
    const int T = batch_cu(b, i + 1) - batch_cu(b, i);
    int need = ceil_div(n + T, bs) - nb;
    need = need < 0 ? 0 : need;
    need_local += need;
    if (nb + need > c.max_blocks) overflow_local += 1;
  }
  const long long need_total = block_sum_ll(need_local, s_red);
  const long long overflow = block_sum_ll(overflow_local, s_red);
  if (need_total > top) {
    if (tid == 0) set_status(c.status, KVS_ST_OUT_OF_BLOCKS, (int)need_total, top, 0);
    return;
  }
  if (overflow) {
    if (tid == 0) set_status(c.status, KVS_ST_TABLE_OVERFLOW, (int)overflow, c.max_blocks, 0);
    return;
  }

  int carry = 0;  // blocks popped by earlier chunks
  for (int base = 0; base < b.num_seqs; base += blockDim.x) {
    const int i = base + tid;
    const bool valid = i < b.num_seqs;
    int slot = 0, n = 0, nb = 0, T = 0, need = 0;
    if (valid) {
      slot = b.seq_slots[i];
      n = c.lengths[slot];
      nb = c.n_blocks[slot];
      T = batch_cu(b, i + 1) - batch_cu(b, i);
      need = ceil_div(n + T, bs) - nb;
      need = need < 0 ? 0 : need;
      s_n[tid] = n;
      s_slot[tid] = slot;
      s_cu[tid] = batch_cu(b, i) - batch_cu(b, base);
    }
    const int chunk_n = min((int)blockDim.x, b.num_seqs - base);
    if (tid == 0) s_cu[chunk_n] = batch_cu(b, base + chunk_n) - batch_cu(b, base);
    int chunk_total = 0;
    const int off = block_exclusive_scan(need, s_scan, &chunk_total);
    if (valid) {
      // paged_cache.py:152-155 -- a block is taken from the end of the free list
      // whenever the token index reaches a new table entry.
      for (int k = 0; k < need; ++k) {
        const int blk = c.free_stack[top - 1 - (carry + off + k)];
        c.tables[(int64_t)slot * c.max_blocks + nb + k] = blk;
        if (c.block_owner[blk] != -1) set_status(c.status, KVS_ST_OWNER, blk, slot, c.block_owner[blk]);
        c.block_owner[blk] = slot;
      }
      c.n_blocks[slot] = nb + need;
    }
    __syncthreads();
    // paged_cache.py:152,161 -- slot of token n+i is (table[(n+i)//bs], (n+i)%bs).
    const int tok0 = batch_cu(b, base);
    const int ntok = s_cu[chunk_n];
    for (int j = tid; j < ntok; j += blockDim.x) {
      int lo = 0, hi = chunk_n - 1;  // last r with s_cu[r] <= j
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_cu[mid] <= j) lo = mid; else hi = mid - 1;
      }
      const int idx = s_n[lo] + (j - s_cu[lo]);
      const int blk = c.tables[(int64_t)s_slot[lo] * c.max_blocks + idx / bs];
      const int o = idx % bs;
      c.slot_pos[(int64_t)blk * bs + o] = positions[tok0 + j];
      out_blocks[tok0 + j] = blk;
      out_offsets[tok0 + j] = o;
    }
    __syncthreads();
    if (valid) c.lengths[slot] = n + T;
    carry += chunk_total;
    __syncthreads();
  }
  if (tid == 0) {
    const int new_top = top - carry;
    *c.free_top = new_top;
    c.stats[KVS_STAT_WRITTEN_TOKENS] += b.total_tokens;
    const long long used = c.num_blocks - new_top;  // paged_cache.py:164
    if (used > c.stats[KVS_STAT_PEAK_BLOCKS]) c.stats[KVS_STAT_PEAK_BLOCKS] = used;
  }
}

// ------------------------------------------------------------------ write_kv
__global__ void write_kv_kernel(kvs_cache c, int layer, const int32_t* __restrict__ blocks,
                                const int32_t* __restrict__ offsets, const uint8_t* __restrict__ k,
                                const uint8_t* __restrict__ v, int n_tokens, int row_bytes) {
  // one 16-byte (or 4-byte) word per thread; rows are contiguous in source and pool
  const int vec = (row_bytes % 16 == 0) ? 16 : 4;
  const int words = row_bytes / vec;
  const int64_t total = (int64_t)n_tokens * words;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total;
       w += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(w / words), x = (int)(w % words);
    const int64_t row = ((int64_t)layer * c.num_blocks + blocks[t]) * c.block_size + offsets[t];
    uint8_t* dk = reinterpret_cast<uint8_t*>(c.k) + row * row_bytes + (int64_t)x * vec;
    uint8_t* dv = reinterpret_cast<uint8_t*>(c.v) + row * row_bytes + (int64_t)x * vec;
    const int64_t so = (int64_t)t * row_bytes + (int64_t)x * vec;
    if (vec == 16) {
      *reinterpret_cast<int4*>(dk) = *reinterpret_cast<const int4*>(k + so);
      *reinterpret_cast<int4*>(dv) = *reinterpret_cast<const int4*>(v + so);
    } else {
      *reinterpret_cast<int*>(dk) = *reinterpret_cast<const int*>(k + so);
      *reinterpret_cast<int*>(dv) = *reinterpret_cast<const int*>(v + so);
    }
  }
}

// ------------------------------------------------------------------ eviction
// Scratch layout shared by the two eviction kernels.
struct EvictScratch {
  int32_t* top_snapshot;  // [1] free_top before the call
  int32_t* counts;        // [num_seqs][2] = {blocks dropped, tokens covered}
  uint8_t* flags;         // [num_seqs][max_blocks] 1 = drop
  int32_t* dropped;       // [num_seqs][max_blocks] dropped block ids, table order
};

__host__ __device__ inline size_t evict_scratch_layout(int num_seqs, int max_blocks, void* base,
                                                       EvictScratch* out) {
  size_t off = 0;
  const size_t a = 256;
  size_t o_top = off; off = align_up(off + 4, a);
  size_t o_cnt = off; off = align_up(off + (size_t)8 * num_seqs, a);
  size_t o_flg = off; off = align_up(off + (size_t)num_seqs * max_blocks, a);
  size_t o_drp = off; off = align_up(off + (size_t)4 * num_seqs * max_blocks, a);
  if (out) {
    uint8_t* p = reinterpret_cast<uint8_t*>(base);
    out->top_snapshot = reinterpret_cast<int32_t*>(p + o_top);
    out->counts = reinterpret_cast<int32_t*>(p + o_cnt);
    out->flags = p + o_flg;
    out->dropped = reinterpret_cast<int32_t*>(p + o_drp);
  }
  return off;
}

// covered(p): p inside one of the sorted, disjoint spans [lo, hi).
__device__ __forceinline__ bool in_spans(int64_t p, const int64_t* __restrict__ ss,
                                         const int64_t* __restrict__ se, int lo, int hi) {
  // last span with start <= p
  if (lo >= hi || p < ss[lo]) return false;
  int a = lo, z = hi - 1;
  while (a < z) {
    const int mid = (a + z + 1) >> 1;
    if (ss[mid] <= p) a = mid; else z = mid - 1;
  }
  return p < se[a];
}

constexpr int kEvictThreads = 256;

// Kernel A of evict_positions: per sequence, which full blocks are entirely covered
// (paged_cache.py:230-236) and how many live tokens are covered (:238).
__global__ void __launch_bounds__(kEvictThreads)
evict_mark_kernel(kvs_cache c, kvs_batch b, const int32_t* __restrict__ cu_spans,
                  const int64_t* __restrict__ span_start, const int64_t* __restrict__ span_end,
                  const uint8_t* __restrict__ given_flags, EvictScratch s) {
  __shared__ long long s_red[32];
  const int i = blockIdx.x;
  const int slot = b.seq_slots[i];
  const int bs = c.block_size;
  const int n = c.lengths[slot], nb = c.n_blocks[slot], n_full = n / bs;
  const int32_t* table = c.tables + (int64_t)slot * c.max_blocks;
  uint8_t* flags = s.flags + (int64_t)i * c.max_blocks;
  if (i == 0 && threadIdx.x == 0) *s.top_snapshot = *c.free_top;
  long long cov_local = 0, drop_local = 0;
  if (given_flags) {
    // evict_blocks: the caller chose the table indices (already validated as full blocks).
    const uint8_t* g = given_flags + (int64_t)i * c.max_blocks;
    for (int j = threadIdx.x; j < nb; j += blockDim.x) {
      const uint8_t d = (j < n_full) ? g[j] : 0;
      flags[j] = d;
      drop_local += d;
    }
    cov_local = drop_local * bs;
  } else {
    const int lo = cu_spans[i], hi = cu_spans[i + 1];
    for (int j = threadIdx.x; j < nb; j += blockDim.x) {
      const int64_t blk = table[j];
      const int ntok = min(bs, n - j * bs);
      int cov = 0;
      if (hi > lo) {
        const int64_t* sp = c.slot_pos + blk * bs;
        for (int o = 0; o < ntok; ++o) cov += in_spans(sp[o], span_start, span_end, lo, hi);
      }
      const uint8_t d = (j < n_full && cov == bs) ? 1 : 0;
      flags[j] = d;
      cov_local += cov;
      drop_local += d;
    }
  }
  const long long cov = block_sum_ll(cov_local, s_red);
  const long long drop = block_sum_ll(drop_local, s_red);
  if (threadIdx.x == 0) {
    s.counts[2 * i] = (int)drop;
    s.counts[2 * i + 1] = (int)cov;
  }
}

// Kernel B: join each table (stream compaction of the kept entries), push the
// dropped blocks on the free stack in canonical order, write the removed logical
// spans, reset slot_pos of freed blocks and update lengths / stats
// (paged_cache.py:207-217 and :237-240).
__global__ void __launch_bounds__(kEvictThreads)
evict_apply_kernel(kvs_cache c, kvs_batch b, EvictScratch s, int64_t* __restrict__ out_spans,
                   int32_t* __restrict__ out_counts, int span_cap) {
  __shared__ int s_scan[33];
  __shared__ long long s_red[32];
  const int i = blockIdx.x, tid = threadIdx.x;
  const int slot = b.seq_slots[i];
  const int bs = c.block_size;
  const int n = c.lengths[slot], nb = c.n_blocks[slot];
  int32_t* table = c.tables + (int64_t)slot * c.max_blocks;
  const uint8_t* flags = s.flags + (int64_t)i * c.max_blocks;
  int32_t* dropped = s.dropped + (int64_t)i * c.max_blocks;
  const int top0 = *s.top_snapshot;

  // Offset of this sequence's first push: blocks dropped by earlier sequences.
  long long before_local = 0;
  for (int k = tid; k < i; k += blockDim.x) before_local += s.counts[2 * k];
  const int before = (int)block_sum_ll(before_local, s_red);
  const int n_drop = s.counts[2 * i], covered = s.counts[2 * i + 1];

  if (n_drop > 0) {
    int keep_carry = 0, drop_carry = 0;
    for (int base = 0; base < nb; base += blockDim.x) {
      const int j = base + tid;
      const bool valid = j < nb;
      const int blk = valid ? table[j] : -1;
      const int d = valid ? flags[j] : 0;
      const int keep = (valid && !d) ? 1 : 0;
      int tot = 0;
      const int pre = block_exclusive_scan(keep | (d << 16), s_scan, &tot);
      if (keep) table[keep_carry + (pre & 0xffff)] = blk;
      if (d) {
        const int r = drop_carry + (pre >> 16);
        dropped[r] = blk;
        // paged_cache.py:47-51 -- free(): the block must be in use (by this sequence).
        const int owner = c.block_owner[blk];
        if (owner != slot)
          set_status(c.status, owner == -1 ? KVS_ST_DOUBLE_FREE : KVS_ST_OWNER, blk, slot, owner);
        c.block_owner[blk] = -1;
        c.free_stack[top0 + before + r] = blk;
      }
      keep_carry += tot & 0xffff;
      drop_carry += tot >> 16;
    }
    __syncthreads();

    // Removed positions in table order are strictly increasing; positions_to_spans
    // merges runs of consecutive positions (utils/spans.py:10-23).
    const int nrem = n_drop * bs;
    int start_carry = 0, end_carry = 0;
    for (int base = 0; out_spans && base < nrem; base += blockDim.x) {
      const int u = base + tid;
      int is_start = 0, is_end = 0;
      int64_t p = 0;
      if (u < nrem) {
        const int r = u / bs, o = u % bs;
        p = c.slot_pos[(int64_t)dropped[r] * bs + o];
        int64_t prev = 0, next = 0;
        if (u > 0)
          prev = (o > 0) ? c.slot_pos[(int64_t)dropped[r] * bs + o - 1]
                         : c.slot_pos[(int64_t)dropped[r - 1] * bs + bs - 1];
        if (u + 1 < nrem)
          next = (o + 1 < bs) ? c.slot_pos[(int64_t)dropped[r] * bs + o + 1]
                              : c.slot_pos[(int64_t)dropped[r + 1] * bs];
        is_start = (u == 0) || (prev != p - 1);
        is_end = (u + 1 == nrem) || (next != p + 1);
      }
      int tot = 0;
      const int pre = block_exclusive_scan(is_start | (is_end << 16), s_scan, &tot);
      if (is_start) {
        const int k = start_carry + (pre & 0xffff);
        if (k < span_cap) out_spans[2 * ((int64_t)i * span_cap + k)] = p;
        else set_status(c.status, KVS_ST_SPAN_CAPACITY, i, k, span_cap);
      }
      if (is_end) {
        const int k = end_carry + (pre >> 16);
        if (k < span_cap) out_spans[2 * ((int64_t)i * span_cap + k) + 1] = p + 1;
      }
      start_carry += tot & 0xffff;
      end_carry += tot >> 16;
    }
    __syncthreads();
    // paged_cache.py:209 -- slot_pos[table[i]] = -1 for every freed block.
    for (int u = tid; u < nrem; u += blockDim.x)
      c.slot_pos[(int64_t)dropped[u / bs] * bs + (u % bs)] = -1;
    if (tid == 0) {
      c.n_blocks[slot] = nb - n_drop;
      c.lengths[slot] = n - n_drop * bs;
      if (out_counts) out_counts[i] = min(start_carry, span_cap);
      atomicAdd(reinterpret_cast<unsigned long long*>(&c.stats[KVS_STAT_EVICTED_BLOCKS]),
                (unsigned long long)n_drop);
      atomicAdd(reinterpret_cast<unsigned long long*>(&c.stats[KVS_STAT_EVICTED_TOKENS]),
                (unsigned long long)nrem);
      atomicAdd(reinterpret_cast<unsigned long long*>(&c.stats[KVS_STAT_EVICTION_CALLS]), 1ull);
    }
  } else if (tid == 0 && out_counts) {
    out_counts[i] = 0;
  }
  if (tid == 0) {
    const long long shrunk = (long long)covered - (long long)n_drop * bs;
    if (shrunk)
      atomicAdd(reinterpret_cast<unsigned long long*>(&c.stats[KVS_STAT_SHRUNK_TOKENS]),
                (unsigned long long)shrunk);
    if (i == b.num_seqs - 1) *c.free_top = top0 + before + n_drop;
  }
}

// ------------------------------------------------------------------ truncate / free
constexpr int kReleaseThreads = 1024;

__global__ void __launch_bounds__(kReleaseThreads)
release_kernel(kvs_cache c, kvs_batch b, const int32_t* __restrict__ new_lengths, int mode) {
  __shared__ int s_scan[33];
  __shared__ int s_top;
  const int tid = threadIdx.x, bs = c.block_size;
  if (tid == 0) s_top = *c.free_top;
  __syncthreads();
  const int top = s_top;
  int carry = 0;
  for (int base = 0; base < b.num_seqs; base += blockDim.x) {
    const int i = base + tid;
    const bool valid = i < b.num_seqs;
    int slot = 0, n = 0, nb = 0, new_len = 0, nfree = 0, keep_blocks = 0;
    if (valid) {
      slot = b.seq_slots[i];
      n = c.lengths[slot];
      nb = c.n_blocks[slot];
      new_len = mode == 1 ? 0 : new_lengths[i];
      if (mode == 0 && (new_len > n || new_len < 0)) {
        set_status(c.status, KVS_ST_TRUNCATE, slot, new_len, n);
        new_len = n;  // leave the sequence untouched
      }
      keep_blocks = mode == 1 ? 0 : ceil_div(new_len, bs);
      if (mode == 0 && new_len == n) keep_blocks = nb;  // truncate(<=0) is a no-op
      nfree = nb - keep_blocks;
      if (nfree < 0) nfree = 0;
    }
    int tot = 0;
    const int off = block_exclusive_scan(nfree, s_scan, &tot);
    if (valid) {
      const int32_t* table = c.tables + (int64_t)slot * c.max_blocks;
      if (mode == 1) {
        // paged_cache.py:130-132 -- every block of the table is cleared and freed in order.
        for (int j = 0; j < nb; ++j)
          for (int o = 0; o < bs; ++o) c.slot_pos[(int64_t)table[j] * bs + o] = -1;
      } else {
        // paged_cache.py:252-254 -- only the truncated tokens lose their position.
        for (int t = new_len; t < n; ++t) c.slot_pos[(int64_t)table[t / bs] * bs + t % bs] = -1;
      }
      for (int k = 0; k < nfree; ++k) {
        const int blk = table[keep_blocks + k];
        const int owner = c.block_owner[blk];
        if (owner != slot)
          set_status(c.status, owner == -1 ? KVS_ST_DOUBLE_FREE : KVS_ST_OWNER, blk, slot, owner);
        c.block_owner[blk] = -1;
        c.free_stack[top + carry + off + k] = blk;
      }
      c.n_blocks[slot] = keep_blocks;
      c.lengths[slot] = new_len;
      if (mode == 0 && n > new_len)
        atomicAdd(reinterpret_cast<unsigned long long*>(&c.stats[KVS_STAT_TRUNCATED_TOKENS]),
                  (unsigned long long)(n - new_len));
    }
    carry += tot;
    __syncthreads();
  }
  if (tid == 0) *c.free_top = top + carry;
}

// ------------------------------------------------------------------ invariants
__global__ void __launch_bounds__(256)
check_kernel(kvs_cache c, kvs_batch b, int32_t* __restrict__ out_codes, uint32_t* __restrict__ seen) {
  __shared__ int s_flags;
  const int i = blockIdx.x, tid = threadIdx.x, bs = c.block_size;
  const int slot = b.seq_slots[i];
  const int n = c.lengths[slot], nb = c.n_blocks[slot];
  const int32_t* table = c.tables + (int64_t)slot * c.max_blocks;
  if (tid == 0) s_flags = 0;
  __syncthreads();
  int f = 0;
  for (int j = tid; j < nb; j += blockDim.x) {
    const int blk = table[j];
    const uint32_t bit = 1u << (blk & 31);
    if (atomicOr(&seen[blk >> 5], bit) & bit) f |= 1;  // paged_cache.py:265
  }
  const bool len_ok = nb == ceil_div(n, bs);  // paged_cache.py:267
  if (!len_ok) f |= 2;
  if (len_ok) {
    for (int t = tid; t < n; t += blockDim.x) {
      const int64_t p = c.slot_pos[(int64_t)table[t / bs] * bs + t % bs];
      if (p < 0) f |= 4;  // paged_cache.py:270
      if (t > 0) {
        const int64_t q = c.slot_pos[(int64_t)table[(t - 1) / bs] * bs + (t - 1) % bs];
        if (!(p > q)) f |= 8;  // paged_cache.py:272
      }
    }
  }
  if (f) atomicOr(&s_flags, f);
  __syncthreads();
  if (tid == 0) {
    const int g = s_flags;
    out_codes[i] = (g & 1) ? KVS_ST_INV_DUP_BLOCK
                 : (g & 2) ? KVS_ST_INV_TABLE_LEN
                 : (g & 4) ? KVS_ST_INV_HOLE
                 : (g & 8) ? KVS_ST_INV_ORDER : KVS_ST_OK;
  }
}

// ------------------------------------------------------------------ evicted_at
__global__ void evicted_at_kernel(const int32_t* __restrict__ cu_spans, const int64_t* __restrict__ ss,
                                  const int64_t* __restrict__ se, const int64_t* __restrict__ st,
                                  const int32_t* __restrict__ lengths, int t_stride,
                                  int64_t* __restrict__ out) {
  const int b = blockIdx.y;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= t_stride) return;
  const int len = lengths[b];
  int64_t v = kNever;
  if (t < len) {
    // events.py:69-73 -- out[s:min(e,length)] = min(out, time)
    for (int j = cu_spans[b]; j < cu_spans[b + 1]; ++j)
      if (ss[j] <= t && t < se[j] && st[j] < v) v = st[j];
  }
  out[(int64_t)b * t_stride + t] = v;
}

}  // namespace

// ====================================================================== C ABI

KVS_API int kvs_cache_reset(const kvs_cache* c, kvs_stream_t stream) {
  if (!c || !c->slot_pos || !c->free_stack || !c->free_top || c->num_blocks <= 0 || c->block_size <= 0)
    return KVS_E_ARG;
  const int64_t work = (int64_t)c->num_blocks * c->block_size;
  int grid = (int)std::min<int64_t>((work + 255) / 256, 148 * 8);
  if (grid < 1) grid = 1;
  reset_kernel<<<grid, 256, 0, to_cuda(stream)>>>(*c);
  return launch_rc();
}

KVS_API int kvs_append_slots(const kvs_cache* c, const kvs_batch* b, const int64_t* positions,
                             int32_t* out_blocks, int32_t* out_offsets, kvs_stream_t stream) {
  if (!c || !b || b->num_seqs < 0 || b->total_tokens < 0) return KVS_E_ARG;
  if (b->num_seqs == 0) return KVS_OK;
  if (b->total_tokens > 0 && (!positions || !out_blocks || !out_offsets)) return KVS_E_ARG;
  if (b->cu_tokens == nullptr && b->total_tokens == b->num_seqs && b->num_seqs <= kAppendThreads)
    append_one_kernel<<<1, kAppendThreads, 0, to_cuda(stream)>>>(*c, *b, positions, out_blocks, out_offsets);
  else
    append_slots_kernel<<<1, kAppendThreads, 0, to_cuda(stream)>>>(*c, *b, positions, out_blocks,
                                                                   out_offsets);
  return launch_rc();
}

KVS_API int kvs_write_kv(const kvs_cache* c, int32_t layer, const int32_t* blocks, const int32_t* offsets,
                         const void* k, const void* v, int32_t n_tokens, kvs_stream_t stream) {
  if (!c || layer < 0 || layer >= c->n_layers || n_tokens < 0) return KVS_E_ARG;
  if (n_tokens == 0) return KVS_OK;
  const int es = c->dtype == KVS_F64 ? 8 : c->dtype == KVS_F32 ? 4 : 2;
  const int row_bytes = c->n_kv_heads * c->head_dim * es;
  if (row_bytes % 4) return KVS_E_UNSUPPORTED;
  const int vec = row_bytes % 16 == 0 ? 16 : 4;
  const int64_t total = (int64_t)n_tokens * (row_bytes / vec);
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  write_kv_kernel<<<grid, 256, 0, to_cuda(stream)>>>(*c, layer, blocks, offsets,
                                                     static_cast<const uint8_t*>(k),
                                                     static_cast<const uint8_t*>(v), n_tokens, row_bytes);
  return launch_rc();
}

KVS_API size_t kvs_evict_scratch_bytes(int32_t num_seqs, int32_t max_blocks) {
  return evict_scratch_layout(num_seqs, max_blocks, nullptr, nullptr);
}

static int evict_common(const kvs_cache* c, const kvs_batch* b, const int32_t* cu_spans,
                        const int64_t* ss, const int64_t* se, const uint8_t* given, int64_t* out_spans,
                        int32_t* out_counts, int32_t span_cap, void* scratch, size_t scratch_bytes,
                        kvs_stream_t stream) {
  if (!c || !b || b->num_seqs < 0) return KVS_E_ARG;
  if (b->num_seqs == 0) return KVS_OK;
  EvictScratch s;
  const size_t need = evict_scratch_layout(b->num_seqs, c->max_blocks, scratch, &s);
  if (!scratch || scratch_bytes < need) return KVS_E_SCRATCH;
  evict_mark_kernel<<<b->num_seqs, kEvictThreads, 0, to_cuda(stream)>>>(*c, *b, cu_spans, ss, se, given, s);
  int rc = launch_rc();
  if (rc) return rc;
  evict_apply_kernel<<<b->num_seqs, kEvictThreads, 0, to_cuda(stream)>>>(*c, *b, s, out_spans, out_counts,
                                                                        span_cap);
  return launch_rc();
}

KVS_API int kvs_evict_positions(const kvs_cache* c, const kvs_batch* b, const int32_t* cu_spans,
                                const int64_t* span_start, const int64_t* span_end, int64_t* out_spans,
                                int32_t* out_counts, int32_t span_cap, void* scratch, size_t scratch_bytes,
                                kvs_stream_t stream) {
  if (!cu_spans || !out_spans || !out_counts || span_cap <= 0) return KVS_E_ARG;
  return evict_common(c, b, cu_spans, span_start, span_end, nullptr, out_spans, out_counts, span_cap,
                      scratch, scratch_bytes, stream);
}

KVS_API int kvs_evict_blocks(const kvs_cache* c, const kvs_batch* b, const uint8_t* drop_flags,
                             void* scratch, size_t scratch_bytes, kvs_stream_t stream) {
  if (!drop_flags) return KVS_E_ARG;
  // evict_blocks (paged_cache.py:190-217) returns a token count, not spans: no span pass.
  return evict_common(c, b, nullptr, nullptr, nullptr, drop_flags, nullptr, nullptr, 0, scratch,
                      scratch_bytes, stream);
}

KVS_API int kvs_release(const kvs_cache* c, const kvs_batch* b, const int32_t* new_lengths, int32_t mode,
                        kvs_stream_t stream) {
  if (!c || !b || (mode != 0 && mode != 1) || (mode == 0 && !new_lengths)) return KVS_E_ARG;
  if (b->num_seqs == 0) return KVS_OK;
  release_kernel<<<1, kReleaseThreads, 0, to_cuda(stream)>>>(*c, *b, new_lengths, mode);
  return launch_rc();
}

KVS_API size_t kvs_check_scratch_bytes(int32_t num_blocks) {
  return align_up((size_t)((num_blocks + 31) / 32) * 4, 256);
}

KVS_API int kvs_check_invariants(const kvs_cache* c, const kvs_batch* b, int32_t* out_codes, void* scratch,
                                 size_t scratch_bytes, kvs_stream_t stream) {
  if (!c || !b || !out_codes) return KVS_E_ARG;
  if (b->num_seqs == 0) return KVS_OK;
  const size_t need = kvs_check_scratch_bytes(c->num_blocks);
  if (!scratch || scratch_bytes < need) return KVS_E_SCRATCH;
  if (cudaMemsetAsync(scratch, 0, need, to_cuda(stream)) != cudaSuccess) return KVS_E_LAUNCH;
  check_kernel<<<b->num_seqs, 256, 0, to_cuda(stream)>>>(*c, *b, out_codes, static_cast<uint32_t*>(scratch));
  return launch_rc();
}

KVS_API int kvs_evicted_at(const int32_t* cu_spans, const int64_t* span_start, const int64_t* span_end,
                           const int64_t* span_time, const int32_t* lengths, int32_t num_streams,
                           int32_t t_stride, int64_t* out, kvs_stream_t stream) {
  if (!cu_spans || !lengths || !out || num_streams < 0 || t_stride < 0 || num_streams > 65535)
    return KVS_E_ARG;
  if (num_streams == 0 || t_stride == 0) return KVS_OK;
  dim3 grid((t_stride + 255) / 256, num_streams);
  evicted_at_kernel<<<grid, 256, 0, to_cuda(stream)>>>(cu_spans, span_start, span_end, span_time, lengths,
                                                       t_stride, out);
  return launch_rc();
}
