// Fused paged decode for bf16, head_dim 128, 8 KV heads, GQA group 4 (the Llama-3-8B
// attention geometry), block_size 16 or 1 (the SGLang-style one-token block): one new token
// per sequence.
//
// One launch does, for every sequence of the batch (TinyLM.forward_cached,
// model.py:160-188, decode step, one layer):
//   * RoPE of q and of the new k at the token's logical position (rope.py:42-46),
//   * append of the rotated k and of v at the slot kvs_append_slots reserved
//     (PagedKVCache.write, paged_cache.py:167-171),
//   * GQA attention of q over every live entry of the block table
//     (Attention.forward, model.py:67-74: head h reads KV head h / 4, scores * D^-0.5,
//     softmax, weighted V).
//
// The unit of work is a group of 16 consecutive live entries of a sequence: one table entry
// when block_size is 16, sixteen table entries when it is 1.  Either way a group is 64 KiB of
// K and V (16 tokens x 8 heads x 128 x 2 B, twice), staged as one pipeline stage.
//
// Work split ("stream-K"): the groups of all sequences, concatenated in batch order,
// are cut into gridDim.x contiguous ranges of equal cost, one per CTA (one CTA per SM):
// a group costs one unit and each sequence SEQ_COST = 4 more (its start, finish and
// merge of partials), so every SM streams about the same number of KV bytes whatever
// the context lengths.  A sequence cut by range boundaries yields one partial
// (m, l, O) per CTA; the last CTA to finish a sequence (per-sequence arrival
// counter) merges its partials.
//
// Per CTA: 8 warps, warp w <-> KV head w (4 query heads).  A 3-stage cp.async
// pipeline stages whole 16-token groups (K and V of all heads, 64 KiB) in shared
// memory with a 16-byte-chunk XOR swizzle (chunk ^ token%8), so ldmatrix reads are
// conflict free.  Per block and warp: S^T[16 tokens x 8] = K[16x128] . Q^T (4 real
// heads + 4 zero columns) with 8 mma.m16n8k16 (bf16 in, fp32 accumulate), online
// softmax in fp32 (base 2), P^T brought into B-fragment layout with movmatrix, and
// O^T[128 x 8] += V^T . P^T with 8 more mma.
//
// One-token blocks: each token's K (or V) row of all heads is 2 KiB contiguous in the pool,
// so a group is gathered as 16 rows of 2 KiB through the block table (a warp copies 512
// contiguous bytes of one row per instruction).  The table entries of the CTA's range are read
// into shared memory through a rolling window of TAB_CAP entries; entries past a sequence's
// end are zero-filled instead of read (cp.async with a source size of 0).
#include "kvs_common.cuh"
#include "kvs_rope.cuh"

#include <mutex>

using namespace kvs;

namespace {

constexpr int D = 128;
constexpr int BS = 16;  // tokens of one work group (= one stage), whatever the block size
constexpr int HKV = 8;
constexpr int G = 4;
constexpr int HQ = HKV * G;
constexpr int NTHREADS = 32 * HKV;
constexpr int ROW_BYTES = D * 2;                       // one token of one head
constexpr int KV_BLOCK_BYTES = BS * HKV * ROW_BYTES;   // 32 KiB: K (or V) of one block, all heads
constexpr int STAGES = 3;
constexpr int STAGE_BYTES = 2 * KV_BLOCK_BYTES;
constexpr int MAX_SEQS = 1024;
constexpr int CHUNKS = KV_BLOCK_BYTES / 16;            // 2048 16-byte chunks per K (or V) block

constexpr int TAB_CAP = 2048;  // table entries of one CTA's range staged in shared memory
constexpr int TAB_GROUPS1 = TAB_CAP / BS;  // groups of one-token blocks per table window

constexpr int SMEM_STAGES = STAGES * STAGE_BYTES;
constexpr int SMEM_Q = HQ * D * 2;
constexpr int SMEM_NEW = 2 * HKV * D * 2;
constexpr int SMEM_PREF = (MAX_SEQS + 1) * 4;
constexpr int SMEM_TAB = TAB_CAP * 4;
constexpr int SEQ_COST = 4;  // a stream's start + finish + merge, in blocks of streaming time (work split)
constexpr int PLAN_HDR = 16;  // ints of the batch plan's header (16-token blocks)
constexpr int PLAN_REC = 8;   // ints of a CTA's start record: g0, g1, block ids of groups g0, g0 + 1
constexpr int PLAN_MAGIC = 0x6B76706C;  // header word 2 of a stored plan
constexpr int SMEM_ROPE = 2 * (D / 2) * 4;  // sin and cos of the D/2 angles of a stream's position
constexpr int SMEM_TOTAL = SMEM_STAGES + SMEM_Q + SMEM_NEW + SMEM_PREF + SMEM_TAB + 256 + SMEM_ROPE;
static_assert(HQ * 8 == NTHREADS, "start(): one thread per (query head, 16-byte chunk)");
static_assert(STAGES == 3, "a start record holds the block ids of the prologue's two stages");

struct DecodeParams {
  kvs_cache c;
  const int32_t* seq_slots;
  int num_seqs;
  int layer;
  const __nv_bfloat16* q;      // [S] rows of [HQ][D], q_stride elements apart
  const __nv_bfloat16* k_new;  // [S] rows of [HKV][D], kv_stride elements apart
  const __nv_bfloat16* v_new;
  int64_t q_stride, kv_stride;
  const int64_t* positions;    // [S]
  const int32_t* slot_blocks;  // [S]
  const int32_t* slot_offsets; // [S]
  const float* inv_freq;       // [D/2]
  __nv_bfloat16* out;          // [S][HQ][D]
  float* part_o;               // [slots][HQ][D]
  float* part_ml;              // [slots][HQ][2]
  int32_t* counters;           // [S]
  int32_t* plan;               // the step's batch plan (16-token blocks), or null
  int plan_mode;               // KVS_PLAN_*
  float scale_log2;            // D^-0.5 * log2(e)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
}
// An arrival on a stream's counter with acquire-release semantics at GPU scope: this thread's
// (and, through the barrier before it, its CTA's) partial writes are visible to whoever
// observes the count, and the partials of earlier arrivals are visible to this CTA after the
// barrier that follows (the same ordering as a full fence on each side, without its cost).
__device__ __forceinline__ int arrive_acq_rel(int32_t* counter) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;\n" : "=r"(old) : "l"(counter) : "memory");
  return old;
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
// 16-byte copy that reads `src_bytes` (16 or 0) bytes and zero-fills the rest
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16(uint32_t w) {
  __nv_bfloat162 v;
  memcpy(&v, &w, sizeof(w));
  return __bfloat1622float2(v);
}

// byte offset of 16-byte chunk `c` (0..15) of row `r` (= token*HKV + head) inside a K or V stage
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * ROW_BYTES + ((c ^ ((r >> 3) & 7)) << 4));
}

__device__ __forceinline__ float warp_max_rows(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  return v;
}
__device__ __forceinline__ float warp_sum_rows(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

// the global inputs of one sequence's start: its q chunk, new k / v chunks, inv_freq slice,
// logical position and append slot (owner = this CTA holds the sequence's last block).  Kept
// as loaded: nothing is computed from them until the sequence starts, so issuing the loads
// never waits for them.
struct SeqIn {
  uint4 q_lo, q_hi, k_lo, k_hi, v_c;
  int64_t pos;
  int32_t blk, off;
  bool owner;
};

// BSZ: the pool's block_size (16 or 1)
template <int BSZ>
__global__ void __launch_bounds__(NTHREADS, 1) decode_bf16_kernel(const DecodeParams p) {
  static_assert(BSZ == BS || BSZ == 1, "block_size 16 or 1");
  constexpr int ENTRY_BYTES = BSZ * HKV * ROW_BYTES;  // one table entry of K (or V), all heads
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  __nv_bfloat16* q_s = reinterpret_cast<__nv_bfloat16*>(smem + SMEM_STAGES);
  __nv_bfloat16* knew_s = reinterpret_cast<__nv_bfloat16*>(smem + SMEM_STAGES + SMEM_Q);
  __nv_bfloat16* vnew_s = knew_s + HKV * D;
  int* s_pref = reinterpret_cast<int*>(smem + SMEM_STAGES + SMEM_Q + SMEM_NEW);
  int* s_tab = s_pref + MAX_SEQS + 1;
  int* s_flag = s_tab + TAB_CAP;
  int* s_scan = s_flag + 4;  // 33 ints
  float* s_sin = reinterpret_cast<float*>(smem + SMEM_STAGES + SMEM_Q + SMEM_NEW + SMEM_PREF + SMEM_TAB + 256);
  float* s_cos = s_sin + D / 2;

  // Launched with programmatic stream serialization: the grid may become resident while the
  // previous kernel of the stream (the q|k|v projection, or the previous layer's decode) is
  // finishing; everything it reads waits for that kernel's completion here.
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const kvs_cache& c = p.c;
  const int S = p.num_seqs;
  const float my_freq = tid < D / 2 ? p.inv_freq[tid] : 0.f;  // inv_freq[tid]: the angle table's row

  const uint8_t* Kpool = static_cast<const uint8_t*>(c.k);
  const uint8_t* Vpool = static_cast<const uint8_t*>(c.v);
  const int64_t layer_rows = (int64_t)p.layer * c.num_blocks;
  // K and V of one 16-token block (all heads) into pipeline stage st, 16-byte copies into the
  // swizzled rows
  auto issue_blk = [&](int64_t blk, int st) {
    const uint32_t kd = smem_u32(stages + st * STAGE_BYTES);
    const uint32_t vd = kd + KV_BLOCK_BYTES;
    const uint8_t* ks = Kpool + (layer_rows + blk) * KV_BLOCK_BYTES;
    const uint8_t* vs = Vpool + (layer_rows + blk) * KV_BLOCK_BYTES;
#pragma unroll
    for (int k = 0; k < CHUNKS / NTHREADS; ++k) {
      const int q = tid + k * NTHREADS;
      const int r = q >> 4, ch = q & 15;
      cp_async16(kd + swz(r, ch), ks + (q << 4));
      cp_async16(vd + swz(r, ch), vs + (q << 4));
    }
  };

  // The batch plan of a decode step (16-token blocks): each CTA's start record (its group
  // range and the block ids of its first two groups), per-sequence prefix sums of the groups
  // and the block ids of every group, the same for all layers of the step.  A launch in
  // KVS_PLAN_BUILD mode computes them as below and stores them; one in KVS_PLAN_REUSE mode
  // reads the record and the prefix sums in one round of independent loads, issues the copies
  // of its first two blocks at once and gathers the other block ids while they fly (it computes
  // everything if the stored plan is for another batch size or grid).
  int32_t* const plan_rec = p.plan ? p.plan + PLAN_HDR : nullptr;
  int32_t* const plan_pref = p.plan ? plan_rec + PLAN_REC * gridDim.x : nullptr;
  int32_t* const plan_tab = p.plan ? plan_pref + S + 1 : nullptr;
  const bool build = BSZ == BS && p.plan && p.plan_mode == KVS_PLAN_BUILD;
  bool reuse = false;
  int pg0 = 0, pg1 = 0;
  if (BSZ == BS && p.plan && p.plan_mode == KVS_PLAN_REUSE) {
    const int hs = p.plan[0], hg = p.plan[1], hm = p.plan[2];
    const int4 rec = *reinterpret_cast<const int4*>(plan_rec + PLAN_REC * blockIdx.x);
    int pv[5];
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      const int i = tid + k * NTHREADS;
      pv[k] = i <= S ? plan_pref[i] : 0;
    }
    reuse = hs == S && hg == (int)gridDim.x && hm == PLAN_MAGIC;  // the same loads in every thread
    if (reuse) {
      pg0 = rec.x;
      pg1 = rec.y;
      // the pipeline's first two stages, as the prologue below would issue them
      if (pg0 < pg1) issue_blk(rec.z, 0);
      cp_async_commit();
      if (pg0 + 1 < pg1) issue_blk(rec.w, 1);
      cp_async_commit();
#pragma unroll
      for (int k = 0; k < 5; ++k) {
        const int i = tid + k * NTHREADS;
        if (i <= S) s_pref[i] = pv[k];
      }
    }
  }
  // prefix sums of table lengths (blocks) over the batch: thread tid owns sequences
  // 4*tid .. 4*tid+3 (MAX_SEQS = 4 * NTHREADS), one block-wide scan
  if (!reuse) {
    int nb[4], sum = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = 4 * tid + k;
      nb[k] = i < S ? (c.lengths[p.seq_slots[i]] + BS - 1) / BS : 0;
      sum += nb[k];
    }
    int total_nb = 0;
    int run = block_exclusive_scan(sum, s_scan, &total_nb);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = 4 * tid + k;
      if (i < S) s_pref[i] = run;
      run += nb[k];
    }
    if (tid == 0) s_pref[S] = total_nb;
  }
  __syncthreads();
  // Cost units: every block is one, and every stream adds SEQ_COST in front of its first block
  // (the start, finish and merge work of a stream, a few blocks of streaming time), so a CTA
  // that carries a stream boundary gets fewer blocks.  Global block gb of stream i sits at unit
  // gb + SEQ_COST (i + 1); CTA c takes the units [c RU, (c + 1) RU).
  const int total = s_pref[S];
  const int total_units = total + SEQ_COST * S;
  const int RU = (total_units + gridDim.x - 1) / gridDim.x;
  auto first_block = [&](int u) {  // the first block at unit >= u
    if (u >= total_units) return total;
    int lo = 0, hi = S - 1;  // last stream i with s_pref[i] + SEQ_COST i <= u
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_pref[mid] + SEQ_COST * mid <= u) lo = mid; else hi = mid - 1;
    }
    const int j = u - (s_pref[lo] + SEQ_COST * (lo + 1));
    return j <= 0 ? s_pref[lo] : min(s_pref[lo] + j, s_pref[lo + 1]);
  };
  const int g0 = reuse ? pg0 : first_block(blockIdx.x * RU);
  const int g1 = reuse ? pg1 : first_block(blockIdx.x * RU + RU);
  if (build) {
    if (tid == 0) {
      plan_rec[PLAN_REC * blockIdx.x] = g0;
      plan_rec[PLAN_REC * blockIdx.x + 1] = g1;
    }
    if (blockIdx.x == 0) {
      for (int i = tid; i <= S; i += NTHREADS) plan_pref[i] = s_pref[i];
      if (tid == 0) {
        p.plan[0] = S;
        p.plan[1] = gridDim.x;
        p.plan[2] = PLAN_MAGIC;
      }
    }
  }
  if (g0 >= g1) return;

  auto seq_of = [&](int gb) {
    int lo = 0, hi = S - 1;  // last i with s_pref[i] <= gb
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_pref[mid] <= gb) lo = mid; else hi = mid - 1;
    }
    return lo;
  };

  // A sequence's start inputs in one round of 16-byte loads: thread -> head h = tid / 8 and
  // chunk d0 = 8 (tid % 8), i.e. elements d0 .. d0+7 of each half of the head.  Threads 0..63
  // also load the new k (8 heads), threads 0..127 the new v, when this CTA appends the token.
  auto load_seq = [&](int i) {
    SeqIn s;
    const int h = tid >> 3, d0 = (tid & 7) * 8;
    s.pos = p.positions[i];
    const int last = s_pref[i + 1] - 1;
    s.owner = last >= g0 && last < g1;
    const uint4* qsrc = reinterpret_cast<const uint4*>(p.q + (int64_t)i * p.q_stride + h * D + d0);
    s.q_lo = qsrc[0];
    s.q_hi = qsrc[D / 16];
    s.k_lo = s.k_hi = s.v_c = make_uint4(0, 0, 0, 0);
    s.blk = s.off = 0;
    if (s.owner) {
      s.blk = p.slot_blocks[i];
      s.off = p.slot_offsets[i];
      if (tid < HKV * 8) {
        const uint4* ksrc = reinterpret_cast<const uint4*>(p.k_new + (int64_t)i * p.kv_stride + h * D + d0);
        s.k_lo = ksrc[0];
        s.k_hi = ksrc[D / 16];
      }
      if (tid < HKV * D / 8) s.v_c = reinterpret_cast<const uint4*>(p.v_new + (int64_t)i * p.kv_stride)[tid];
    }
    return s;
  };
  // the first sequence's loads overlap the table gather and the prologue's KV copies
  const int first = seq_of(g0);
  const int last_seq = seq_of(g1 - 1);
  const SeqIn first_in = load_seq(first);

  // block ids of this CTA's range, gathered once (the copies below then need no global lookups).
  // One-token blocks: a window of TAB_GROUPS1 groups (16 entries each, -1 past a sequence's
  // end), starting at group w0 and moved forward by the main loop when the prefetch leaves it.
  const bool tab_in_smem = BSZ == 1 || (g1 - g0) <= TAB_CAP;
  int w0 = g0;
  auto gather1 = [&](int w) {
    const int n = min(TAB_GROUPS1, g1 - w) * BS;
    for (int e = tid; e < n; e += NTHREADS) {
      const int gb = w + (e >> 4);
      const int i = seq_of(gb);
      const int slot = p.seq_slots[i];
      const int idx = (gb - s_pref[i]) * BS + (e & 15);
      s_tab[e] = idx < c.lengths[slot] ? c.tables[(int64_t)slot * c.max_blocks + idx] : -1;
    }
  };
  if constexpr (BSZ == 1) {
    gather1(g0);
    __syncthreads();
  } else if (tab_in_smem) {
    for (int gb = g0 + tid; gb < g1; gb += NTHREADS) {
      int blk;
      if (reuse) {
        blk = plan_tab[gb];
      } else {
        const int i = seq_of(gb);
        blk = c.tables[(int64_t)p.seq_slots[i] * c.max_blocks + (gb - s_pref[i])];
        if (build) {
          plan_tab[gb] = blk;
          if (gb - g0 < 2) plan_rec[PLAN_REC * blockIdx.x + 2 + (gb - g0)] = blk;
        }
      }
      s_tab[gb - g0] = blk;
    }
    __syncthreads();
  } else if (build) {
    for (int gb = g0 + tid; gb < g1; gb += NTHREADS) {
      const int i = seq_of(gb);
      const int blk = c.tables[(int64_t)p.seq_slots[i] * c.max_blocks + (gb - s_pref[i])];
      plan_tab[gb] = blk;
      if (gb - g0 < 2) plan_rec[PLAN_REC * blockIdx.x + 2 + (gb - g0)] = blk;
    }
  }

  auto issue = [&](int gb, int st) {
    if constexpr (BSZ == 1) {
      const uint32_t kd = smem_u32(stages + st * STAGE_BYTES);
      const uint32_t vd = kd + KV_BLOCK_BYTES;
      // chunk q = tid + k NTHREADS is 16-byte chunk (q & 127) of token q >> 7 (row q >> 4)
      const int* ent = s_tab + (gb - w0) * BS;
#pragma unroll
      for (int k = 0; k < CHUNKS / NTHREADS; ++k) {
        const int q = tid + k * NTHREADS;
        const int r = q >> 4, ch = q & 15;
        const int blk = ent[q >> 7];
        const int64_t off = (layer_rows + (blk < 0 ? 0 : blk)) * ENTRY_BYTES + ((q & 127) << 4);
        cp_async16_zfill(kd + swz(r, ch), Kpool + off, blk < 0 ? 0 : 16);
        cp_async16_zfill(vd + swz(r, ch), Vpool + off, blk < 0 ? 0 : 16);
      }
    } else {
      int64_t blk;
      if (tab_in_smem) {
        blk = s_tab[gb - g0];
      } else if (reuse) {
        blk = plan_tab[gb];
      } else {
        const int i = seq_of(gb);
        blk = c.tables[(int64_t)p.seq_slots[i] * c.max_blocks + (gb - s_pref[i])];
      }
      issue_blk(blk, st);
    }
  };

  // prologue (a reusing launch issued it from its start record)
  if (!reuse) {
#pragma unroll
    for (int k = 0; k < STAGES - 1; ++k) {
      if (g0 + k < g1) issue(g0 + k, k);
      cp_async_commit();
    }
  }

  // per-warp state of the current segment (one sequence inside this CTA's range)
  uint32_t bq[8][2];
  float acc[8][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  int cur = -1;

  // CTAs [c0, c0 + expected) share sequence i (the ranges that hold one of its blocks)
  auto seq_ctas = [&](int i, int& c0) {
    const int P0 = s_pref[i], nb = s_pref[i + 1] - P0;
    c0 = (P0 + SEQ_COST * (i + 1)) / RU;
    return (P0 + nb - 1 + SEQ_COST * (i + 1)) / RU - c0 + 1;
  };
  // Streams shared with other CTAs: at most the first and the last of this CTA's range.  Each
  // CTA writes its partial when it leaves the stream and arrives on the stream's counter; the
  // last to arrive merges.  A stream left mid-range arrives at once but reads the counter's
  // answer only at the end of the kernel (e_seq), the stream the range ends in arrives at the
  // end (t_seq), so moving on to the next stream waits for no global round trip.
  int e_seq = -1, t_seq = -1;
  int arrived0 = 0;  // thread 0: the counter value the early arrival for e_seq returned
  auto finish = [&](int i) {
    // sequence i: this CTA's part is done; write the output, or this CTA's partial
    int c0;
    const int expected = seq_ctas(i, c0);
    const float lt0 = warp_sum_rows(l0), lt1 = warp_sum_rows(l1);
    const int hq0 = warp * G + 2 * t;  // query heads hq0, hq0+1 (valid for t < 2)
    if (expected == 1) {
      if (t < 2) {
        __nv_bfloat16* o = p.out + ((int64_t)i * HQ + hq0) * D;
        const float r0 = 1.f / lt0, r1 = 1.f / lt1;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int d = mt * 16 + g;
          o[d] = __float2bfloat16_rn(acc[mt][0] * r0);
          o[D + d] = __float2bfloat16_rn(acc[mt][1] * r1);
          o[d + 8] = __float2bfloat16_rn(acc[mt][2] * r0);
          o[D + d + 8] = __float2bfloat16_rn(acc[mt][3] * r1);
        }
      }
      return;
    }
    const int slot_id = blockIdx.x + i;  // unique per (CTA, sequence) pair
    if (t < 2) {
      float* o = p.part_o + ((int64_t)slot_id * HQ + hq0) * D;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int d = mt * 16 + g;
        o[d] = acc[mt][0];
        o[D + d] = acc[mt][1];
        o[d + 8] = acc[mt][2];
        o[D + d + 8] = acc[mt][3];
      }
      if (g == 0) {
        float* ml = p.part_ml + ((int64_t)slot_id * HQ + hq0) * 2;
        ml[0] = m0;
        ml[1] = lt0;
        ml[2] = m1;
        ml[3] = lt1;
      }
    }
    if (i == last_seq) {
      t_seq = i;
    } else {
      e_seq = i;
      // a stream this CTA leaves mid-range (its first one): arrive now, with every thread's
      // partial writes ordered before the arrival by the barrier and the release; the value
      // returned is only read at the end of the kernel, so nothing waits for it here
      __syncthreads();
      if (tid == 0) arrived0 = arrive_acq_rel(&p.counters[i]);
    }
  };
  // the last CTA to arrive for sequence i combines the partials of its `expected` CTAs
  auto merge = [&](int i) {
    int c0;
    const int expected = seq_ctas(i, c0);
    // thread -> head h = tid / 8, dims d0 = 16 (tid % 8) .. +16.  The partials are read four at
    // a time with all their loads in flight and combined under a running maximum:
    // out = sum_k 2^(m_k - M) o_k / sum_k 2^(m_k - M) l_k
    const int h = tid >> 3, d0 = (tid & 7) * 16;
    float M = -INFINITY, den = 0.f;
    float4 o[4];
#pragma unroll
    for (int v = 0; v < 4; ++v) o[v] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = 0; k0 < expected; k0 += 4) {
      float mk[4], lk[4];
      float4 xk[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        mk[u] = -INFINITY;
        lk[u] = 0.f;
#pragma unroll
        for (int v = 0; v < 4; ++v) xk[u][v] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k0 + u < expected) {
          const int64_t slot = c0 + k0 + u + i;
          const float* ml = p.part_ml + (slot * HQ + h) * 2;
          mk[u] = __ldcg(ml);
          lk[u] = __ldcg(ml + 1);
          const float4* src = reinterpret_cast<const float4*>(p.part_o + (slot * HQ + h) * D + d0);
#pragma unroll
          for (int v = 0; v < 4; ++v) xk[u][v] = __ldcg(src + v);
        }
      }
      float Mn = M;
#pragma unroll
      for (int u = 0; u < 4; ++u) Mn = fmaxf(Mn, mk[u]);
      const float sc = exp2f(M - Mn);  // 0 on the first group (M = -inf)
      den *= sc;
#pragma unroll
      for (int v = 0; v < 4; ++v) o[v] = make_float4(o[v].x * sc, o[v].y * sc, o[v].z * sc, o[v].w * sc);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float w = exp2f(mk[u] - Mn);  // 0 for the slots beyond `expected`
        den += w * lk[u];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          o[v].x += w * xk[u][v].x;
          o[v].y += w * xk[u][v].y;
          o[v].z += w * xk[u][v].z;
          o[v].w += w * xk[u][v].w;
        }
      }
      M = Mn;
    }
    const float inv = 1.f / den;
    uint32_t packed[8];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      packed[2 * v] = pack_bf16(o[v].x * inv, o[v].y * inv);
      packed[2 * v + 1] = pack_bf16(o[v].z * inv, o[v].w * inv);
    }
    int4* dst = reinterpret_cast<int4*>(p.out + ((int64_t)i * HQ + h) * D + d0);
    dst[0] = make_int4(packed[0], packed[1], packed[2], packed[3]);
    dst[1] = make_int4(packed[4], packed[5], packed[6], packed[7]);
    if (tid == 0) p.counters[i] = 0;  // ready for the next launch
  };

  // RoPE of q into shared memory, and the append of the rotated new k and of v (same rotation
  // as every other kernel of the library); pairs (d, d + D/2) of each head
  auto apply_seq = [&](const SeqIn& in) {
    const int h = tid >> 3, d0 = (tid & 7) * 8;
    const int64_t pos = in.pos, row = ((layer_rows + in.blk) * BSZ + in.off) * HKV;
    // the D/2 angles of this position, once per stream (every head of q and of the new k
    // rotates by the same ones): one sincos per thread of the first D/2 instead of eight each
    if (tid < D / 2) rope_sincos<float, float>(pos, my_freq, s_sin[tid], s_cos[tid]);
    __syncthreads();
    // words w of lo / hi hold elements (d0 + 2w, d0 + 2w + 1) and (d0 + D/2 + 2w, ...)
    auto rot2 = [&](uint32_t lo, uint32_t hi, int w, uint32_t& out_lo, uint32_t& out_hi) {
      const float2 a = unpack_bf16(lo), b = unpack_bf16(hi);
      float r0, r1, r2, r3;
      const int f = d0 + 2 * w;
      rope_apply(a.x, b.x, s_sin[f], s_cos[f], r0, r1);
      rope_apply(a.y, b.y, s_sin[f + 1], s_cos[f + 1], r2, r3);
      out_lo = pack_bf16(r0, r2);
      out_hi = pack_bf16(r1, r3);
    };
    auto rotate = [&](const uint4 lo, const uint4 hi, uint4& out_lo, uint4& out_hi) {
      rot2(lo.x, hi.x, 0, out_lo.x, out_hi.x);
      rot2(lo.y, hi.y, 1, out_lo.y, out_hi.y);
      rot2(lo.z, hi.z, 2, out_lo.z, out_hi.z);
      rot2(lo.w, hi.w, 3, out_lo.w, out_hi.w);
    };
    uint4 o_lo, o_hi;
    rotate(in.q_lo, in.q_hi, o_lo, o_hi);
    *reinterpret_cast<uint4*>(q_s + h * D + d0) = o_lo;
    *reinterpret_cast<uint4*>(q_s + h * D + d0 + D / 2) = o_hi;
    if (in.owner) {
      __nv_bfloat16* K = static_cast<__nv_bfloat16*>(c.k);
      __nv_bfloat16* V = static_cast<__nv_bfloat16*>(c.v);
      if (tid < HKV * 8) {
        rotate(in.k_lo, in.k_hi, o_lo, o_hi);
        *reinterpret_cast<uint4*>(knew_s + h * D + d0) = o_lo;
        *reinterpret_cast<uint4*>(knew_s + h * D + d0 + D / 2) = o_hi;
        *reinterpret_cast<uint4*>(K + (row + h) * D + d0) = o_lo;
        *reinterpret_cast<uint4*>(K + (row + h) * D + d0 + D / 2) = o_hi;
      }
      if (tid < HKV * D / 8) {
        *reinterpret_cast<uint4*>(vnew_s + tid * 8) = in.v_c;
        *reinterpret_cast<uint4*>(V + row * D + tid * 8) = in.v_c;
      }
    }
    __syncthreads();
    const __nv_bfloat16* qh = q_s + (warp * G + g) * D;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      bq[kk][0] = g < G ? *reinterpret_cast<const uint32_t*>(qh + kk * 16 + 2 * t) : 0u;
      bq[kk][1] = g < G ? *reinterpret_cast<const uint32_t*>(qh + kk * 16 + 2 * t + 8) : 0u;
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
  };
  // the next sequence of the range, its inputs loaded while the current one streams
  int nxt = -1;
  SeqIn nxt_in;
  auto prefetch_after = [&](int i) {
    nxt = (i + 1 < S && s_pref[i + 1] < g1) ? i + 1 : -1;
    if (nxt >= 0) nxt_in = load_seq(nxt);
  };

  cur = first;
  apply_seq(first_in);
  prefetch_after(first);

  for (int gb = g0; gb < g1; ++gb) {
    const int it = gb - g0;
    const int st = it % STAGES;
    if constexpr (BSZ == 1) {
      // every thread finished last iteration's issue before the trailing barrier, so the
      // window may be refilled here; groups gb .. gb + STAGES - 2 are in flight already
      if (gb + STAGES - 1 < g1 && gb + STAGES - 1 >= w0 + TAB_GROUPS1) {
        w0 = gb;
        gather1(w0);
        __syncthreads();
      }
    }
    if (gb + STAGES - 1 < g1) issue(gb + STAGES - 1, (it + STAGES - 1) % STAGES);
    cp_async_commit();
    cp_async_wait<STAGES - 1>();
    __syncthreads();

    const int i = seq_of(gb);
    if (i != cur) {
      if (cur >= 0) finish(cur);
      apply_seq(i == nxt ? nxt_in : load_seq(i));
      prefetch_after(i);
      cur = i;
    }
    const int j = gb - s_pref[i];
    const int nb = s_pref[i + 1] - s_pref[i];
    // the new token is the last live entry: at offset slot_offsets[i] of the last block
    // (block_size 16), or the (length - 1) % 16-th token of the last group (one-token blocks)
    const int tail = (j == nb - 1) ? (BSZ == BS ? p.slot_offsets[i] + 1
                                                : ((c.lengths[p.seq_slots[i]] - 1) & (BS - 1)) + 1)
                                   : BS;
    const int valid = tail;
    uint8_t* kst = stages + st * STAGE_BYTES;
    uint8_t* vst = kst + KV_BLOCK_BYTES;
    if (j == nb - 1) {
      // the prefetch may predate the append: patch the new token's rows in shared memory
      const int off = tail - 1;
      const int r = off * HKV + (tid >> 4) % HKV, ch = tid & 15;  // 256 threads = 8 heads x 16 chunks
      const __nv_bfloat16* srck = (tid < HKV * 16) ? knew_s + ((tid >> 4)) * D + ch * 8 : nullptr;
      if (tid < HKV * 16) {
        *reinterpret_cast<int4*>(kst + swz(r, ch)) = *reinterpret_cast<const int4*>(srck);
        *reinterpret_cast<int4*>(vst + swz(r, ch)) =
            *reinterpret_cast<const int4*>(vnew_s + (tid >> 4) * D + ch * 8);
      }
      __syncthreads();
    }

    // ---- S^T = K . Q^T  (16 tokens x 8 head columns)
    const uint32_t kbase = smem_u32(kst), vbase = smem_u32(vst);
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int mi = lane >> 3, rr = lane & 7;
      const int tok = rr + ((mi & 1) << 3);
      const int row = tok * HKV + warp;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kbase + swz(row, 2 * kk + (mi >> 1)), a0, a1, a2, a3);
        mma_bf16(sc, a0, a1, a2, a3, bq[kk][0], bq[kk][1]);
      }
    }
    // ---- online softmax (base 2); lane holds tokens g, g+8 and heads 2t, 2t+1
    float s0 = sc[0] * p.scale_log2, s1 = sc[1] * p.scale_log2;
    float s2 = sc[2] * p.scale_log2, s3 = sc[3] * p.scale_log2;
    if (g >= valid) s0 = s1 = -INFINITY;
    if (g + 8 >= valid) s2 = s3 = -INFINITY;
    const float bm0 = warp_max_rows(fmaxf(s0, s2));
    const float bm1 = warp_max_rows(fmaxf(s1, s3));
    const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
    const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
    const float p0 = exp2f(s0 - mn0), p1 = exp2f(s1 - mn1);
    const float p2 = exp2f(s2 - mn0), p3 = exp2f(s3 - mn1);
    l0 = l0 * al0 + p0 + p2;
    l1 = l1 * al1 + p1 + p3;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      acc[mt][0] *= al0;
      acc[mt][1] *= al1;
      acc[mt][2] *= al0;
      acc[mt][3] *= al1;
    }
    // P as the sum of two bf16 terms, hi = bf16(p) and lo = bf16(p - hi): 16 significant bits
    // for P V at two MMAs per fragment instead of one (free in this HBM-bound kernel), so the
    // decode and the masked replay kernel round P far less differently
    const uint32_t h01 = pack_bf16(p0, p1), h23 = pack_bf16(p2, p3);
    const float2 r01 = unpack_bf16(h01), r23 = unpack_bf16(h23);
    const uint32_t pb0 = movm_t(h01);  // P[head g][tokens 2t, 2t+1]
    const uint32_t pb1 = movm_t(h23);  // P[head g][tokens 8+2t, 9+2t]
    const uint32_t pl0 = movm_t(pack_bf16(p0 - r01.x, p1 - r01.y));
    const uint32_t pl1 = movm_t(pack_bf16(p2 - r23.x, p3 - r23.y));
    // ---- O^T += V^T . P^T
    {
      const int mi = lane >> 3, rr = lane & 7;
      const int tok = rr + ((mi >> 1) << 3);
      const int row = tok * HKV + warp;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(vbase + swz(row, 2 * mt + (mi & 1)), a0, a1, a2, a3);
        mma_bf16(acc[mt], a0, a1, a2, a3, pb0, pb1);
        mma_bf16(acc[mt], a0, a1, a2, a3, pl0, pl1);
      }
    }
    __syncthreads();  // the stage is refilled by the next iteration's prefetch
  }
  cp_async_wait<0>();
  if (cur >= 0) finish(cur);
  // arrivals for the shared streams (each after this CTA's partial writes are visible), then
  // the merges of those for which this CTA arrived last
  if (e_seq >= 0 || t_seq >= 0) {
    __syncthreads();
    if (tid == 0) {
      int c0;
      s_flag[0] = e_seq >= 0 && arrived0 == seq_ctas(e_seq, c0) - 1;
      s_flag[1] = 0;
      if (t_seq >= 0) s_flag[1] = arrive_acq_rel(&p.counters[t_seq]) == seq_ctas(t_seq, c0) - 1;
    }
    __syncthreads();
    if (s_flag[0]) merge(e_seq);
    if (s_flag[1]) merge(t_seq);
  }
}

std::mutex g_attr_mu;
bool g_attr_done[2][64] = {};  // [block_size == 1][device]

}  // namespace

// ---------------------------------------------------------------------------- host
// Scratch: arrival counters first, at a fixed offset and for the largest batch, so that a
// buffer reused by calls of different batch sizes always finds them where the previous call
// left them at zero; then the partial rows (data, written before they are read).
constexpr size_t COUNTER_BYTES = (size_t)MAX_SEQS * 4;
static_assert(COUNTER_BYTES % 256 == 0, "partials stay 256-byte aligned");

// the batch plan: header, a start record per CTA (8 ints, 16-byte aligned), num_seqs + 1
// prefix sums, one block id per group (at most max_blocks per sequence); 16-token blocks only
static size_t plan_bytes(const kvs_cache* c, int num_seqs, int grid) {
  if (c->block_size != BS) return 0;
  return align_up(((size_t)PLAN_HDR + PLAN_REC * (size_t)grid + num_seqs + 1 + (size_t)num_seqs * c->max_blocks) * 4,
                  256);
}
static size_t partial_bytes(int num_seqs, int grid) {
  const size_t slots = (size_t)grid + num_seqs;
  return align_up(slots * HQ * D * 4, 256) + align_up(slots * HQ * 2 * 4, 256);
}

size_t kvs_decode_bf16_scratch(const kvs_cache* c, int num_seqs, int grid) {
  return COUNTER_BYTES + partial_bytes(num_seqs, grid) + plan_bytes(c, num_seqs, grid);
}

bool kvs_decode_bf16_supported(const kvs_cache* c, const kvs_batch* b, int n_heads) {
  return c->dtype == KVS_BF16 && c->head_dim == D && (c->block_size == BS || c->block_size == 1) &&
         c->n_kv_heads == HKV &&
         n_heads == HQ && b->cu_tokens == nullptr && b->num_seqs <= MAX_SEQS;
}

int kvs_decode_bf16_grid(int override_ctas) {
  if (override_ctas > 0) return override_ctas;
  const int sms = kvs_device_sm_count();
  return sms > 0 ? sms : 148;
}

int kvs_decode_bf16_launch(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a, int grid,
                           cudaStream_t st) {
  if (a->scratch_bytes < kvs_decode_bf16_scratch(c, b->num_seqs, grid) || !a->scratch) return KVS_E_SCRATCH;
  if (a->plan < KVS_PLAN_NONE || a->plan > KVS_PLAN_REUSE) return KVS_E_ARG;
  int dev = 0;
  cudaGetDevice(&dev);
  const int one = c->block_size == 1;
  const auto kernel = one ? decode_bf16_kernel<1> : decode_bf16_kernel<BS>;
  {
    std::lock_guard<std::mutex> lock(g_attr_mu);
    if (dev < 64 && !g_attr_done[one][dev]) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TOTAL) != cudaSuccess)
        return KVS_E_LAUNCH;
      g_attr_done[one][dev] = true;
    }
  }
  DecodeParams p;
  p.c = *c;
  p.seq_slots = b->seq_slots;
  p.num_seqs = b->num_seqs;
  p.layer = a->layer;
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.k_new = static_cast<const __nv_bfloat16*>(a->k_new);
  p.v_new = static_cast<const __nv_bfloat16*>(a->v_new);
  p.q_stride = a->q_stride ? a->q_stride : (int64_t)HQ * D;
  p.kv_stride = a->kv_stride ? a->kv_stride : (int64_t)HKV * D;
  p.positions = a->positions;
  p.slot_blocks = a->slot_blocks;
  p.slot_offsets = a->slot_offsets;
  p.inv_freq = static_cast<const float*>(a->inv_freq);
  p.out = static_cast<__nv_bfloat16*>(a->out);
  const size_t slots = (size_t)grid + b->num_seqs;
  uint8_t* s = static_cast<uint8_t*>(a->scratch);
  p.counters = reinterpret_cast<int32_t*>(s);
  p.part_o = reinterpret_cast<float*>(s + COUNTER_BYTES);
  p.part_ml = reinterpret_cast<float*>(s + COUNTER_BYTES + align_up(slots * HQ * D * 4, 256));
  p.plan = plan_bytes(c, b->num_seqs, grid)
               ? reinterpret_cast<int32_t*>(s + COUNTER_BYTES + partial_bytes(b->num_seqs, grid))
               : nullptr;
  p.plan_mode = a->plan;
  p.scale_log2 = (float)(a->scale * 1.4426950408889634);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(NTHREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return KVS_E_LAUNCH;
  }
  return launch_rc();
}
