// Masked replay attention on the 5th-generation tensor cores (tcgen05 / TMEM), bf16,
// head_dim 128: the trainer's one-pass replay of a KV-streams rollout
// (TinyLM.forward attention, model.py:71-74, under the mask of replay.py:55-63):
//
//   visible(t, s) = s <= t && t < evicted_at[b][s]     (t < lengths[b])
//   visible(t, s) = s == t                             (padded rows, collate replay.py:221-222)
//
// Two kernels share the tile skipping, the TMA/UMMA plumbing and the mask:
//   pair_attn_kernel<false> (GQA group size even, the default there): a CTA takes two query
//     heads of one KV head at the same 128 positions (pair_attn_kernel<true> is the same
//     pipeline over paged K/V for prefill chunks), so every staged K/V tile feeds four
//     UMMA tiles and two softmax warpgroups (one full row per thread) alternate with the
//     tensor pipe; described at the kernel.
//   replay_tc_kernel (any group size): CTA = (stream b, query head h, 128-query tile),
//     320 threads:
//   warp 0      TMA producer: Q tile once; per active key tile the K and V tiles
//               (128 keys x 128 dims, 128-byte swizzle) and the tile's evicted_at
//               values, into 2-slot rings;
//   warp 1      TMEM owner + UMMA issuer: S[k%2] = Q K^T (8 x M128 N128 K16) into
//               TMEM, then O += P V (P from TMEM, V MN-major) into TMEM;
//   warps 2..9  softmax: two warps per TMEM lane quadrant, each owning 64 key columns of
//               32 query rows; online softmax in fp32 base 2 with a lazy rescale (O is
//               only rescaled when the row max grew by more than 2^8), the row maximum
//               exchanged through shared memory, P written as bf16 into TMEM.
//     TMEM: S0 [0,128), S1 [128,256), O [256,384), P buffers [384,448) [448,512).
//
// Tile skipping: per 128-key tile the prepass records min/max evicted_at; a key
// tile is skipped when every key in it was evicted at or before the tile's first
// query, or lies above the diagonal; tiles fully visible to every row of the query
// tile run without per-element masking.
#include "kvs_common.cuh"
#include "kvs_sm100.cuh"

#include <mutex>

using namespace kvs;
using namespace kvs::sm100;

namespace {

constexpr int BM = 128, BN = 128, HD = 128;
constexpr int NSOFT = 256;                 // 8 softmax warps: two per TMEM lane quadrant
constexpr int NT = 64 + NSOFT;             // + producer warp + UMMA warp
constexpr int HALF_BYTES = 128 * 64 * 2;  // 128 rows x 64 bf16 (one 128-byte swizzled half tile)
constexpr int TILE_BYTES = 2 * HALF_BYTES;  // 128 x 128 bf16
constexpr int E_BYTES = BN * 4;

// shared memory map (offsets from a 1024-byte aligned base)
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE_BYTES;          // 2 slots
constexpr int OFF_V = OFF_K + 2 * TILE_BYTES;      // 2 slots
constexpr int OFF_E = OFF_V + 2 * TILE_BYTES;      // 2 slots of 128 int32
constexpr int OFF_RED = OFF_E + 2 * E_BYTES;       // [2 tiles][2 halves][128 rows] f32 row maxima
constexpr int OFF_LIST = OFF_RED + 2 * 2 * BM * 4; // active key tiles
constexpr int MAX_KT = 256;  // key tiles per stream: T <= 32768
constexpr int OFF_BAR = OFF_LIST + MAX_KT * 2;
constexpr int NBAR = 18;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_MISC + 64 + 33 * 4 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 232448, "replay kernel shared memory");

// K and V rings are refilled independently: a K slot as soon as Q K^T has read it, a V slot
// (with the tile's evicted_at values) once P V has read it.  P lives in TMEM, two buffers:
// PFULLb = P of the tile using buffer b written, PVDONEb = the P V that read buffer b done.
enum { B_KFULL0 = 0, B_KFULL1, B_VFULL0, B_VFULL1, B_KEMPTY0, B_KEMPTY1, B_VEMPTY0, B_VEMPTY1, B_QFULL,
       B_SFULL0, B_SFULL1, B_SFREE0, B_SFREE1, B_PFULL0, B_PFULL1, B_PVDONE0, B_PVDONE1, B_FINAL };

// named barrier over the softmax warps only (id 1; id 0 is __syncthreads)
__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, %0;\n" ::"n"(NSOFT) : "memory"); }

struct ReplayParams {
  const int32_t* e32;      // [B][T_pad] evicted_at clamped to int32, 0 past T
  const int32_t* tile_min; // [B][n_kt]
  const int32_t* tile_max; // [B][n_kt]
  const int32_t* lengths;  // [B]
  __nv_bfloat16* out;      // [B][T][Hq][D]
  float* lse;              // optional [B][Hq][T_pad]: log2 sum of 2^(scaled score) per row
  int32_t* error;          // [1]
  int B, T, T_pad, Hq, Hkv, n_qt, n_kt;
  float scale_log2;
};

// Paged prefill source: queries are the new tokens of a batch of sequences (concatenated,
// rotated), keys/values the live entries of each sequence in the paged pool.
struct PagedParams {
  const int32_t* seq_slots;  // [num_seqs]
  const int32_t* cu_tokens;  // [num_seqs + 1] new-token offsets
  const int32_t* cu_qt;      // [num_seqs + 1] 128-query tile offsets
  const int32_t* lengths;    // cache lengths (new tokens included), by slot
  const int32_t* tables;     // [max_seqs][max_blocks]
  int32_t* status;           // the cache's status words
  int num_seqs, max_blocks;
  int pool_rows;             // num_blocks * 16: a row coordinate past the pool reads zeros
};

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
// (a, b) as an f16 pair, a in the low half; finite inputs beyond the f16 range saturate
__device__ __forceinline__ uint32_t pack2h(float a, float b) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;\n" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
// a bf16 pair re-encoded as an f16 pair (exact for magnitudes in [2^-14, 65504])
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t x) {
  return pack2h(__uint_as_float(x << 16), __uint_as_float(x & 0xffff0000u));
}

__global__ void __launch_bounds__(NT, 1)
replay_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const ReplayParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Qs = smem + OFF_Q;
  uint16_t* list = reinterpret_cast<uint16_t*>(smem + OFF_LIST);  // key tile | 0x8000 if masked
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
  int* s_n = reinterpret_cast<int*>(smem + OFF_MISC + 8);
  int* s_scan = reinterpret_cast<int*>(smem + OFF_MISC + 64);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // CTA order: (stream, KV head) slowest, then query tiles heaviest first, then the query
  // heads of the GQA group -- CTAs resident together read the same K/V tiles (L2 reuse)
  const int G = p.Hq / p.Hkv;
  const int g = (int)(blockIdx.x % G);
  const int rest = (int)(blockIdx.x / G);
  const int qt = p.n_qt - 1 - rest % p.n_qt;
  const int bhk = rest / p.n_qt;
  const int b = bhk / p.Hkv, hk = bhk % p.Hkv;
  const int h = hk * G + g;
  const int t0 = qt * BM, t1 = t0 + BM - 1;
  const int L = p.lengths[b];

  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(&bar[i], 1);
    mbar_init(&bar[B_SFREE0], NSOFT);
    mbar_init(&bar[B_SFREE1], NSOFT);
    mbar_init(&bar[B_PFULL0], NSOFT);
    mbar_init(&bar[B_PFULL1], NSOFT);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }

  // ---- active key tiles for this query tile (same list for every role)
  {
    const int real_last = min(t1, L - 1);
    int carry = 0;
    for (int base = 0; base <= qt; base += NT) {
      const int j = base + tid;
      int flag = 0;
      if (j <= qt) {
        const int emin = p.tile_min[b * p.n_kt + j], emax = p.tile_max[b * p.n_kt + j];
        const bool active = (j == qt) || (j * BN <= real_last && emax > t0);
        const bool masked = (j == qt) || (emin <= t1) || (t1 >= L);
        flag = (active ? 1 : 0) | (masked ? 2 : 0);
      }
      int tot = 0;
      const int pre = block_exclusive_scan(flag & 1, s_scan, &tot);
      if (flag & 1) list[carry + pre] = (uint16_t)(j | ((flag & 2) ? 0x8000 : 0));
      carry += tot;
      __syncthreads();
    }
    if (tid == 0) *s_n = carry;
  }
  __syncthreads();
  tc_fence_after();
  const int n = *s_n;
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S buffers [0,128) [128,256), O [256,384), P buffers (bf16 pairs) [384,448) [448,512)
  const uint32_t S_col = 0, O_col = 256, P_col = 384;

  if (warp == 0) {
    // ------------------------------------------------------------ producers
    // lane 0: Q once, then the K ring; lane 1: the V ring (+ evicted_at of each tile)
    if (lane == 0) {
      mbar_arrive_expect_tx(&bar[B_QFULL], TILE_BYTES);
      tma_load_3d(Qs, &tm_q, 0, h, b * p.T + t0, &bar[B_QFULL]);
      tma_load_3d(Qs + HALF_BYTES, &tm_q, 64, h, b * p.T + t0, &bar[B_QFULL]);
      for (int k = 0; k < n; ++k) {
        const int slot = k & 1;
        if (k >= 2 && !mbar_wait(&bar[B_KEMPTY0 + slot], ((k >> 1) - 1) & 1, abort_flag)) {
          *abort_flag = 1;
          atomicExch(p.error, 1);
          break;
        }
        const int row = b * p.T + (list[k] & 0x7fff) * BN;
        uint8_t* Ks = smem + OFF_K + slot * TILE_BYTES;
        mbar_arrive_expect_tx(&bar[B_KFULL0 + slot], TILE_BYTES);
        tma_load_3d(Ks, &tm_k, 0, hk, row, &bar[B_KFULL0 + slot]);
        tma_load_3d(Ks + HALF_BYTES, &tm_k, 64, hk, row, &bar[B_KFULL0 + slot]);
      }
    } else if (lane == 1) {
      for (int k = 0; k < n; ++k) {
        const int slot = k & 1;
        if (k >= 2 && !mbar_wait(&bar[B_VEMPTY0 + slot], ((k >> 1) - 1) & 1, abort_flag)) {
          *abort_flag = 1;
          atomicExch(p.error, 1);
          break;
        }
        const int j = list[k] & 0x7fff;
        const int row = b * p.T + j * BN;
        uint8_t* Vs = smem + OFF_V + slot * TILE_BYTES;
        mbar_arrive_expect_tx(&bar[B_VFULL0 + slot], TILE_BYTES + E_BYTES);
        tma_load_3d(Vs, &tm_v, 0, hk, row, &bar[B_VFULL0 + slot]);
        tma_load_3d(Vs + HALF_BYTES, &tm_v, 64, hk, row, &bar[B_VFULL0 + slot]);
        bulk_load(smem + OFF_E + slot * E_BYTES, p.e32 + (int64_t)b * p.T_pad + j * BN, E_BYTES,
                  &bar[B_VFULL0 + slot]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_QK = idesc_bf16(128, 128, 0);
      constexpr uint32_t ID_PV = idesc_bf16(128, 128, 1);
      // descriptors built once, K16 steps add their byte offset >> 4 (see the head-pair kernel)
      const uint64_t dq = desc_kmajor_sw128(smem_addr(Qs));
      const uint64_t dk0 = desc_kmajor_sw128(smem_addr(smem + OFF_K));
      const uint64_t dk1 = desc_kmajor_sw128(smem_addr(smem + OFF_K + TILE_BYTES));
      const uint64_t dv0 = desc_mnmajor_sw128(smem_addr(smem + OFF_V), HALF_BYTES);
      const uint64_t dv1 = desc_mnmajor_sw128(smem_addr(smem + OFF_V + TILE_BYTES), HALF_BYTES);
      bool ok = mbar_wait(&bar[B_QFULL], 0, abort_flag);
      for (int k = 0; ok && k <= n; ++k) {
        if (k < n) {
          const int slot = k & 1;
          ok = mbar_wait_fast(&bar[B_KFULL0 + slot], (k >> 1) & 1, abort_flag);
          if (ok && k >= 2) ok = mbar_wait_fast(&bar[B_SFREE0 + slot], ((k >> 1) - 1) & 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint64_t b = slot ? dk1 : dk0;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = ((kk >> 2) * HALF_BYTES + (kk & 3) * 32) >> 4;
            umma_bf16(tmem + S_col + slot * 128, dq + off, b + off, ID_QK, kk > 0);
          }
          umma_commit(&bar[B_KEMPTY0 + slot]);
          umma_commit(&bar[B_SFULL0 + slot]);
        }
        if (k >= 1) {
          const int pk = k - 1, ps = pk & 1;
          ok = mbar_wait_fast(&bar[B_PFULL0 + ps], (pk >> 1) & 1, abort_flag);
          if (ok) ok = mbar_wait_fast(&bar[B_VFULL0 + ps], (pk >> 1) & 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint64_t b = ps ? dv1 : dv0;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // A = P from TMEM: 16 keys = 8 columns per step
            umma_bf16_tmem_a(tmem + O_col, tmem + P_col + ps * 64 + kk * 8, b + ((kk * 2048) >> 4), ID_PV,
                             (pk > 0 || kk > 0));
          umma_commit(&bar[B_VEMPTY0 + ps]);
          umma_commit(&bar[B_PVDONE0 + ps]);
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(p.error, 2);
      }
      // every issued UMMA has finished before TMEM is released
      umma_commit(&bar[B_FINAL]);
      mbar_wait(&bar[B_FINAL], 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------ softmax
    // 8 warps; warps w and w+4 share TMEM lane quadrant w%4 (32 query rows).  The first of
    // the pair owns key / output columns 0..63 of those rows, the second 64..127; the row
    // maximum is exchanged through shared memory once per key tile.
    const int sw = warp - 2;
    const int quad = warp & 3;
    const int half = sw >> 2;
    const int cbase = half * 64;
    const int r = quad * 32 + lane;
    const int t = t0 + r;
    const bool real = t < L;
    const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
    const float sl2 = p.scale_log2;
    float* red = reinterpret_cast<float*>(smem + OFF_RED);  // [2 tiles][2 halves][128 rows]
    float m = -INFINITY, l = 0.f;  // l: this half's partial row sum
    // `ok` stays warp-uniform; after a timeout a thread keeps passing the named barrier once
    // per tile (so its partner warp is never left waiting) but does no further work.
    bool ok = true;
    for (int k = 0; k < n; ++k) {
      const int slot = k & 1;
      const int j = list[k] & 0x7fff;
      const bool masked = (list[k] >> 15) & 1;
      const int s0 = j * BN + cbase;
      if (ok) ok = mbar_wait_fast(&bar[B_SFULL0 + slot], (k >> 1) & 1, abort_flag);
      // evicted_at of the tile arrives with its V slot, which outlives this softmax step
      if (ok && masked) ok = mbar_wait(&bar[B_VFULL0 + slot], (k >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      uint32_t v[64];
      if (ok) {
        tc_fence_after();
        tmem_ld32(tl + S_col + slot * 128 + cbase, *reinterpret_cast<uint32_t(*)[32]>(v));
        tmem_ld32(tl + S_col + slot * 128 + cbase + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&bar[B_SFREE0 + slot]);
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = 0xff800000u;
      }
      if (masked) {
        // key i (of this half) is visible to row t iff i <= t - s0 and t < evicted_at (real
        // rows), or i == t - s0 (padded rows); hidden scores become -inf, branch-free
        const int lim = t - s0;
        const int4* E4 = reinterpret_cast<const int4*>(smem + OFF_E + slot * E_BYTES + cbase * 4);
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int4 e = E4[q];
          const int ev[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = 4 * q + u;
            const bool vis = (i <= lim) && (real ? (t < ev[u]) : (i >= lim));
            v[i] = vis ? v[i] : 0xff800000u;
          }
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; i += 4) {
        mx0 = fmaxf(mx0, __uint_as_float(v[i]));
        mx1 = fmaxf(mx1, __uint_as_float(v[i + 1]));
        mx2 = fmaxf(mx2, __uint_as_float(v[i + 2]));
        mx3 = fmaxf(mx3, __uint_as_float(v[i + 3]));
      }
      const float mh = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      red[(slot * 2 + half) * BM + r] = mh;
      softmax_bar();
      const float mx = fmaxf(mh, red[(slot * 2 + (half ^ 1)) * BM + r]) * sl2;  // sl2 > 0: max commutes
      float alpha = 1.f;
      bool rescale = false;
      if (m == -INFINITY) {
        m = mx;
      } else if (mx > m + 8.f) {  // lazy rescale: exact, p <= 2^8 in between
        alpha = ex2_approx(m - mx);
        m = mx;
        rescale = true;
      }
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      uint32_t pk[32];  // bf16 pairs of this half's probabilities
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int i = 0; i < 64; i += 4) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(v[i]), sl2, neg_m));
        const float p1 = ex2_approx(fmaf(__uint_as_float(v[i + 1]), sl2, neg_m));
        const float p2 = ex2_approx(fmaf(__uint_as_float(v[i + 2]), sl2, neg_m));
        const float p3 = ex2_approx(fmaf(__uint_as_float(v[i + 3]), sl2, neg_m));
        a0 += p0;
        a1 += p1;
        a2 += p2;
        a3 += p3;
        pk[i >> 1] = pack2(p0, p1);
        pk[(i >> 1) + 1] = pack2(p2, p3);
      }
      l = l * alpha + ((a0 + a1) + (a2 + a3));
      // P buffer `slot` was last read by the P V of tile k-2; a rescale of O additionally
      // needs the P V of tile k-1 (the other buffer) to have landed in O
      const bool any_rescale = __any_sync(0xffffffffu, rescale);
      if (ok && k >= 2) ok = mbar_wait_fast(&bar[B_PVDONE0 + slot], ((k >> 1) - 1) & 1, abort_flag);
      if (ok && k >= 1 && any_rescale)
        ok = mbar_wait_fast(&bar[B_PVDONE0 + (slot ^ 1)], ((k - 1) >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) continue;
      tc_fence_after();
      // bf16 P of this half's 64 keys -> 32 TMEM columns of P buffer `slot`
      tmem_st32(tl + P_col + slot * 64 + half * 32, pk);
      if (any_rescale) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32(tl + O_col + cbase + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tl + O_col + cbase + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar[B_PFULL0 + slot]);
    }
    if (ok) ok = mbar_wait(&bar[B_PVDONE0 + ((n - 1) & 1)], ((n - 1) >> 1) & 1, abort_flag);
    // full row sum from the two halves (buffer n&1 was last read at tile n-2)
    red[((n & 1) * 2 + half) * BM + r] = l;
    softmax_bar();
    const float lsum = l + red[((n & 1) * 2 + (half ^ 1)) * BM + r];
    if (ok && half == 0 && p.lse != nullptr && t < p.T) p.lse[((int64_t)b * p.Hq + h) * p.T_pad + t] = m + log2f(lsum);
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.error, 3);
    } else {
      tc_fence_after();
      const float inv = 1.f / lsum;
      __nv_bfloat16* orow = p.out + (((int64_t)b * p.T + t) * p.Hq + h) * HD + cbase;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        tmem_ld32(tl + O_col + cbase + c * 32, o);
        tmem_wait_ld();
        if (t < p.T) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            dst[q4] = make_uint4(pack2(__uint_as_float(o[8 * q4]) * inv, __uint_as_float(o[8 * q4 + 1]) * inv),
                                 pack2(__uint_as_float(o[8 * q4 + 2]) * inv, __uint_as_float(o[8 * q4 + 3]) * inv),
                                 pack2(__uint_as_float(o[8 * q4 + 4]) * inv, __uint_as_float(o[8 * q4 + 5]) * inv),
                                 pack2(__uint_as_float(o[8 * q4 + 6]) * inv, __uint_as_float(o[8 * q4 + 7]) * inv));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ head-pair kernel
// CTA = (stream b, KV head, 128-query tile, pair of query heads h0, h0+1 of the GQA group).
// Both heads see the same positions, hence the same mask and the same key-tile list, so
// each K/V tile staged in shared memory feeds four UMMA tiles.  Roles (384 threads):
//   warpgroup 0   warp 0 TMA producer (lane 0: both Q tiles, then the K ring; lane 1: the
//                 V ring with each tile's evicted_at values); warp 1 TMEM owner + UMMA
//                 issuer; warps 2-3 idle.  Registers trimmed to 56 per thread.
//   warpgroup 1   softmax of head h0: one thread per query row (TMEM lane), all 128 key
//                 columns of the row in registers, so no cross-warp reduction;
//   warpgroup 2   softmax of head h0+1.  Both at 224 registers per thread.
// TMEM: S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512).  The bf16 probabilities
// P_t overwrite the first 64 columns of S_t once the row is in registers.
// UMMA issue order per key tile k:  S0(k), P1(k-1) V(k-1), S1(k), P0(k) V(k).  tcgen05.mma
// ops of one thread run in issue order, so S_t(k+1) is issued right behind the P_t V
// that reads the columns it overwrites, and the commit that signals S_t(k+1) also
// covers that P V: softmax t may rescale O_t as soon as S_t(k+1) is signalled.
constexpr int NT2 = 384;
constexpr int REGS_CTRL = 56, REGS_SOFT = 224;
static_assert(REGS_CTRL * 128 + REGS_SOFT * 256 <= 168 * NT2, "register split exceeds the launch budget");
constexpr int OFF2_Q = 0;                          // 2 query tiles
constexpr int OFF2_K = OFF2_Q + 2 * TILE_BYTES;    // 2 slots
constexpr int OFF2_V = OFF2_K + 2 * TILE_BYTES;    // 2 slots
constexpr int OFF2_E = OFF2_V + 2 * TILE_BYTES;    // 2 slots of 128 int32
constexpr int OFF2_LIST = OFF2_E + 2 * E_BYTES;
constexpr int OFF2_ROWS = OFF2_LIST + MAX_KT * 2;  // paged: pool row of each 16-key block of the list
constexpr int OFF2_BAR = OFF2_ROWS + MAX_KT * (BN / 16) * 4;
constexpr int NBAR2 = 16;
constexpr int OFF2_MISC = OFF2_BAR + NBAR2 * 8;
constexpr int SMEM2_BYTES = OFF2_MISC + 64 + 33 * 4 + 1024;
static_assert(SMEM2_BYTES <= 232448, "head-pair replay kernel shared memory");
static_assert(232448 + 1024 < (1 << 18), "descriptor start-address field (addr >> 4, 14 bits) must not carry");

// descriptor start-address offsets (bytes >> 4) of K16 step kk: for a K-major 128x128 tile,
// half kk/4 (16 KB apart) and 32 bytes into the 128-byte swizzled row; for the MN-major V
// tile, rows 16kk.. (2 KB per step).  P supplies 8 TMEM columns (bf16 pairs) per step.
__host__ __device__ constexpr uint32_t s_step(int kk) { return (uint32_t)(((kk >> 2) * HALF_BYTES + (kk & 3) * 32) >> 4); }
__host__ __device__ constexpr uint32_t pv_step(int kk) { return (uint32_t)((kk * 2048) >> 4); }

enum { C_KFULL0 = 0, C_KFULL1, C_VFULL0, C_VFULL1, C_KEMPTY0, C_KEMPTY1, C_VEMPTY0, C_VEMPTY1, C_QFULL,
       C_SFULL0, C_SFULL1, C_PFULL0, C_PFULL1, C_FINAL, C_VCONV0, C_VCONV1 };
constexpr int NCONV = 64;  // warps 2 and 3: V tiles to f16 in place

template <bool PAGED>
__global__ void __launch_bounds__(NT2, 1)
pair_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const ReplayParams p, const PagedParams g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Qs = smem + OFF2_Q;
  uint16_t* list = reinterpret_cast<uint16_t*>(smem + OFF2_LIST);  // key tile | 0x8000 if masked
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF2_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF2_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF2_MISC + 4);
  int* s_n = reinterpret_cast<int*>(smem + OFF2_MISC + 8);
  int* s_scan = reinterpret_cast<int*>(smem + OFF2_MISC + 64);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // a bounded wait that expired: replay reports the site in its error word, the paged path
  // in the cache's status words (KVS_ST_KERNEL_TIMEOUT, site, CTA)
  auto fail_site = [&](int site) {
    if (PAGED)
      set_status(g.status, KVS_ST_KERNEL_TIMEOUT, site, (int)blockIdx.x, 0);
    else
      atomicExch(p.error, site);
  };
  const int G = p.Hq / p.Hkv, GP = G >> 1;
  int gp, hk, qt, b = 0, t0 = 0, t1 = 0, L = 0;  // replay: stream b, query rows t0..t1, length L
  int seq_slot = 0, tok0 = 0, Ti = 0, n_all = 0, n_past = 0;  // paged: cache slot, new tokens, live entries
  int q_row0;  // TMA row of the tile's first query
  if (!PAGED) {
    // CTA order: (stream, KV head) slowest, then query tiles heaviest first, then head pairs
    gp = (int)(blockIdx.x % GP);
    const int rest = (int)(blockIdx.x / GP);
    qt = p.n_qt - 1 - rest % p.n_qt;
    const int bhk = rest / p.n_qt;
    b = bhk / p.Hkv;
    hk = bhk % p.Hkv;
    t0 = qt * BM;
    t1 = t0 + BM - 1;
    L = p.lengths[b];
    q_row0 = b * p.T + t0;
  } else {
    // CTA order: query tiles of the batch (sequence by sequence) slowest, then KV head, then
    // head pairs.  The grid is an upper bound on the number of tiles; surplus CTAs leave here.
    gp = (int)(blockIdx.x % GP);
    hk = (int)((blockIdx.x / GP) % p.Hkv);
    const int item = (int)(blockIdx.x / (GP * p.Hkv));
    if (item >= g.cu_qt[g.num_seqs]) return;
    int lo = 0, hi = g.num_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (g.cu_qt[mid] <= item) lo = mid; else hi = mid - 1;
    }
    qt = item - g.cu_qt[lo];
    seq_slot = g.seq_slots[lo];
    tok0 = g.cu_tokens[lo];
    Ti = g.cu_tokens[lo + 1] - tok0;
    n_all = g.lengths[seq_slot];
    n_past = n_all - Ti;
    q_row0 = tok0 + qt * BM;
    if ((n_all + BN - 1) / BN > MAX_KT) {  // the key-tile list holds MAX_KT tiles
      if (tid == 0) set_status(g.status, KVS_ST_SEQ_TOO_LONG, seq_slot, n_all, 0);
      return;
    }
  }
  const int h0 = hk * G + 2 * gp;

  if (tid == 0) {
    for (int i = 0; i < NBAR2; ++i) mbar_init(&bar[i], 1);
    mbar_init(&bar[C_PFULL0], 128);
    mbar_init(&bar[C_PFULL1], 128);
    mbar_init(&bar[C_VCONV0], NCONV);
    mbar_init(&bar[C_VCONV1], NCONV);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }

  // ---- active key tiles for this query tile (same list for every role).  Replay: tiles
  // up to the diagonal, skipping those every key of which was evicted before the first
  // query.  Paged: every tile up to the last visible key of the tile's last query; masked
  // where the causal limit or the end of the sequence cuts through.
  {
    const int real_last = min(t1, L - 1);
    const int jlast = PAGED ? (n_past + min(qt * BM + BM - 1, Ti - 1)) / BN : qt;
    int carry = 0;
    for (int base = 0; base <= jlast; base += NT2) {
      const int j = base + tid;
      int flag = 0;
      if (j <= jlast) {
        if (PAGED) {
          const bool masked = (j * BN + BN - 1 > n_past + qt * BM) || (j * BN + BN > n_all);
          flag = 1 | (masked ? 2 : 0);
        } else {
          const int emin = p.tile_min[b * p.n_kt + j], emax = p.tile_max[b * p.n_kt + j];
          const bool active = (j == qt) || (j * BN <= real_last && emax > t0);
          const bool masked = (j == qt) || (emin <= t1) || (t1 >= L);
          flag = (active ? 1 : 0) | (masked ? 2 : 0);
        }
      }
      int tot = 0;
      const int pre = block_exclusive_scan(flag & 1, s_scan, &tot);
      if (flag & 1) list[carry + pre] = (uint16_t)(j | ((flag & 2) ? 0x8000 : 0));
      carry += tot;
      __syncthreads();
    }
    if (tid == 0) *s_n = carry;
  }
  __syncthreads();
  const int n = *s_n;  // >= 1: the diagonal tile is always active
  int* rows = reinterpret_cast<int*>(smem + OFF2_ROWS);
  if (PAGED) {
    // pool rows of every block the producer will gather, read once by all threads (its loads
    // then issue back to back); blocks past the sequence read past the pool, i.e. zeros
    for (int e = tid; e < n * (BN / 16); e += NT2) {
      const int j = list[e >> 3] & 0x7fff, b8 = e & 7;
      rows[e] = (j * BN + b8 * 16 < n_all)
                    ? g.tables[(int64_t)seq_slot * g.max_blocks + j * (BN / 16) + b8] * 16
                    : g.pool_rows;
    }
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // one 128-key x 128-dim tile of K or V into a 128-byte swizzled shared tile: replay rows
  // are contiguous; paged keys come as eight 16-token pool blocks (2 KB per half each),
  // and blocks past the sequence are read out of bounds of the pool, i.e. as zeros.
  auto load_kv = [&](uint8_t* dst, const CUtensorMap* map, int k, uint64_t* bb) {
    if (!PAGED) {
      const int row = b * p.T + (list[k] & 0x7fff) * BN;
      tma_load_3d(dst, map, 0, hk, row, bb);
      tma_load_3d(dst + HALF_BYTES, map, 64, hk, row, bb);
    } else {
      const int* r8 = rows + k * (BN / 16);
#pragma unroll
      for (int b8 = 0; b8 < BN / 16; ++b8) {
        tma_load_3d(dst + b8 * 2048, map, 0, hk, r8[b8], bb);
        tma_load_3d(dst + HALF_BYTES + b8 * 2048, map, 64, hk, r8[b8], bb);
      }
    }
  };

  if (warp < 4) {
    regs_dealloc<REGS_CTRL>();
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------- producer: Q tiles, K ring
      mbar_arrive_expect_tx(&bar[C_QFULL], 2 * TILE_BYTES);
      for (int t = 0; t < 2; ++t) {
        tma_load_3d(Qs + t * TILE_BYTES, &tm_q, 0, h0 + t, q_row0, &bar[C_QFULL]);
        tma_load_3d(Qs + t * TILE_BYTES + HALF_BYTES, &tm_q, 64, h0 + t, q_row0, &bar[C_QFULL]);
      }
      for (int k = 0; k < n; ++k) {
        const int ks = k & 1;
        if (k >= 2 && !mbar_wait(&bar[C_KEMPTY0 + ks], ((k >> 1) - 1) & 1, abort_flag)) {
          *abort_flag = 1;
          fail_site(1);
          break;
        }
        uint8_t* Ks = smem + OFF2_K + ks * TILE_BYTES;
        mbar_arrive_expect_tx(&bar[C_KFULL0 + ks], TILE_BYTES);
        load_kv(Ks, &tm_k, k, &bar[C_KFULL0 + ks]);
      }
    } else if (warp == 0 && lane == 1) {
      // ---------------------------------------------------------- producer: V ring + evicted_at
      for (int k = 0; k < n; ++k) {
        const int vs = k & 1;
        if (k >= 2 && !mbar_wait(&bar[C_VEMPTY0 + vs], ((k >> 1) - 1) & 1, abort_flag)) {
          *abort_flag = 1;
          fail_site(1);
          break;
        }
        const int j = list[k] & 0x7fff;
        uint8_t* Vs = smem + OFF2_V + vs * TILE_BYTES;
        mbar_arrive_expect_tx(&bar[C_VFULL0 + vs], TILE_BYTES + (PAGED ? 0 : E_BYTES));
        load_kv(Vs, &tm_v, k, &bar[C_VFULL0 + vs]);
        if (!PAGED)
          bulk_load(smem + OFF2_E + vs * E_BYTES, p.e32 + (int64_t)b * p.T_pad + j * BN, E_BYTES,
                    &bar[C_VFULL0 + vs]);
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------- UMMA issuer (whole warp,
      // one elected lane issues; every value on this path is warp-uniform)
      constexpr uint32_t ID_QK = idesc_bf16(128, 128, 0);
      constexpr uint32_t ID_PV = idesc_f16(128, 128, 1);  // P and V in f16
      // Descriptors are built once; each K16 step adds its byte offset >> 4 to the start-address
      // field (no carry: shared addresses stay below 2^18).
      const uint64_t dq0 = desc_kmajor_sw128(smem_addr(Qs)), dq1 = desc_kmajor_sw128(smem_addr(Qs + TILE_BYTES));
      const uint64_t dk0 = desc_kmajor_sw128(smem_addr(smem + OFF2_K));
      const uint64_t dk1 = desc_kmajor_sw128(smem_addr(smem + OFF2_K + TILE_BYTES));
      const uint64_t dv0 = desc_mnmajor_sw128(smem_addr(smem + OFF2_V), HALF_BYTES);
      const uint64_t dv1 = desc_mnmajor_sw128(smem_addr(smem + OFF2_V + TILE_BYTES), HALF_BYTES);
      // S_t = Q_t K^T (8 x K16 steps over the two 64-column halves)
      auto issue_s = [&](int t, int slot) {
        const uint64_t a = t ? dq1 : dq0, b = slot ? dk1 : dk0;
        const uint32_t d = tmem + t * 128;
#define KVS_S_STEP(kk) umma_bf16_warp_at<s_step(kk), s_step(kk)>(d, a, b, ID_QK, kk > 0)
        KVS_S_STEP(0); KVS_S_STEP(1); KVS_S_STEP(2); KVS_S_STEP(3);
        KVS_S_STEP(4); KVS_S_STEP(5); KVS_S_STEP(6); KVS_S_STEP(7);
#undef KVS_S_STEP
      };
      // O_t (+)= P_t V: P_t from TMEM (16 keys = 8 columns per step), V MN-major
      auto issue_pv = [&](int t, int slot, bool acc) {
        const uint64_t b = slot ? dv1 : dv0;
        const uint32_t d = tmem + 256 + t * 128, a = tmem + t * 128;
#define KVS_PV_STEP(kk) umma_bf16_tmem_a_warp_at<kk * 8, pv_step(kk)>(d, a, b, ID_PV, (kk > 0) || acc)
        KVS_PV_STEP(0); KVS_PV_STEP(1); KVS_PV_STEP(2); KVS_PV_STEP(3);
        KVS_PV_STEP(4); KVS_PV_STEP(5); KVS_PV_STEP(6); KVS_PV_STEP(7);
#undef KVS_PV_STEP
      };
      // all lanes poll; `ok` is made warp-uniform after every wait
      auto wait = [&](uint64_t* b, int parity) {
        return __all_sync(0xffffffffu, mbar_wait_fast(b, parity, abort_flag));
      };
      bool ok = __all_sync(0xffffffffu, mbar_wait(&bar[C_QFULL], 0, abort_flag));
      for (int k = 0; ok && k < n; ++k) {
        const int slot = k & 1, ph = (k >> 1) & 1;
        ok = wait(&bar[C_KFULL0 + slot], ph);
        if (!ok) break;
        tc_fence_after();
        issue_s(0, slot);
        umma_commit_warp(&bar[C_SFULL0]);
        if (k >= 1) {
          ok = wait(&bar[C_PFULL1], (k - 1) & 1);
          if (!ok) break;
          tc_fence_after();
          issue_pv(1, slot ^ 1, k > 1);
          umma_commit_warp(&bar[C_VEMPTY0 + (slot ^ 1)]);
        }
        issue_s(1, slot);
        umma_commit_warp(&bar[C_KEMPTY0 + slot]);
        umma_commit_warp(&bar[C_SFULL1]);
        // V(k) normally landed (and was converted to f16) long ago: take its wait before head
        // 0's P, which is on the softmax -> P V -> S critical path
        ok = wait(&bar[C_VCONV0 + slot], ph);
        if (ok) ok = wait(&bar[C_PFULL0], k & 1);
        if (!ok) break;
        tc_fence_after();
        issue_pv(0, slot, k > 0);
      }
      if (ok) {
        ok = wait(&bar[C_PFULL1], (n - 1) & 1);
        if (ok) {
          tc_fence_after();
          issue_pv(1, (n - 1) & 1, n > 1);
        }
      }
      if (!ok && lane == 0) {
        *abort_flag = 1;
        fail_site(2);
      }
      // every issued UMMA has finished before the softmax warps read O and TMEM is released
      umma_commit_warp(&bar[C_FINAL]);
      mbar_wait(&bar[C_FINAL], 0, nullptr);
      __syncwarp();
    } else if (warp >= 2) {
      // ---------------------------------------------------------- warps 2, 3: each V tile to f16
      // in place once it lands, for the f16 P V products (P keeps 11 significant bits instead
      // of bf16's 8, so the replay and the paged decode agree far more closely).  The swizzled
      // layout is unchanged: every 16-byte chunk is converted where it lies.
      const int ct = tid - 64;
      bool ok = true;
      for (int k = 0; k < n; ++k) {
        const int vs = k & 1;
        ok = mbar_wait(&bar[C_VFULL0 + vs], (k >> 1) & 1, abort_flag);
        if (!ok) break;
        uint4* v4 = reinterpret_cast<uint4*>(smem + OFF2_V + vs * TILE_BYTES);
#pragma unroll 2
        for (int c = ct; c < TILE_BYTES / 16; c += NCONV) {
          uint4 x = v4[c];
          x.x = bf16x2_to_f16x2(x.x);
          x.y = bf16x2_to_f16x2(x.y);
          x.z = bf16x2_to_f16x2(x.z);
          x.w = bf16x2_to_f16x2(x.w);
          v4[c] = x;
        }
        fence_proxy_async_smem();  // the UMMA reads the tile through the async proxy
        mbar_arrive(&bar[C_VCONV0 + vs]);
      }
      if (!ok) {
        *abort_flag = 1;
        fail_site(4);
      }
    }
  } else {
    regs_alloc<REGS_SOFT>();
    // ------------------------------------------------------------ softmax of head h0 + team
    const int team = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int t = t0 + r;  // replay: query position
    const bool real = t < L;
    const int ci = qt * BM + r;                              // paged: index among the new tokens
    const int qidx = (ci < Ti) ? n_past + ci : -1;           // paged: last visible key (-1: no row)
    const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t S_col = team * 128, O_col = 256 + team * 128;
    uint64_t* sfull = &bar[C_SFULL0 + team];
    uint64_t* pfull = &bar[C_PFULL0 + team];
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int k = 0; k < n; ++k) {
      const int slot = k & 1;
      const int j = list[k] & 0x7fff;
      const bool masked = (list[k] >> 15) & 1;
      ok = mbar_wait_fast(sfull, k & 1, abort_flag);
      // evicted_at of the tile arrives with its V slot, which outlives both softmax steps
      if (!PAGED && ok && masked) ok = mbar_wait_fast(&bar[C_VFULL0 + slot], (k >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t v[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tl + S_col + c * 32, *reinterpret_cast<uint32_t(*)[32]>(v + c * 32));
      tmem_wait_ld();
      if (masked) {
        // key i is visible to row t iff i <= t - j*BN and t < evicted_at (real rows), or
        // i == t - j*BN (padded rows).  The 128 visibility bits are gathered into four words
        // first (so the tile's evicted_at values are never all live in registers at once),
        // then hidden scores become -inf, branch-free.
        uint32_t bits[4];
        if (PAGED) {
          // key i of the tile is visible iff j*BN + i <= qidx (a prefix of the tile)
          const int lim = qidx - j * BN;
#pragma unroll
          for (int w = 0; w < 4; ++w)
            bits[w] = lim >= 32 * w + 31 ? 0xffffffffu : (lim < 32 * w ? 0u : (2u << (lim - 32 * w)) - 1u);
        } else {
          const int lim = t - j * BN;
          const int4* E4 = reinterpret_cast<const int4*>(smem + OFF2_E + slot * E_BYTES);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            uint32_t bw = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const int4 e = E4[w * 8 + q];
              const int ev[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int i = 32 * w + 4 * q + u;
                const bool vis = (i <= lim) && (real ? (t < ev[u]) : (i >= lim));
                bw |= (vis ? 1u : 0u) << (4 * q + u);
              }
            }
            bits[w] = bw;
          }
        }
#pragma unroll
        for (int i = 0; i < 128; ++i) v[i] = ((bits[i >> 5] >> (i & 31)) & 1) ? v[i] : 0xff800000u;
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; i += 8) {
        mx0 = fmax3(mx0, __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
        mx1 = fmax3(mx1, __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
        mx2 = fmax3(mx2, __uint_as_float(v[i + 4]), __uint_as_float(v[i + 5]));
        mx3 = fmax3(mx3, __uint_as_float(v[i + 6]), __uint_as_float(v[i + 7]));
      }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;  // sl2 > 0: max commutes
      float alpha = 1.f;
      bool rescale = false;
      if (m == -INFINITY) {
        m = mx;
      } else if (mx > m + 8.f) {  // lazy rescale: exact, p <= 2^8 in between
        alpha = ex2_approx(m - mx);
        m = mx;
        rescale = true;
      }
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];  // f16 pairs of keys 32c .. 32c+31
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const int e = 32 * c + i;
          // scale-and-shift and the row sums as packed pairs (one instruction per two keys)
          float x0, x1, x2, x3;
          ffma2(x0, x1, __uint_as_float(v[e]), __uint_as_float(v[e + 1]), sl2, neg_m);
          ffma2(x2, x3, __uint_as_float(v[e + 2]), __uint_as_float(v[e + 3]), sl2, neg_m);
          const float p0 = ex2_approx(x0), p1 = ex2_approx(x1), p2 = ex2_approx(x2), p3 = ex2_approx(x3);
          fadd2(a0, a1, p0, p1);
          fadd2(a2, a3, p2, p3);
          pk[i >> 1] = pack2h(p0, p1);  // p <= 2^8 (lazy rescale): within the f16 range
          pk[(i >> 1) + 1] = pack2h(p2, p3);
        }
        tmem_st16(tl + S_col + c * 16, pk);
      }
      l = l * alpha + ((a0 + a1) + (a2 + a3));
      // O_t holds P V up to tile k-1: its last P V finished before S_t(k) was signalled
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tl + O_col + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tl + O_col + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(pfull);
    }
    if (ok) ok = mbar_wait(&bar[C_FINAL], 0, abort_flag);
    if (!ok) {
      *abort_flag = 1;
      fail_site(3);
    } else {
      tc_fence_after();
      const float inv = 1.f / l;
      if (!PAGED && p.lse != nullptr && t < p.T)
        p.lse[((int64_t)b * p.Hq + h0 + team) * p.T_pad + t] = m + log2f(l);
      const int64_t orow_idx = PAGED ? (int64_t)tok0 + ci : (int64_t)b * p.T + t;
      const bool store = PAGED ? ci < Ti : t < p.T;
      __nv_bfloat16* orow = p.out + (orow_idx * p.Hq + h0 + team) * HD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tl + O_col + c * 32, o);
        tmem_wait_ld();
        if (store) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            dst[q4] = make_uint4(pack2(__uint_as_float(o[8 * q4]) * inv, __uint_as_float(o[8 * q4 + 1]) * inv),
                                 pack2(__uint_as_float(o[8 * q4 + 2]) * inv, __uint_as_float(o[8 * q4 + 3]) * inv),
                                 pack2(__uint_as_float(o[8 * q4 + 4]) * inv, __uint_as_float(o[8 * q4 + 5]) * inv),
                                 pack2(__uint_as_float(o[8 * q4 + 6]) * inv, __uint_as_float(o[8 * q4 + 7]) * inv));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ backward (tcgen05)
// Gradients of the masked replay attention on the tensor cores, bf16, head_dim 128.  With
// the forward's row statistics lse2[b][h][t] = log2 sum_s 2^(scale*log2(e)*q_t.k_s) (written
// by the forward kernels) and D[b][h][t] = sum_d dO O (replay_rowdot_kernel):
//   P = 2^(scale*log2(e)*Q K^T - lse2),  dS = P o (dO V^T - D),
//   dV = P^T dO,  dK = scale dS^T Q,  dQ = scale dS K.
// Two kernels, no atomics: replay_dkdv_kernel owns a 128-key tile of one KV head and loops
// over the query tiles and query heads that see it; replay_dq_kernel owns a 128-query tile
// of one head and loops over its active key tiles (the forward's list).  P and dS are
// rounded to bf16 as UMMA operands (as P is in the forward).

// -lse2 and -D of each (stream, head, row); both kernels add them.  A warp takes four
// consecutive rows of one head, half a warp per row and 16 bytes of dO and of O per lane, with
// every load of a lane (and the rows' lse) issued before the first product: a pure stream of
// dO and O whose outputs land in consecutive words.
constexpr int ROWDOT_PER_WARP = 4;
__global__ void __launch_bounds__(256) replay_rowdot_kernel(const __nv_bfloat16* __restrict__ dout,
                                                            const __nv_bfloat16* __restrict__ o,
                                                            const float* __restrict__ lse, float* __restrict__ nlse,
                                                            float* __restrict__ nd, int B, int T, int T_pad, int Hq) {
  const int nt4 = (T + ROWDOT_PER_WARP - 1) / ROWDOT_PER_WARP;
  const int64_t w = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= (int64_t)B * Hq * nt4) return;
  const int tq = (int)(w % nt4), h = (int)((w / nt4) % Hq), b = (int)(w / ((int64_t)nt4 * Hq));
  const int lane = threadIdx.x & 31, half = lane >> 4, l16 = lane & 15;
  const int64_t vrow = ((int64_t)b * Hq + h) * T_pad;  // this head's row vectors
  uint4 x[ROWDOT_PER_WARP / 2], y[ROWDOT_PER_WARP / 2];
  float ls[ROWDOT_PER_WARP / 2];
#pragma unroll
  for (int it = 0; it < ROWDOT_PER_WARP / 2; ++it) {
    const int t = tq * ROWDOT_PER_WARP + 2 * it + half;
    x[it] = y[it] = make_uint4(0u, 0u, 0u, 0u);
    ls[it] = 0.f;
    if (t < T) {
      const int64_t row = ((int64_t)b * T + t) * Hq + h;
      x[it] = reinterpret_cast<const uint4*>(dout + row * HD)[l16];
      y[it] = reinterpret_cast<const uint4*>(o + row * HD)[l16];
      if (l16 == 0) ls[it] = lse[vrow + t];
    }
  }
#pragma unroll
  for (int it = 0; it < ROWDOT_PER_WARP / 2; ++it) {
    const __nv_bfloat162* xa = reinterpret_cast<const __nv_bfloat162*>(&x[it]);
    const __nv_bfloat162* ya = reinterpret_cast<const __nv_bfloat162*>(&y[it]);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = __bfloat1622float2(xa[e]), c = __bfloat1622float2(ya[e]);
      s += a.x * c.x + a.y * c.y;
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    const int t = tq * ROWDOT_PER_WARP + 2 * it + half;
    if (l16 == 0 && t < T) {
      nd[vrow + t] = -s;
      nlse[vrow + t] = -ls[it];
    }
  }
}

constexpr int NGRP = 4;                 // softmax groups of four warps (one per TMEM lane quadrant)
constexpr int GCOLS = 128 / NGRP;       // columns of S / dP per group
constexpr int NTB = 64 + NGRP * 128;    // warp 0 producers, warp 1 UMMA, then the softmax groups
constexpr int VEC_BYTES = BM * 4;

struct BwdParams {
  const int32_t* e32;       // [B][T_pad] evicted_at clamped to int32 (prepass)
  const int32_t* tile_min;  // [B][n_kt] (prepass)
  const int32_t* tile_max;
  const int32_t* lengths;
  const float* nlse;        // [B][Hq][T_pad] -lse2 (log2 units)
  const float* nd;          // [B][Hq][T_pad] -D
  __nv_bfloat16* dq;        // [B][T][Hq][D]
  __nv_bfloat16* dk;        // [B][T][Hkv][D]
  __nv_bfloat16* dv;
  int32_t* error;
  int B, T, T_pad, Hq, Hkv, n_qt, n_kt;
  float scale_log2, scale;
};

// One arrival per softmax warp: each thread orders its own TMEM / shared writes (fences), the
// warp synchronises, and lane 0 arrives (one arrival per warp instead of one per thread).
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// Both kernels: one thread per TMEM lane (a key row in dK/dV, a query row in dQ) in each of
// NGRP groups of four warps; group g owns columns [32g, 32g + 32) of the 128-wide S and dP
// tiles (16 softmax warps: four per SM sub-partition hide the TMEM and MUFU latencies).  A
// step runs in two phases so that the tensor cores work through the next product while the
// softmax warps compute: phase A turns S into P (kept in fp32 registers) as soon as S lands;
// phase B forms dS = P (dP - D) when dP lands.
//
// Operand tiles of the loop sit in a pool of four 32 KB slots: the tile of step i + 2 takes
// the slot that step i frees first (in dK/dV, Q(i+2) goes where dO(i) was, released by dV(i)
// mid-step, and dO(i+2) where Q(i) was, released by dK(i)), so each load has about a step
// to land; tiles two steps ahead are also prefetched into L2.
__host__ __device__ constexpr int slot_a(int i) { return (0x3120 >> (4 * (i & 3))) & 0xF; }  // 0 2 1 3
__host__ __device__ constexpr int slot_b(int i) { return (0x2031 >> (4 * (i & 3))) & 0xF; }  // 1 3 0 2
static_assert(slot_a(2) == slot_b(0) && slot_a(3) == slot_b(1) && slot_b(2) == slot_a(0) && slot_b(3) == slot_a(1),
              "slot pool: step i + 2 reuses the slots of step i crosswise");

__host__ __device__ constexpr uint32_t kq_step(int kk) { return (uint32_t)(((kk >> 2) * HALF_BYTES + (kk & 3) * 32) >> 4); }
__host__ __device__ constexpr uint32_t mn_step(int kk) { return (uint32_t)((kk * 2048) >> 4); }
// TMEM column of K step kk (16 rows of the K dimension = 8 packed columns) when group g packed
// its 32 bf16 values into columns [32g, 32g + 16) of a 128-column region
__host__ __device__ constexpr uint32_t split_col(int kk) { return (uint32_t)((kk >> 1) * GCOLS + (kk & 1) * 8); }

// smem of the dK/dV kernel (the dynamic shared base is 1024-aligned: no padding; the host
// checks that once per device before the first launch)
constexpr int OFFB_K = 0, OFFB_V = TILE_BYTES;
constexpr int OFFB_SLOT = 2 * TILE_BYTES;             // 4 slots: Q and dO tiles of the loop
constexpr int OFFB_P = OFFB_SLOT + 4 * TILE_BYTES;    // P^T bf16, K-major 128B-swizzled (UMMA A of dV)
constexpr int OFFB_LSE = OFFB_P + TILE_BYTES;         // 2 slots of 128 f32 (-lse2), loaded with dO
constexpr int OFFB_D = OFFB_LSE + 2 * VEC_BYTES;      // 2 slots of 128 f32 (-D), loaded with dO
constexpr int OFFB_BAR = OFFB_D + 2 * VEC_BYTES;
enum {
  D_KVFULL = 0, D_FULL0, D_EMPTY0 = D_FULL0 + 4, D_SFULL = D_EMPTY0 + 4, D_SREAD, D_PFULL, D_PEMPTY, D_DPFULL,
  D_DSFULL, D_FINAL, NBARB
};
constexpr int OFFB_MISC = OFFB_BAR + NBARB * 8;
constexpr int SMEMB_BYTES = OFFB_MISC + 16;
static_assert(SMEMB_BYTES <= 232448, "dK/dV kernel shared memory");

__global__ void __launch_bounds__(NTB, 1)
replay_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                   const BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_bwd[];
  uint8_t* smem = smem_bwd;
  if (smem_addr(smem) & 1023) {  // never expected (the host checked); no work, no TMEM
    if (threadIdx.x == 0) atomicExch(p.error, 15);
    return;
  }
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFFB_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFFB_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFFB_MISC + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // CTA order: blocks of up to eight (stream, KV head) pairs slowest; inside a block, key tiles
  // ascending (an early tile is seen by the most query tiles, so the longest CTAs start
  // first) and the pairs innermost.  The CTAs in flight then cover a few heads and nearby key
  // tiles, whose query tiles they share in L2.
  const int G = p.Hq / p.Hkv;
  const int nbh = p.B * p.Hkv;
  const int blk = (int)(blockIdx.x / (8 * p.n_kt));
  const int in_blk = (int)(blockIdx.x % (8 * p.n_kt));
  const int bw = min(8, nbh - blk * 8);
  const int kt = in_blk / bw;
  const int bhk = blk * 8 + in_blk % bw;
  const int b = bhk / p.Hkv, hk = bhk % p.Hkv;
  const int k0 = kt * BN;
  const int L = p.lengths[b];
  // query tiles that see a key of this tile: from the diagonal to the last row any key's
  // interval [s, min(evicted_at[s], L)) reaches (padded rows see only themselves, on the diagonal)
  const int reach = min(p.tile_max[b * p.n_kt + kt], L);
  const int qlast = max(kt, min(p.n_qt - 1, (reach - 1) / BM));
  const int nsteps = (qlast - kt + 1) * G;  // step i: query tile kt + i / G, query head hk * G + i % G

  if (tid == 0) {
    for (int i = 0; i < NBARB; ++i) mbar_init(&bar[i], 1);
    mbar_init(&bar[D_SREAD], 4 * NGRP);
    mbar_init(&bar[D_PFULL], 4 * NGRP);
    mbar_init(&bar[D_DSFULL], 4 * NGRP);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM: S^T [0,128), dP^T [128,256) (dS^T bf16 of group g over [128+32g, +16)), dV [256,384),
  // dK [384,512).  P^T goes to shared memory, so S^T(i+1) is computed while the softmax warps
  // still work on step i.

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- K, V; the Q tiles
      mbar_arrive_expect_tx(&bar[D_KVFULL], 2 * TILE_BYTES);
      tma_load_3d(smem + OFFB_K, &tm_k, 0, hk, b * p.T + k0, &bar[D_KVFULL]);
      tma_load_3d(smem + OFFB_K + HALF_BYTES, &tm_k, 64, hk, b * p.T + k0, &bar[D_KVFULL]);
      tma_load_3d(smem + OFFB_V, &tm_v, 0, hk, b * p.T + k0, &bar[D_KVFULL]);
      tma_load_3d(smem + OFFB_V + HALF_BYTES, &tm_v, 64, hk, b * p.T + k0, &bar[D_KVFULL]);
      for (int i = 0; i < nsteps; ++i) {
        const int sl = slot_a(i);
        if (i >= 2 && !mbar_wait(&bar[D_EMPTY0 + sl], ((i >> 1) - 1) & 1, abort_flag)) {
          *abort_flag = 1;
          atomicExch(p.error, 11);
          break;
        }
        const int row = b * p.T + (kt + i / G) * BM, h = hk * G + i % G;
        uint64_t* fb = &bar[D_FULL0 + sl];
        mbar_arrive_expect_tx(fb, TILE_BYTES);
        uint8_t* qs = smem + OFFB_SLOT + sl * TILE_BYTES;
        tma_load_3d(qs, &tm_q, 0, h, row, fb);
        tma_load_3d(qs + HALF_BYTES, &tm_q, 64, h, row, fb);
        if (i + 2 < nsteps) {
          const int row2 = b * p.T + (kt + (i + 2) / G) * BM, h2 = hk * G + (i + 2) % G;
          tma_prefetch_3d(&tm_q, 0, h2, row2);
          tma_prefetch_3d(&tm_q, 64, h2, row2);
        }
      }
    } else if (lane == 1) {
      // ---------------------------------------------------------- the dO tiles (+ -lse2, -D)
      for (int i = 0; i < nsteps; ++i) {
        const int sl = slot_b(i);
        if (i >= 2 && !mbar_wait(&bar[D_EMPTY0 + sl], ((i >> 1) - 1) & 1, abort_flag)) {
          *abort_flag = 1;
          atomicExch(p.error, 14);
          break;
        }
        const int qt = kt + i / G, h = hk * G + i % G;
        const int row = b * p.T + qt * BM;
        uint64_t* fb = &bar[D_FULL0 + sl];
        mbar_arrive_expect_tx(fb, TILE_BYTES + 2 * VEC_BYTES);
        uint8_t* ds = smem + OFFB_SLOT + sl * TILE_BYTES;
        tma_load_3d(ds, &tm_do, 0, h, row, fb);
        tma_load_3d(ds + HALF_BYTES, &tm_do, 64, h, row, fb);
        const int64_t vo = ((int64_t)b * p.Hq + h) * p.T_pad + qt * BM;
        bulk_load(smem + OFFB_LSE + (i & 1) * VEC_BYTES, p.nlse + vo, VEC_BYTES, fb);
        bulk_load(smem + OFFB_D + (i & 1) * VEC_BYTES, p.nd + vo, VEC_BYTES, fb);
        if (i + 2 < nsteps) {
          const int row2 = b * p.T + (kt + (i + 2) / G) * BM, h2 = hk * G + (i + 2) % G;
          tma_prefetch_3d(&tm_do, 0, h2, row2);
          tma_prefetch_3d(&tm_do, 64, h2, row2);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- UMMA issuer (whole warp)
    // per step i: S^T(i+1) once S^T(i) is read; dV += P^T(i) dO(i); dK += dS^T(i) Q(i); dP^T(i+1)
    constexpr uint32_t ID_T = idesc_bf16(128, 128, 0);   // S^T, dP^T: both operands K-major
    constexpr uint32_t ID_MN = idesc_bf16(128, 128, 1);  // dV, dK: B (dO, Q) MN-major
    const uint64_t dk_ = desc_kmajor_sw128(smem_addr(smem + OFFB_K));
    const uint64_t dv_ = desc_kmajor_sw128(smem_addr(smem + OFFB_V));
    const uint64_t dp_ = desc_kmajor_sw128(smem_addr(smem + OFFB_P));
    auto wait = [&](uint64_t* bb, int parity) {
      return __all_sync(0xffffffffu, mbar_wait_fast(bb, parity, abort_flag));
    };
    auto issue_s = [&](int sl) {  // S^T = K Q^T into [0,128)
      const uint64_t dq_k = desc_kmajor_sw128(smem_addr(smem + OFFB_SLOT + sl * TILE_BYTES));
      const uint32_t d = tmem;
#define KVS_ST(kk) umma_bf16_warp_at<kq_step(kk), kq_step(kk)>(d, dk_, dq_k, ID_T, kk > 0)
      KVS_ST(0); KVS_ST(1); KVS_ST(2); KVS_ST(3); KVS_ST(4); KVS_ST(5); KVS_ST(6); KVS_ST(7);
#undef KVS_ST
    };
    auto issue_dp = [&](int sl) {  // dP^T = V dO^T into [128,256)
      const uint64_t ddo_k = desc_kmajor_sw128(smem_addr(smem + OFFB_SLOT + sl * TILE_BYTES));
      const uint32_t d = tmem + 128;
#define KVS_DPT(kk) umma_bf16_warp_at<kq_step(kk), kq_step(kk)>(d, dv_, ddo_k, ID_T, kk > 0)
      KVS_DPT(0); KVS_DPT(1); KVS_DPT(2); KVS_DPT(3); KVS_DPT(4); KVS_DPT(5); KVS_DPT(6); KVS_DPT(7);
#undef KVS_DPT
    };
    bool ok = wait(&bar[D_KVFULL], 0);
    if (ok) ok = wait(&bar[D_FULL0 + slot_a(0)], 0);
    if (ok) {
      tc_fence_after();
      issue_s(slot_a(0));
      umma_commit_warp(&bar[D_SFULL]);
      ok = wait(&bar[D_FULL0 + slot_b(0)], 0);
    }
    if (ok) {
      tc_fence_after();
      issue_dp(slot_b(0));
      umma_commit_warp(&bar[D_DPFULL]);
    }
    for (int i = 0; ok && i < nsteps; ++i) {
      const bool more = i + 1 < nsteps;
      const int ph1 = ((i + 1) >> 1) & 1;
      if (more) {
        ok = wait(&bar[D_SREAD], i & 1);
        if (ok) ok = wait(&bar[D_FULL0 + slot_a(i + 1)], ph1);
        if (!ok) break;
        tc_fence_after();
        issue_s(slot_a(i + 1));
        umma_commit_warp(&bar[D_SFULL]);
      }
      ok = wait(&bar[D_PFULL], i & 1);
      if (!ok) break;
      tc_fence_after();
      {
        const uint64_t ddo_mn =
            desc_mnmajor_sw128(smem_addr(smem + OFFB_SLOT + slot_b(i) * TILE_BYTES), HALF_BYTES);
        const uint32_t d = tmem + 256;
        const uint32_t acc = i > 0;
#define KVS_DV(kk) umma_bf16_warp_at<kq_step(kk), mn_step(kk)>(d, dp_, ddo_mn, ID_MN, (kk > 0) || acc)
        KVS_DV(0); KVS_DV(1); KVS_DV(2); KVS_DV(3); KVS_DV(4); KVS_DV(5); KVS_DV(6); KVS_DV(7);
#undef KVS_DV
      }
      umma_commit_warp(&bar[D_EMPTY0 + slot_b(i)]);
      umma_commit_warp(&bar[D_PEMPTY]);
      ok = wait(&bar[D_DSFULL], i & 1);
      if (!ok) break;
      tc_fence_after();
      {
        const uint64_t dq_mn =
            desc_mnmajor_sw128(smem_addr(smem + OFFB_SLOT + slot_a(i) * TILE_BYTES), HALF_BYTES);
        const uint32_t d = tmem + 384, a = tmem + 128;
        const uint32_t acc = i > 0;
#define KVS_DK(kk) umma_bf16_tmem_a_warp_at<split_col(kk), mn_step(kk)>(d, a, dq_mn, ID_MN, (kk > 0) || acc)
        KVS_DK(0); KVS_DK(1); KVS_DK(2); KVS_DK(3); KVS_DK(4); KVS_DK(5); KVS_DK(6); KVS_DK(7);
#undef KVS_DK
      }
      umma_commit_warp(&bar[D_EMPTY0 + slot_a(i)]);
      if (more) {
        ok = wait(&bar[D_FULL0 + slot_b(i + 1)], ph1);
        if (!ok) break;
        tc_fence_after();
        issue_dp(slot_b(i + 1));
        umma_commit_warp(&bar[D_DPFULL]);
      }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicExch(p.error, 12);
    }
    umma_commit_warp(&bar[D_FINAL]);
    mbar_wait(&bar[D_FINAL], 0, nullptr);
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax: key row r, query columns [cb, cb+32)
    const int grp = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int s = k0 + r;
    const int cb = GCOLS * grp;
    const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
    const float sl2 = p.scale_log2;
    // this thread's 32 columns of P^T: half cb / 64 of the K-major tile, 16-byte chunks
    // (cb % 64) / 8 + c, XOR-swizzled by row
    uint8_t* prow = smem + OFFB_P + (cb >> 6) * HALF_BYTES + r * 128;
    const int c0 = (cb & 63) >> 3, sw = r & 7;
    // the query rows that see key s: [s, min(evicted_at[s], L)) for a real key, s itself for a
    // padded one, nothing past the stream
    int rlo = 0, rhi = 0;
    if (s < L) {
      rlo = s;
      rhi = min(p.e32[(int64_t)b * p.T_pad + s], L);
    } else if (s < p.T) {
      rlo = s;
      rhi = s + 1;
    }
    bool ok = true;
    for (int i = 0; i < nsteps; ++i) {
      const int t0 = (kt + i / G) * BM + cb;  // query row of this thread's first column
      ok = mbar_wait_fast(&bar[D_SFULL], i & 1, abort_flag);
      if (ok) ok = mbar_wait_fast(&bar[D_FULL0 + slot_b(i)], (i >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int lo = max(rlo - t0, 0), hi = min(rhi - t0, GCOLS);  // visible columns [lo, hi)
      // warp-uniform cases: every key of the warp sees all the columns (no masking), or none
      const bool full = __all_sync(0xffffffffu, lo == 0 && hi == GCOLS);
      const bool none = __all_sync(0xffffffffu, lo >= hi);
      const float* nl = reinterpret_cast<const float*>(smem + OFFB_LSE + (i & 1) * VEC_BYTES) + cb;
      const float* nd = reinterpret_cast<const float*>(smem + OFFB_D + (i & 1) * VEC_BYTES) + cb;
      // phase A: P = 2^(S * scale * log2 e - lse) over the visible columns
      float pf[GCOLS];
      if (!none) {
        uint32_t sv[32];
        tmem_ld32(tl + cb, sv);
        tmem_wait_ld();
        tc_fence_before();
        warp_arrive(&bar[D_SREAD]);  // S^T may be overwritten from here on
#pragma unroll
        for (int e = 0; e < GCOLS; e += 4) {
          const float4 n4 = *reinterpret_cast<const float4*>(nl + e);
          float x[4];
          ffma2v(x[0], x[1], __uint_as_float(sv[e]), __uint_as_float(sv[e + 1]), sl2, n4.x, n4.y);
          ffma2v(x[2], x[3], __uint_as_float(sv[e + 2]), __uint_as_float(sv[e + 3]), sl2, n4.z, n4.w);
#pragma unroll
          for (int u = 0; u < 4; ++u) pf[e + u] = ex2_approx(x[u]);
        }
        if (!full) {
#pragma unroll
          for (int col = 0; col < GCOLS; ++col) pf[col] = (col >= lo && col < hi) ? pf[col] : 0.f;
        }
      } else {
        warp_arrive(&bar[D_SREAD]);
#pragma unroll
        for (int e = 0; e < GCOLS; ++e) pf[e] = 0.f;
      }
      // P^T into shared memory once dV of the previous step has read it
      if (i > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait_fast(&bar[D_PEMPTY], (i - 1) & 1, abort_flag));
        if (!ok) break;
      }
#pragma unroll
      for (int c = 0; c < GCOLS / 8; ++c)
        *reinterpret_cast<uint4*>(prow + (((c0 + c) ^ sw) << 4)) =
            make_uint4(pack2(pf[8 * c], pf[8 * c + 1]), pack2(pf[8 * c + 2], pf[8 * c + 3]),
                       pack2(pf[8 * c + 4], pf[8 * c + 5]), pack2(pf[8 * c + 6], pf[8 * c + 7]));
      fence_proxy_async_smem();
      warp_arrive(&bar[D_PFULL]);
      // phase B: dS = P (dP - D)
      ok = __all_sync(0xffffffffu, mbar_wait_fast(&bar[D_DPFULL], i & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      uint32_t dk[GCOLS / 2];
      if (none) {
#pragma unroll
        for (int e = 0; e < GCOLS / 2; ++e) dk[e] = 0u;
      } else {
        uint32_t dp[32];
        tmem_ld32(tl + 128 + cb, dp);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < GCOLS; e += 4) {
          const float4 n4 = *reinterpret_cast<const float4*>(nd + e);
          float d[4];
          addmul2(d[0], d[1], __uint_as_float(dp[e]), __uint_as_float(dp[e + 1]), n4.x, n4.y, pf[e], pf[e + 1]);
          addmul2(d[2], d[3], __uint_as_float(dp[e + 2]), __uint_as_float(dp[e + 3]), n4.z, n4.w, pf[e + 2], pf[e + 3]);
          if (!full) {  // D past the stream is not defined: select, do not multiply
#pragma unroll
            for (int u = 0; u < 4; ++u) d[u] = (e + u >= lo && e + u < hi) ? d[u] : 0.f;
          }
          dk[e >> 1] = pack2(d[0], d[1]);
          dk[(e >> 1) + 1] = pack2(d[2], d[3]);
        }
      }
      tmem_st16(tl + 128 + cb, dk);
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(&bar[D_DSFULL]);
    }
    if (ok) ok = mbar_wait(&bar[D_FINAL], 0, abort_flag);
    ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.error, 13);
    } else {
      tc_fence_after();
      const int64_t row = ((int64_t)b * p.T + s) * p.Hkv + hk;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {  // dV, then dK (times the softmax scale)
        __nv_bfloat16* dst = (which == 0 ? p.dv : p.dk) + row * HD + cb;
        const float mul = which == 0 ? 1.f : p.scale;
#pragma unroll 1
        for (int c = 0; c < GCOLS / 32; ++c) {
          uint32_t o[32];
          __syncwarp();
          tmem_ld32(tl + 256 + 128 * which + cb + 32 * c, o);
          tmem_wait_ld();
          if (s >= p.T) continue;  // rows past the stream: loaded by the whole warp, not stored
          uint4* d4o = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            d4o[q4] = make_uint4(pack2(__uint_as_float(o[8 * q4]) * mul, __uint_as_float(o[8 * q4 + 1]) * mul),
                                 pack2(__uint_as_float(o[8 * q4 + 2]) * mul, __uint_as_float(o[8 * q4 + 3]) * mul),
                                 pack2(__uint_as_float(o[8 * q4 + 4]) * mul, __uint_as_float(o[8 * q4 + 5]) * mul),
                                 pack2(__uint_as_float(o[8 * q4 + 6]) * mul, __uint_as_float(o[8 * q4 + 7]) * mul));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Base address of the dynamic shared memory of a kernel without static shared memory (the
// dK/dV kernel's layout has no padding for alignment and needs it 1024-aligned)
__global__ void replay_smem_base_kernel(uint32_t* out) {
  extern __shared__ __align__(1024) uint8_t smem_bwd[];
  if (threadIdx.x == 0) *out = smem_addr(smem_bwd);
}

// smem of the dQ kernel
constexpr int OFFQ_Q = 0, OFFQ_DO = TILE_BYTES;
constexpr int OFFQ_SLOT = 2 * TILE_BYTES;            // 4 slots: K and V tiles of the loop
constexpr int OFFQ_E = OFFQ_SLOT + 4 * TILE_BYTES;   // 4 slots of 128 int32, loaded with K
constexpr int OFFQ_LIST = OFFQ_E + 4 * E_BYTES;
constexpr int OFFQ_BAR = OFFQ_LIST + MAX_KT * 2;
// Q_SREAD: every softmax warp has S of the step in registers (S may be overwritten);
// Q_AFULL: the softmax warps have copied Q and dO into TMEM (the A operands of S and dP)
enum { Q_QFULL = 0, Q_FULL0, Q_EMPTY0 = Q_FULL0 + 4, Q_SFULL = Q_EMPTY0 + 4, Q_DPFULL, Q_SREAD, Q_DSFULL, Q_AFULL,
       Q_FINAL, NBARQ };
constexpr int OFFQ_MISC = OFFQ_BAR + NBARQ * 8;
constexpr int SMEMQ_BYTES = OFFQ_MISC + 64 + 33 * 4;
static_assert(SMEMQ_BYTES <= 232448, "dQ kernel shared memory");

__global__ void __launch_bounds__(NTB, 1)
replay_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                 const BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_bwd[];
  uint8_t* smem = smem_bwd;
  if (smem_addr(smem) & 1023) {  // never expected (the host checked); no work, no TMEM
    if (threadIdx.x == 0) atomicExch(p.error, 25);
    return;
  }
  uint16_t* list = reinterpret_cast<uint16_t*>(smem + OFFQ_LIST);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFFQ_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFFQ_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFFQ_MISC + 4);
  int* s_n = reinterpret_cast<int*>(smem + OFFQ_MISC + 8);
  int* s_scan = reinterpret_cast<int*>(smem + OFFQ_MISC + 64);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // CTA order: query tiles descending slowest (a late tile has the most key tiles, so the
  // longest CTAs start first), then (stream, KV head), then the heads of a group (which read
  // the same K/V tiles)
  const int G = p.Hq / p.Hkv;
  const int nbh = p.B * p.Hkv;
  const int g = (int)(blockIdx.x % G);
  const int rest = (int)(blockIdx.x / G);
  const int qt = p.n_qt - 1 - rest / nbh;
  const int bhk = rest % nbh;
  const int b = bhk / p.Hkv, hk = bhk % p.Hkv;
  const int h = hk * G + g;
  const int t0 = qt * BM, t1 = t0 + BM - 1;
  const int L = p.lengths[b];

  if (tid == 0) {
    for (int i = 0; i < NBARQ; ++i) mbar_init(&bar[i], 1);
    mbar_init(&bar[Q_SREAD], 4 * NGRP);
    mbar_init(&bar[Q_DSFULL], 4 * NGRP);
    mbar_init(&bar[Q_AFULL], 4 * NGRP);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // active key tiles (the forward's list)
  {
    const int real_last = min(t1, L - 1);
    int carry = 0;
    for (int base = 0; base <= qt; base += NTB) {
      const int j = base + tid;
      int flag = 0;
      if (j <= qt) {
        const int emin = p.tile_min[b * p.n_kt + j], emax = p.tile_max[b * p.n_kt + j];
        const bool active = (j == qt) || (j * BN <= real_last && emax > t0);
        const bool masked = (j == qt) || (emin <= t1) || (t1 >= L);
        flag = (active ? 1 : 0) | (masked ? 2 : 0);
      }
      int tot = 0;
      const int pre = block_exclusive_scan(flag & 1, s_scan, &tot);
      if (flag & 1) list[carry + pre] = (uint16_t)(j | ((flag & 2) ? 0x8000 : 0));
      carry += tot;
      __syncthreads();
    }
    if (tid == 0) *s_n = carry;
  }
  __syncthreads();
  tc_fence_after();
  const int n = *s_n;
  const uint32_t tmem = *tmem_slot;
  // TMEM: S [0,128), dP [128,256) (dS bf16 of group g over [128+32g, +16) once dP is read),
  // dQ [256,384), Q [384,448) and dO [448,512) as bf16 A operands.  Q and dO are the same for
  // every step, so S = Q K^T and dP = dO V^T read only K and V from shared memory.

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- Q, dO; the K tiles (+ evicted_at)
      mbar_arrive_expect_tx(&bar[Q_QFULL], 2 * TILE_BYTES);
      tma_load_3d(smem + OFFQ_Q, &tm_q, 0, h, b * p.T + t0, &bar[Q_QFULL]);
      tma_load_3d(smem + OFFQ_Q + HALF_BYTES, &tm_q, 64, h, b * p.T + t0, &bar[Q_QFULL]);
      tma_load_3d(smem + OFFQ_DO, &tm_do, 0, h, b * p.T + t0, &bar[Q_QFULL]);
      tma_load_3d(smem + OFFQ_DO + HALF_BYTES, &tm_do, 64, h, b * p.T + t0, &bar[Q_QFULL]);
      for (int k = 0; k < n; ++k) {
        const int sl = slot_a(k);
        if (k >= 2 && !mbar_wait(&bar[Q_EMPTY0 + sl], ((k >> 1) - 1) & 1, abort_flag)) {
          *abort_flag = 1;
          atomicExch(p.error, 21);
          break;
        }
        const int j = list[k] & 0x7fff;
        uint64_t* fb = &bar[Q_FULL0 + sl];
        mbar_arrive_expect_tx(fb, TILE_BYTES + E_BYTES);
        uint8_t* ks = smem + OFFQ_SLOT + sl * TILE_BYTES;
        tma_load_3d(ks, &tm_k, 0, hk, b * p.T + j * BN, fb);
        tma_load_3d(ks + HALF_BYTES, &tm_k, 64, hk, b * p.T + j * BN, fb);
        bulk_load(smem + OFFQ_E + (k & 3) * E_BYTES, p.e32 + (int64_t)b * p.T_pad + j * BN, E_BYTES, fb);
        if (k + 2 < n) {
          const int j2 = list[k + 2] & 0x7fff;
          tma_prefetch_3d(&tm_k, 0, hk, b * p.T + j2 * BN);
          tma_prefetch_3d(&tm_k, 64, hk, b * p.T + j2 * BN);
        }
      }
    } else if (lane == 1) {
      // ---------------------------------------------------------- the V tiles
      for (int k = 0; k < n; ++k) {
        const int sl = slot_b(k);
        if (k >= 2 && !mbar_wait(&bar[Q_EMPTY0 + sl], ((k >> 1) - 1) & 1, abort_flag)) {
          *abort_flag = 1;
          atomicExch(p.error, 24);
          break;
        }
        const int j = list[k] & 0x7fff;
        uint64_t* fb = &bar[Q_FULL0 + sl];
        mbar_arrive_expect_tx(fb, TILE_BYTES);
        uint8_t* vs = smem + OFFQ_SLOT + sl * TILE_BYTES;
        tma_load_3d(vs, &tm_v, 0, hk, b * p.T + j * BN, fb);
        tma_load_3d(vs + HALF_BYTES, &tm_v, 64, hk, b * p.T + j * BN, fb);
        if (k + 2 < n) {
          const int j2 = list[k + 2] & 0x7fff;
          tma_prefetch_3d(&tm_v, 0, hk, b * p.T + j2 * BN);
          tma_prefetch_3d(&tm_v, 64, hk, b * p.T + j2 * BN);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- UMMA issuer (whole warp)
    // per step k: S(k+1) once S(k) is read; dQ += dS(k) K(k); dP(k+1).  K(k) is released by
    // dQ(k), V(k) by dP(k): K(k+2) takes V(k)'s slot and V(k+2) K(k)'s.
    constexpr uint32_t ID_K = idesc_bf16(128, 128, 0);   // S, dP: A from TMEM, B K-major
    constexpr uint32_t ID_MN = idesc_bf16(128, 128, 1);  // dQ: B (K) MN-major
    auto wait = [&](uint64_t* bb, int parity) {
      return __all_sync(0xffffffffu, mbar_wait_fast(bb, parity, abort_flag));
    };
    auto issue_s = [&](int sl) {  // S = Q K^T into [0,128), Q from TMEM [384,448)
      const uint64_t dk_k = desc_kmajor_sw128(smem_addr(smem + OFFQ_SLOT + sl * TILE_BYTES));
      const uint32_t d = tmem, a = tmem + 384;
#define KVS_S(kk) umma_bf16_tmem_a_warp_at<kk * 8, kq_step(kk)>(d, a, dk_k, ID_K, kk > 0)
      KVS_S(0); KVS_S(1); KVS_S(2); KVS_S(3); KVS_S(4); KVS_S(5); KVS_S(6); KVS_S(7);
#undef KVS_S
    };
    auto issue_dp = [&](int sl) {  // dP = dO V^T into [128,256), dO from TMEM [448,512)
      const uint64_t dv_k = desc_kmajor_sw128(smem_addr(smem + OFFQ_SLOT + sl * TILE_BYTES));
      const uint32_t d = tmem + 128, a = tmem + 448;
#define KVS_DP(kk) umma_bf16_tmem_a_warp_at<kk * 8, kq_step(kk)>(d, a, dv_k, ID_K, kk > 0)
      KVS_DP(0); KVS_DP(1); KVS_DP(2); KVS_DP(3); KVS_DP(4); KVS_DP(5); KVS_DP(6); KVS_DP(7);
#undef KVS_DP
    };
    bool ok = wait(&bar[Q_AFULL], 0);
    if (ok) ok = wait(&bar[Q_FULL0 + slot_a(0)], 0);
    if (ok) {
      tc_fence_after();
      issue_s(slot_a(0));
      umma_commit_warp(&bar[Q_SFULL]);
      ok = wait(&bar[Q_FULL0 + slot_b(0)], 0);
    }
    if (ok) {
      tc_fence_after();
      issue_dp(slot_b(0));
      umma_commit_warp(&bar[Q_EMPTY0 + slot_b(0)]);
      umma_commit_warp(&bar[Q_DPFULL]);
    }
    for (int k = 0; ok && k < n; ++k) {
      const bool more = k + 1 < n;
      const int ph1 = ((k + 1) >> 1) & 1;
      if (more) {
        ok = wait(&bar[Q_SREAD], k & 1);
        if (ok) ok = wait(&bar[Q_FULL0 + slot_a(k + 1)], ph1);
        if (!ok) break;
        tc_fence_after();
        issue_s(slot_a(k + 1));
        umma_commit_warp(&bar[Q_SFULL]);
      }
      ok = wait(&bar[Q_DSFULL], k & 1);
      if (!ok) break;
      tc_fence_after();
      {
        const uint64_t dk_mn =
            desc_mnmajor_sw128(smem_addr(smem + OFFQ_SLOT + slot_a(k) * TILE_BYTES), HALF_BYTES);
        const uint32_t d = tmem + 256, a = tmem + 128;
        const uint32_t acc = k > 0;
#define KVS_DQ(kk) umma_bf16_tmem_a_warp_at<split_col(kk), mn_step(kk)>(d, a, dk_mn, ID_MN, (kk > 0) || acc)
        KVS_DQ(0); KVS_DQ(1); KVS_DQ(2); KVS_DQ(3); KVS_DQ(4); KVS_DQ(5); KVS_DQ(6); KVS_DQ(7);
#undef KVS_DQ
      }
      umma_commit_warp(&bar[Q_EMPTY0 + slot_a(k)]);
      if (more) {
        ok = wait(&bar[Q_FULL0 + slot_b(k + 1)], ph1);
        if (!ok) break;
        tc_fence_after();
        issue_dp(slot_b(k + 1));
        umma_commit_warp(&bar[Q_EMPTY0 + slot_b(k + 1)]);
        umma_commit_warp(&bar[Q_DPFULL]);
      }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicExch(p.error, 22);
    }
    umma_commit_warp(&bar[Q_FINAL]);
    mbar_wait(&bar[Q_FINAL], 0, nullptr);
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax: query row r, key columns [cb, cb+32)
    const int grp = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int t = t0 + r;
    const int cb = GCOLS * grp;
    const bool real = t < L;
    const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
    const float sl2 = p.scale_log2;
    const int64_t vrow = ((int64_t)b * p.Hq + h) * p.T_pad + t;
    const float nlse = t < p.T ? p.nlse[vrow] : 0.f;
    const float nd = t < p.T ? p.nd[vrow] : 0.f;
    // Q and dO of row r into TMEM: dims [32 grp, +32) of each, 16-byte chunks of the 128-byte
    // swizzled row, as 16 columns of bf16 pairs at 384 + 16 grp and 448 + 16 grp
    bool ok = __all_sync(0xffffffffu, mbar_wait(&bar[Q_QFULL], 0, abort_flag));
    if (ok) {
      const int c0 = (grp & 1) * 4, sw = r & 7;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint8_t* row = smem + (which ? OFFQ_DO : OFFQ_Q) + (grp >> 1) * HALF_BYTES + r * 128;
        uint32_t w[16];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 x = *reinterpret_cast<const uint4*>(row + (((c0 + c) ^ sw) << 4));
          w[4 * c] = x.x;
          w[4 * c + 1] = x.y;
          w[4 * c + 2] = x.z;
          w[4 * c + 3] = x.w;
        }
        tmem_st16(tl + 384 + 64 * which + 16 * grp, w);
      }
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(&bar[Q_AFULL]);
    }
    for (int k = 0; ok && k < n; ++k) {
      const int j = list[k] & 0x7fff;
      const bool masked = (list[k] >> 15) & 1;
      ok = mbar_wait_fast(&bar[Q_SFULL], k & 1, abort_flag);
      if (ok) ok = mbar_wait_fast(&bar[Q_FULL0 + slot_a(k)], (k >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // phase A: P over the visible keys; S may be overwritten as soon as it is in registers
      float pf[GCOLS];
      {
        uint32_t sv[32];
        tmem_ld32(tl + cb, sv);
        tmem_wait_ld();
        tc_fence_before();
        warp_arrive(&bar[Q_SREAD]);
#pragma unroll
        for (int e = 0; e < GCOLS; e += 2) {
          float x0, x1;
          ffma2(x0, x1, __uint_as_float(sv[e]), __uint_as_float(sv[e + 1]), sl2, nlse);
          pf[e] = ex2_approx(x0);
          pf[e + 1] = ex2_approx(x1);
        }
      }
      // visibility bits of this thread's 32 keys (all set for an unmasked tile)
      uint32_t bits = 0xffffffffu;
      if (masked) {
        const int lim = t - j * BN;
        const int4* E4 = reinterpret_cast<const int4*>(smem + OFFQ_E + (k & 3) * E_BYTES) + cb / 4;
        uint32_t bw = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int4 e = E4[q];
          const int ev[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = cb + 4 * q + u;
            const bool vis = (i <= lim) && (real ? (t < ev[u]) : (i >= lim));
            bw |= (vis ? 1u : 0u) << (4 * q + u);
          }
        }
        bits = (t < p.T) ? bw : 0u;
#pragma unroll
        for (int e = 0; e < GCOLS; ++e) pf[e] = ((bits >> e) & 1) ? pf[e] : 0.f;
      }
      // phase B: dS = P (dP - D)
      ok = __all_sync(0xffffffffu, mbar_wait_fast(&bar[Q_DPFULL], k & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      uint32_t dk[GCOLS / 2];
      {
        uint32_t dp[32];
        tmem_ld32(tl + 128 + cb, dp);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < GCOLS; e += 2) {
          float d0, d1;
          addmul2(d0, d1, __uint_as_float(dp[e]), __uint_as_float(dp[e + 1]), nd, nd, pf[e], pf[e + 1]);
          if (masked) {
            d0 = ((bits >> e) & 1) ? d0 : 0.f;
            d1 = ((bits >> (e + 1)) & 1) ? d1 : 0.f;
          }
          dk[e >> 1] = pack2(d0, d1);
        }
      }
      tmem_st16(tl + 128 + cb, dk);
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(&bar[Q_DSFULL]);
    }
    if (ok) ok = mbar_wait(&bar[Q_FINAL], 0, abort_flag);
    ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.error, 23);
    } else {
      tc_fence_after();
      __nv_bfloat16* dst = p.dq + (((int64_t)b * p.T + t) * p.Hq + h) * HD + cb;
      const float mul = p.scale;
#pragma unroll 1
      for (int c = 0; c < GCOLS / 32; ++c) {
        uint32_t o[32];
        __syncwarp();
        tmem_ld32(tl + 256 + cb + 32 * c, o);
        tmem_wait_ld();
        if (t >= p.T) continue;  // rows past the stream: loaded by the whole warp, not stored
        uint4* d4o = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          d4o[q4] = make_uint4(pack2(__uint_as_float(o[8 * q4]) * mul, __uint_as_float(o[8 * q4 + 1]) * mul),
                               pack2(__uint_as_float(o[8 * q4 + 2]) * mul, __uint_as_float(o[8 * q4 + 3]) * mul),
                               pack2(__uint_as_float(o[8 * q4 + 4]) * mul, __uint_as_float(o[8 * q4 + 5]) * mul),
                               pack2(__uint_as_float(o[8 * q4 + 6]) * mul, __uint_as_float(o[8 * q4 + 7]) * mul));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// per-(stream, key tile) min / max of evicted_at and the padded int32 copy
__global__ void replay_prepass_kernel(const int64_t* __restrict__ ev, int T, int T_pad, int n_kt,
                                      int32_t* __restrict__ e32, int32_t* __restrict__ tmin, int32_t* __restrict__ tmax) {
  const int b = blockIdx.y, j = blockIdx.x;  // one CTA of 128 threads per key tile
  const int s = j * BN + threadIdx.x;
  int32_t e = 0;
  int32_t lo = INT32_MAX, hi = INT32_MIN;
  if (s < T) {
    const int64_t x = ev[(int64_t)b * T + s];
    e = x > INT32_MAX ? INT32_MAX : (int32_t)x;
    lo = hi = e;
  }
  if (s < T_pad) e32[(int64_t)b * T_pad + s] = e;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  __shared__ int32_t slo[4], shi[4];
  if ((threadIdx.x & 31) == 0) {
    slo[threadIdx.x >> 5] = lo;
    shi[threadIdx.x >> 5] = hi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    tmin[b * n_kt + j] = min(min(slo[0], slo[1]), min(slo[2], slo[3]));
    tmax[b * n_kt + j] = max(max(shi[0], shi[1]), max(shi[2], shi[3]));
  }
}

// ------------------------------------------------------------------ UMMA self-test
// C[128][128] (f32) = A[128][128] (bf16, row-major = K-major) x B, with B given as
// Bt[128 n][128 k] (K-major, b_mn = 0) or B[128 k][128 n] (MN-major, b_mn = 1).
__global__ void __launch_bounds__(128, 1)
umma_selftest_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, int mode,
                     const uint32_t* __restrict__ a_raw, float* __restrict__ c, int32_t* __restrict__ error) {
  // mode bit 0: B is MN-major; bit 1: A is staged in TMEM (row = lane, bf16 pairs per column)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* As = smem;
  uint8_t* Bs = smem + TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * TILE_BYTES);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 2 * TILE_BYTES + 64);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b_mn = mode & 1, a_tmem = (mode >> 1) & 1;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  if (a_tmem) {
    // row r of A -> TMEM lane r, columns 128..191 (64 columns of bf16 pairs)
    const int r = warp * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16) + 128;
    for (int cc = 0; cc < 2; ++cc) {
      uint32_t v[32];
      for (int i = 0; i < 32; ++i) v[i] = a_raw[r * 64 + cc * 32 + i];
      tmem_st32(lane_base + cc * 32, v);
    }
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  bool ok = true;
  if (threadIdx.x == 0) {
    tc_fence_after();
    mbar_arrive_expect_tx(&bars[0], 2 * TILE_BYTES);
    tma_load_3d(As, &tm_a, 0, 0, 0, &bars[0]);
    tma_load_3d(As + HALF_BYTES, &tm_a, 64, 0, 0, &bars[0]);
    tma_load_3d(Bs, &tm_b, 0, 0, 0, &bars[0]);
    tma_load_3d(Bs + HALF_BYTES, &tm_b, 64, 0, 0, &bars[0]);
    ok = mbar_wait(&bars[0], 0, nullptr);
    if (ok) {
      tc_fence_after();
      const uint32_t a0 = smem_addr(As), b0 = smem_addr(Bs);
      const uint32_t id = idesc_bf16(128, 128, b_mn);
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
        const uint64_t bd = b_mn ? desc_mnmajor_sw128(b0 + kk * 2048, HALF_BYTES) : desc_kmajor_sw128(b0 + off);
        if (a_tmem)
          umma_bf16_tmem_a(tmem, tmem + 128 + kk * 8, bd, id, kk > 0);
        else
          umma_bf16(tmem, desc_kmajor_sw128(a0 + off), bd, id, kk > 0);
      }
      umma_commit(&bars[1]);
    } else {
      atomicExch(error, 1);
    }
  }
  __syncthreads();
  if (mbar_wait(&bars[1], 0, nullptr)) {
    tc_fence_after();
    const int r = warp * 32 + lane;
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + cc * 32, v);
      tmem_wait_ld();
      for (int i = 0; i < 32; ++i) c[r * 128 + cc * 32 + i] = __uint_as_float(v[i]);
    }
  } else if (threadIdx.x == 0) {
    atomicExch(error, 2);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ------------------------------------------------------------------ host helpers
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D bf16 map over rows of `inner` elements: dims {inner, mid, outer}, box {64, 1, rows},
// 128-byte swizzle
bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t mid, uint64_t outer, uint32_t rows = 128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {inner, mid, outer};
  const cuuint64_t strides[2] = {inner * 2, inner * mid * 2};
  const cuuint32_t box[3] = {64, 1, rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

std::mutex g_attr_mu;
bool g_attr_done[64][2] = {};

bool set_smem_attr(const void* fn, int which, int bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_attr_mu);
  if (dev < 64 && !g_attr_done[dev][which]) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
    g_attr_done[dev][which] = true;
  }
  return true;
}

// The head-pair kernel redistributes registers between its warpgroups with setmaxnreg;
// that is only sound when the block is launched with at least the budget the split adds
// up to, so the launch register count is checked once per device before its first use.
template <bool PAGED>
bool pair_kernel_ready() {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static int state[64] = {};  // 0 unknown, 1 ready, 2 unusable
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 64) return false;
  if (state[dev] == 0) {
    cudaFuncAttributes fa;
    bool ok = cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(pair_attn_kernel<PAGED>)) == cudaSuccess &&
              fa.numRegs * NT2 >= REGS_CTRL * 128 + REGS_SOFT * 256 &&
              cudaFuncSetAttribute(reinterpret_cast<const void*>(pair_attn_kernel<PAGED>),
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES) == cudaSuccess;
    if (!ok) (void)cudaGetLastError();  // leave no error behind for the next launch check
    state[dev] = ok ? 1 : 2;
  }
  return state[dev] == 1;
}

struct ReplayScratch {
  int32_t* e32;
  int32_t* tmin;
  int32_t* tmax;
  int32_t* error;
};

size_t replay_scratch_layout(int B, int T, void* base, ReplayScratch* s) {
  const int T_pad = (T + BN - 1) / BN * BN;
  const int n_kt = T_pad / BN;
  size_t off = 0;
  const size_t o_e = off; off = align_up(off + (size_t)B * T_pad * 4, 256);
  const size_t o_lo = off; off = align_up(off + (size_t)B * n_kt * 4, 256);
  const size_t o_hi = off; off = align_up(off + (size_t)B * n_kt * 4, 256);
  const size_t o_err = off; off = align_up(off + 4, 256);
  if (s) {
    uint8_t* p = static_cast<uint8_t*>(base);
    s->e32 = reinterpret_cast<int32_t*>(p + o_e);
    s->tmin = reinterpret_cast<int32_t*>(p + o_lo);
    s->tmax = reinterpret_cast<int32_t*>(p + o_hi);
    s->error = reinterpret_cast<int32_t*>(p + o_err);
  }
  return off;
}

}  // namespace

size_t kvs_replay_tc_scratch(int B, int T) { return replay_scratch_layout(B, T, nullptr, nullptr); }

bool kvs_replay_tc_supported(const kvs_replay_args* a) {
  return a->dtype == KVS_BF16 && a->head_dim == HD && (a->n_heads % a->n_kv_heads) == 0 &&
         (a->seq_len + BN - 1) / BN <= MAX_KT && (reinterpret_cast<uintptr_t>(a->out) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a->q) & 15) == 0 && (reinterpret_cast<uintptr_t>(a->k) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a->v) & 15) == 0 && encode_fn() != nullptr;
}

int kvs_replay_tc_launch(const kvs_replay_args* a, cudaStream_t st) {
  ReplayScratch s;
  const size_t need = replay_scratch_layout(a->batch, a->seq_len, a->scratch, &s);
  if (!a->scratch || a->scratch_bytes < need) return KVS_E_SCRATCH;
  const int T = a->seq_len, B = a->batch;
  const int T_pad = (T + BN - 1) / BN * BN, n_kt = T_pad / BN;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, a->q, HD, a->n_heads, (uint64_t)B * T) || !make_map(&mk, a->k, HD, a->n_kv_heads, (uint64_t)B * T) ||
      !make_map(&mv, a->v, HD, a->n_kv_heads, (uint64_t)B * T))
    return KVS_E_UNSUPPORTED;
  if (!set_smem_attr(reinterpret_cast<const void*>(replay_tc_kernel), 0, SMEM_BYTES)) return KVS_E_LAUNCH;
  if (cudaMemsetAsync(s.error, 0, 4, st) != cudaSuccess) return KVS_E_LAUNCH;
  replay_prepass_kernel<<<dim3(n_kt, B), BN, 0, st>>>(a->evicted_at, T, T_pad, n_kt, s.e32, s.tmin, s.tmax);
  int rc = launch_rc();
  if (rc) return rc;
  ReplayParams p;
  p.e32 = s.e32;
  p.tile_min = s.tmin;
  p.tile_max = s.tmax;
  p.lengths = a->lengths;
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.lse = a->row_lse;
  p.error = s.error;
  p.B = B;
  p.T = T;
  p.T_pad = T_pad;
  p.Hq = a->n_heads;
  p.Hkv = a->n_kv_heads;
  p.n_qt = n_kt;
  p.n_kt = n_kt;
  p.scale_log2 = (float)(a->scale * 1.4426950408889634);
  const int G = a->n_heads / a->n_kv_heads;
  if (G % 2 == 0 && !(a->flags & 2) && pair_kernel_ready<false>()) {
    const int64_t grid = (int64_t)B * a->n_heads / 2 * n_kt;
    pair_attn_kernel<false><<<(unsigned)grid, NT2, SMEM2_BYTES, st>>>(mq, mk, mv, p, PagedParams{});
  } else {
    const int64_t grid = (int64_t)B * a->n_heads * n_kt;
    replay_tc_kernel<<<(unsigned)grid, NT, SMEM_BYTES, st>>>(mq, mk, mv, p);
  }
  return launch_rc();
}


size_t kvs_replay_tc_backward_scratch(int B, int T, int Hq) {
  const int T_pad = (T + BN - 1) / BN * BN;
  return replay_scratch_layout(B, T, nullptr, nullptr) + 2 * align_up((size_t)B * Hq * T_pad * 4, 256);
}

namespace {
// Once per device: kernel attributes, a check that the dynamic shared base is 1024-aligned
// (the backward layouts rely on it) and that one CTA of each kernel fits on an SM.
// 1 ready, 0 not available (the exact kernels run), < 0 a CUDA error.
int bwd_device_ready(cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KVS_E_LAUNCH;
  static std::mutex mu;
  static int state[64] = {};  // 0 unknown, 1 ready, 2 unsupported
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 64) return 0;
  if (state[dev] == 0) {
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(replay_dkdv_kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEMB_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(reinterpret_cast<const void*>(replay_dq_kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEMQ_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(reinterpret_cast<const void*>(replay_smem_base_kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEMB_BYTES) != cudaSuccess)
      return KVS_E_LAUNCH;
    int nb_dkdv = 0, nb_dq = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb_dkdv, replay_dkdv_kernel, NTB, SMEMB_BYTES) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb_dq, replay_dq_kernel, NTB, SMEMQ_BYTES) != cudaSuccess)
      return KVS_E_LAUNCH;
    uint32_t* d_base = nullptr;
    uint32_t h_base = 1;
    if (cudaMalloc(&d_base, 4) != cudaSuccess) return KVS_E_LAUNCH;
    replay_smem_base_kernel<<<1, 32, SMEMB_BYTES, st>>>(d_base);
    const bool got = cudaGetLastError() == cudaSuccess &&
                     cudaMemcpyAsync(&h_base, d_base, 4, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
                     cudaStreamSynchronize(st) == cudaSuccess;
    cudaFree(d_base);
    if (!got) return KVS_E_LAUNCH;
    state[dev] = ((h_base & 1023) == 0 && nb_dkdv >= 1 && nb_dq >= 1) ? 1 : 2;
  }
  return state[dev] == 1 ? 1 : 0;
}

bool bwd_args_covered(const kvs_replay_args* a, const void* dout, const void* dq, const void* dk, const void* dv) {
  auto al = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  return a->row_lse != nullptr && kvs_replay_tc_supported(a) && al(a->row_lse) && al(a->scratch) && al(dout) &&
         al(dq) && al(dk) && al(dv);
}
}  // namespace

// 1 when kvs_replay_attention_backward would run the tensor-core kernels for these arguments
// (the gradient pointers are not known here and assumed 16-byte aligned), 0 for the exact ones.
int kvs_replay_tc_backward_path(const kvs_replay_args* a, cudaStream_t st) {
  if (!bwd_args_covered(a, a->q, a->q, a->k, a->v)) return 0;
  const int ready = bwd_device_ready(st);
  return ready;
}

// Tensor-core backward (bf16, head_dim 128, the forward's row_lse given).  Returns
// KVS_E_UNSUPPORTED when the shape, alignment or device is not covered (the caller then runs
// the exact kernels).
int kvs_replay_tc_backward(const kvs_replay_args* a, const void* dout, void* dq, void* dk, void* dv,
                           cudaStream_t st) {
  if (!bwd_args_covered(a, dout, dq, dk, dv)) return KVS_E_UNSUPPORTED;
  const int T = a->seq_len, B = a->batch;
  if (!a->scratch || a->scratch_bytes < kvs_replay_tc_backward_scratch(B, T, a->n_heads)) return KVS_E_SCRATCH;
  ReplayScratch s;
  const size_t off = replay_scratch_layout(B, T, a->scratch, &s);
  const int T_pad = (T + BN - 1) / BN * BN, n_kt = T_pad / BN;
  float* nlse = reinterpret_cast<float*>(static_cast<uint8_t*>(a->scratch) + off);
  float* nd = reinterpret_cast<float*>(static_cast<uint8_t*>(a->scratch) + off +
                                       align_up((size_t)B * a->n_heads * T_pad * 4, 256));
  CUtensorMap mq, mk, mv, mdo;
  if (!make_map(&mq, a->q, HD, a->n_heads, (uint64_t)B * T) || !make_map(&mk, a->k, HD, a->n_kv_heads, (uint64_t)B * T) ||
      !make_map(&mv, a->v, HD, a->n_kv_heads, (uint64_t)B * T) || !make_map(&mdo, dout, HD, a->n_heads, (uint64_t)B * T))
    return KVS_E_UNSUPPORTED;
  const int ready = bwd_device_ready(st);
  if (ready < 0) return ready;
  if (ready == 0) return KVS_E_UNSUPPORTED;
  if (cudaMemsetAsync(s.error, 0, 4, st) != cudaSuccess) return KVS_E_LAUNCH;
  replay_prepass_kernel<<<dim3(n_kt, B), BN, 0, st>>>(a->evicted_at, T, T_pad, n_kt, s.e32, s.tmin, s.tmax);
  int rc = launch_rc();
  if (rc) return rc;
  const int64_t rowdot_warps = (int64_t)B * a->n_heads * ((T + ROWDOT_PER_WARP - 1) / ROWDOT_PER_WARP);
  replay_rowdot_kernel<<<(unsigned)((rowdot_warps + 7) / 8), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(dout),
                                                                    static_cast<const __nv_bfloat16*>(a->out),
                                                                    a->row_lse, nlse, nd, B, T, T_pad, a->n_heads);
  if ((rc = launch_rc())) return rc;
  BwdParams p;
  p.e32 = s.e32;
  p.tile_min = s.tmin;
  p.tile_max = s.tmax;
  p.lengths = a->lengths;
  p.nlse = nlse;
  p.nd = nd;
  p.dq = static_cast<__nv_bfloat16*>(dq);
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.error = s.error;
  p.B = B;
  p.T = T;
  p.T_pad = T_pad;
  p.Hq = a->n_heads;
  p.Hkv = a->n_kv_heads;
  p.n_qt = n_kt;
  p.n_kt = n_kt;
  p.scale = (float)a->scale;
  p.scale_log2 = (float)(a->scale * 1.4426950408889634);
  replay_dkdv_kernel<<<(unsigned)((int64_t)B * a->n_kv_heads * n_kt), NTB, SMEMB_BYTES, st>>>(mq, mk, mv, mdo, p);
  if ((rc = launch_rc())) return rc;
  replay_dq_kernel<<<(unsigned)((int64_t)B * a->n_heads * n_kt), NTB, SMEMQ_BYTES, st>>>(mq, mk, mv, mdo, p);
  return launch_rc();
}

// ------------------------------------------------------------------ paged prefill (host)
namespace {
// cu_qt[i] = number of 128-query tiles of sequences 0..i-1 (one CTA)
__global__ void prefill_tiles_kernel(const int32_t* __restrict__ cu_tokens, int num_seqs, int32_t* __restrict__ cu_qt) {
  __shared__ int scan[33];
  int carry = 0;
  for (int base = 0; base < num_seqs; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int tiles = i < num_seqs ? (cu_tokens[i + 1] - cu_tokens[i] + BM - 1) / BM : 0;
    int tot = 0;
    const int pre = block_exclusive_scan(tiles, scan, &tot);
    if (i < num_seqs) cu_qt[i] = carry + pre;
    carry += tot;
  }
  if (threadIdx.x == 0) cu_qt[num_seqs] = carry;
}
}  // namespace

size_t kvs_prefill_tc_scratch(int num_seqs) { return align_up((size_t)(num_seqs + 1) * 4, 256); }

// bf16, D 128, 16-token blocks, an even GQA group (sequences longer than MAX_KT * 128 entries
// are reported through the status words)
bool kvs_prefill_tc_capable(const kvs_cache* c, int n_heads) {
  return c->dtype == KVS_BF16 && c->head_dim == HD && c->block_size == 16 && n_heads % c->n_kv_heads == 0 &&
         (n_heads / c->n_kv_heads) % 2 == 0 && (int64_t)c->num_blocks * c->block_size < INT32_MAX &&
         encode_fn() != nullptr;
}

// Attention of the new tokens of a chunked batch (q already rotated, in `qo`; their k/v already
// appended) over the paged pool, written back into `qo`.  `scratch` holds cu_qt.
int kvs_prefill_tc_launch(const kvs_cache* c, const kvs_batch* b, int layer, void* qo, int n_heads, double scale,
                          void* scratch, cudaStream_t st) {
  if (!pair_kernel_ready<true>()) return KVS_E_UNSUPPORTED;
  int32_t* cu_qt = static_cast<int32_t*>(scratch);
  prefill_tiles_kernel<<<1, 1024, 0, st>>>(b->cu_tokens, b->num_seqs, cu_qt);
  int rc = launch_rc();
  if (rc) return rc;
  const uint64_t pool_rows = (uint64_t)c->num_blocks * c->block_size;
  const size_t layer_elems = (size_t)pool_rows * c->n_kv_heads * c->head_dim;
  const __nv_bfloat16* kl = static_cast<const __nv_bfloat16*>(c->k) + (size_t)layer * layer_elems;
  const __nv_bfloat16* vl = static_cast<const __nv_bfloat16*>(c->v) + (size_t)layer * layer_elems;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, qo, HD, n_heads, (uint64_t)b->total_tokens) ||
      !make_map(&mk, kl, HD, c->n_kv_heads, pool_rows, 16) || !make_map(&mv, vl, HD, c->n_kv_heads, pool_rows, 16))
    return KVS_E_UNSUPPORTED;
  ReplayParams p{};
  p.out = static_cast<__nv_bfloat16*>(qo);
  p.Hq = n_heads;
  p.Hkv = c->n_kv_heads;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  PagedParams g;
  g.seq_slots = b->seq_slots;
  g.cu_tokens = b->cu_tokens;
  g.cu_qt = cu_qt;
  g.lengths = c->lengths;
  g.tables = c->tables;
  g.status = c->status;
  g.num_seqs = b->num_seqs;
  g.max_blocks = c->max_blocks;
  g.pool_rows = (int)pool_rows;
  // upper bound on the query tiles of the batch: ceil(total / 128) + one partial tile per sequence
  const int64_t items = ((int64_t)b->total_tokens + BM - 1) / BM + b->num_seqs;
  const int64_t grid = items * n_heads / 2;
  pair_attn_kernel<true><<<(unsigned)grid, NT2, SMEM2_BYTES, st>>>(mq, mk, mv, p, g);
  return launch_rc();
}

namespace {
// One warp waits on an mbarrier with the library's bounded waits.  mode bit 0: the fast wait
// (default time slices) instead of the suspending one; bit 1: thread 0 arrives first, so the
// wait completes.  out[0] = 1 if the wait gave up, 0 if it saw the phase complete; out[1..2] =
// the wait's clock64 cycles (low, high word).
__global__ void wait_selftest_kernel(int mode, uint32_t limit, int32_t* out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncwarp();
  if ((mode & 2) && threadIdx.x == 0) mbar_arrive(&bar);
  __syncwarp();
  const long long t0 = clock64();
  const bool ok = (mode & 1) ? mbar_wait_fast(&bar, 0, nullptr, limit) : mbar_wait(&bar, 0, nullptr, limit);
  const long long dt = clock64() - t0;
  if (threadIdx.x == 0) {
    out[0] = ok ? 0 : 1;
    out[1] = (int32_t)(dt & 0xffffffffLL);
    out[2] = (int32_t)(dt >> 32);
  }
}
}  // namespace

KVS_API int kvs_selftest_wait(int32_t mode, uint32_t limit, int32_t* out, kvs_stream_t stream) {
  if (!out || mode < 0 || mode > 3 || limit == 0) return KVS_E_ARG;
  wait_selftest_kernel<<<1, 32, 0, to_cuda(stream)>>>(mode, limit, out);
  return launch_rc();
}

KVS_API int kvs_selftest_umma(const void* a, const void* b, float* c, int32_t mode, int32_t* error,
                              kvs_stream_t stream) {
  if (!a || !b || !c || !error || mode < 0 || mode > 3) return KVS_E_ARG;
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15)) return KVS_E_ARG;
  CUtensorMap ma, mb;
  if (!make_map(&ma, a, 128, 1, 128) || !make_map(&mb, b, 128, 1, 128)) return KVS_E_UNSUPPORTED;
  const int smem = 2 * TILE_BYTES + 128 + 1024;
  if (!set_smem_attr(reinterpret_cast<const void*>(umma_selftest_kernel), 1, smem)) return KVS_E_LAUNCH;
  umma_selftest_kernel<<<1, 128, smem, to_cuda(stream)>>>(ma, mb, mode, static_cast<const uint32_t*>(a), c, error);
  return launch_rc();
}
