// token_logprobs' lm_head stage without materialising the logits (training/logprobs.py:17-20):
// for hidden rows h [M][K] (bf16) and the lm_head weight W [N][K] (bf16), with x = h W^T,
//   lse[r]  = log sum_n exp(x[r][n] / T)
//   logp[r] = x[r][target[r]] / T - lse[r]
// The GEMM runs on the tensor cores in float32 and its epilogue reduces every 256-wide vocab
// tile of a row to (max, sum of 2^(x s - max)), s = log2(e) / T; the [M][N] float32 logits
// (4.2 GB per 8192-token chunk at N = 128256) never reach HBM.  A small second kernel merges
// the per-tile partials of each row.
//
// Work unit: 256 rows x 256 vocab entries, computed by a pair of CTAs (a 2-CTA cluster) with
// M = 256 tcgen05 MMAs (cta_group::2): each CTA stages its own 128 rows of h and its own 128
// rows of W per 64-wide K block, the even CTA issues the MMAs, and each CTA's TMEM receives
// its 128 accumulator rows x 256 columns.  Compared with one CTA per 128 x 256 tile, every SM
// stages a third less operand data per FLOP, which keeps a 1 GB weight and a 64 MB activation
// block streaming from L2 at tensor speed.  Persistent grid: pair p takes units p, p + P, ...
// in vocab-tile-major order, so the pairs in flight read the same few W tiles (from L2) while
// the h rows stay resident in L2.
//
// Roles per CTA (256 threads): warp 0 lane 0 = TMA producer (6-stage ring of 32 KB), warp 1
// = TMEM allocation and, in the even CTA, the MMA issuer; warps 4..7 = epilogue (warp w
// reads TMEM lanes 32 (w - 4) .. +32, one row per thread).  TMEM holds two 256-column
// accumulators, so the epilogue of one unit overlaps the MMAs of the next.
//
// Barriers: full[s] (even CTA's; both CTAs' copies complete on it, the even CTA's producer
// posts the byte count of both), empty[s] (each CTA's; the MMA warp commits to both),
// acc_full[b] (each CTA's; committed to both after a unit's last MMA), acc_empty[b] (even
// CTA's; one arrival per epilogue warp of both CTAs).  Every wait is bounded; a wait that
// runs out records its site in the error word, and the merge kernel then writes NaN.
#include "kvs_common.cuh"
#include "kvs_sm100.cuh"

#include <mutex>

using namespace kvs;
using namespace kvs::sm100;

namespace {

constexpr int BM = 128;          // rows of h per CTA (256 per pair)
constexpr int BN = 256;          // vocab entries per unit (128 per CTA's share of W)
constexpr int BK = 64;           // K elements per stage (one 128-byte swizzled row)
constexpr int STAGES = 6;
constexpr int TILE_BYTES = BM * BK * 2;       // 16 KB: 128 rows x 64 bf16
constexpr int STAGE_BYTES = 2 * TILE_BYTES;   // A + B of one CTA
constexpr int NT = 256;
constexpr int OFF_BAR = STAGES * STAGE_BYTES;
enum { B_FULL = 0, B_EMPTY = STAGES, B_ACCF = 2 * STAGES, B_ACCE = 2 * STAGES + 2, B_FINAL = 2 * STAGES + 4,
       NBAR = 2 * STAGES + 5 };
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 232448, "lm_head kernel shared memory");

struct LmHeadParams {
  const int64_t* targets;  // [M]
  float* part_m;           // [n_tiles][M]: max of x s over the tile (log2 units)
  float* part_l;           // [n_tiles][M]: sum of 2^(x s - max)
  float* tlogit;           // [M]: x at the target
  int32_t* error;          // [1]
  int M, N, n_kb, mb, n_units;
  float s;                 // log2(e) / T
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NT, 1)
lmhead_lse_kernel(const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_w,
                  const LmHeadParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the even CTA, which issues the MMAs
  const int pair = (int)(blockIdx.x >> 1), n_pairs = (int)(gridDim.x >> 1);

  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(&bar[i], 1);
    mbar_init(&bar[B_ACCE + 0], 8);  // 4 epilogue warps x 2 CTAs
    mbar_init(&bar[B_ACCE + 1], 8);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barrier inits and the TMEM allocation visible to both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int site) {
    *abort_flag = 1;
    atomicExch(p.error, site);
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      bool ok = true;
      int it = 0;
      for (int u = pair; ok && u < p.n_units; u += n_pairs) {
        const int nt = u / p.mb, mb = u % p.mb;
        const int row = mb * 2 * BM + (int)rank * BM, vrow = nt * BN + (int)rank * BM;
        for (int kb = 0; kb < p.n_kb; ++kb, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(&bar[B_EMPTY + s], ((it / STAGES) - 1) & 1, abort_flag)) {
            fail(1);
            ok = false;
            break;
          }
          const uint32_t full = mapa_shared(&bar[B_FULL + s], 0);
          if (rank == 0) mbar_arrive_expect_tx(&bar[B_FULL + s], 2 * STAGE_BYTES);
          uint8_t* st = smem + s * STAGE_BYTES;
          tma_load_2d_pair(st, &tm_h, kb * BK, row, full);
          tma_load_2d_pair(st + TILE_BYTES, &tm_w, kb * BK, vrow, full);
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------------------------------------------------------- MMA issuer (even CTA)
      constexpr uint32_t IDESC = idesc_bf16(2 * BM, BN, 0);
      const uint32_t base = smem_addr(smem);
      bool ok = true;
      int it = 0, ui = 0;
      for (int u = pair; ok && u < p.n_units; u += n_pairs, ++ui) {
        const int ab = ui & 1;
        if (ui >= 2) {
          ok = __all_sync(0xffffffffu, mbar_wait_fast(&bar[B_ACCE + ab], ((ui >> 1) - 1) & 1, abort_flag));
          if (!ok) break;
        }
        tc_fence_after();
        const uint32_t d = tmem + ab * BN;
        for (int kb = 0; kb < p.n_kb; ++kb, ++it) {
          const int s = it % STAGES;
          ok = __all_sync(0xffffffffu, mbar_wait_fast(&bar[B_FULL + s], (it / STAGES) & 1, abort_flag));
          if (!ok) break;
          tc_fence_after();
          const uint64_t da = desc_kmajor_sw128(base + s * STAGE_BYTES);
          const uint64_t db = desc_kmajor_sw128(base + s * STAGE_BYTES + TILE_BYTES);
          // four K16 steps: +32 bytes each along the swizzled 128-byte row
          umma_pair_warp_at<0, 0>(d, da, db, IDESC, kb > 0);
          umma_pair_warp_at<2, 2>(d, da, db, IDESC, 1);
          umma_pair_warp_at<4, 4>(d, da, db, IDESC, 1);
          umma_pair_warp_at<6, 6>(d, da, db, IDESC, 1);
          umma_commit_pair_warp(mapa_shared(&bar[B_EMPTY + s], 0));
          umma_commit_pair_warp(mapa_shared(&bar[B_EMPTY + s], 1));
        }
        if (!ok) break;
        umma_commit_pair_warp(mapa_shared(&bar[B_ACCF + ab], 0));
        umma_commit_pair_warp(mapa_shared(&bar[B_ACCF + ab], 1));
      }
      if (!ok && lane == 0) fail(2);
      // every MMA issued has completed before TMEM is released
      umma_commit_pair_warp(mapa_shared(&bar[B_FINAL], 0));
      mbar_wait(&bar[B_FINAL], 0, nullptr);
      __syncwarp();
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- epilogue
    const int q = warp - 4;  // TMEM lane quadrant
    const int r_local = q * 32 + lane;
    const uint32_t acce = mapa_shared(&bar[B_ACCE], 0);
    const float s = p.s;
    int ui = 0;
    for (int u = pair; u < p.n_units; u += n_pairs, ++ui) {
      const int ab = ui & 1;
      const int nt = u / p.mb, mb = u % p.mb;
      const int grow = mb * 2 * BM + (int)rank * BM + r_local;
      const int n0 = nt * BN;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&bar[B_ACCF + ab], (ui >> 1) & 1, abort_flag));
      if (!ok) {
        if (lane == 0) fail(3);
        break;
      }
      tc_fence_after();
      const int tcol = grow < p.M ? (int)(p.targets[grow] - n0) : -1;
      const int valid = min(BN, p.N - n0);
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + ab * BN;
      float m = -INFINITY, l = 0.f, tv = 0.f;
      bool found = false;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(taddr + c * 32, v);
        tmem_wait_ld();
        const int cv = min(32, valid - c * 32);  // vocab entries of this chunk that exist
        float cm = -INFINITY;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float x = __uint_as_float(v[j]);
          if (j < cv) cm = fmaxf(cm, x);
          if (j < cv && c * 32 + j == tcol) {  // a target past the vocabulary stays NaN
            tv = x;
            found = true;
          }
        }
        if (cv <= 0) continue;
        cm *= s;
        if (cm > m) {
          l *= ex2_approx(m - cm);  // 0 on the first chunk (m = -inf)
          m = cm;
        }
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          if (j < cv) a0 += ex2_approx(__uint_as_float(v[j]) * s - m);
          if (j + 1 < cv) a1 += ex2_approx(__uint_as_float(v[j + 1]) * s - m);
        }
        l += a0 + a1;
      }
      // this thread's TMEM reads are done: release the accumulator to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce + ab * 8);
      if (grow < p.M) {
        p.part_m[(int64_t)nt * p.M + grow] = m;
        p.part_l[(int64_t)nt * p.M + grow] = l;
        if (found) p.tlogit[grow] = tv;
      }
    }
  }
  tc_fence_before();
  cluster_sync();  // both CTAs done with TMEM and with each other's barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// One thread per row: merge the per-tile partials.  NaN outputs if the GEMM kernel gave up.
__global__ void lmhead_merge_kernel(const float* __restrict__ part_m, const float* __restrict__ part_l,
                                    const float* __restrict__ tlogit, const int32_t* __restrict__ error, int M,
                                    int n_tiles, float inv_temp, float* __restrict__ logp, float* __restrict__ lse) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= M) return;
  if (*error != 0) {
    logp[r] = __int_as_float(0x7fc00000);
    lse[r] = __int_as_float(0x7fc00000);
    return;
  }
  float mm = -INFINITY;
  for (int t = 0; t < n_tiles; ++t) mm = fmaxf(mm, part_m[(int64_t)t * M + r]);
  float L = 0.f;
  for (int t = 0; t < n_tiles; ++t) L += part_l[(int64_t)t * M + r] * exp2f(part_m[(int64_t)t * M + r] - mm);
  const float lse_nat = (mm + log2f(L)) * 0.69314718055994531f;
  logp[r] = tlogit[r] * inv_temp - lse_nat;
  lse[r] = lse_nat;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// rows of `k` bf16 (row pitch `ld` elements): box {64, 128}, 128-byte swizzle; rows past
// `rows` read as zeros
bool make_rows_map(CUtensorMap* m, const void* base, uint64_t k, uint64_t rows, uint64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {k, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {BK, BM};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

std::mutex g_mu;
bool g_attr[64] = {};
int g_clusters[64] = {};

// pairs that can run at once on the current device (0 if the kernel cannot be set up)
int max_pairs() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_attr[dev]) {
    if (cudaFuncSetAttribute(lmhead_lse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
        cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    cudaLaunchConfig_t cfg = {};  // the cluster size (2) is the kernel's compile-time attribute
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, lmhead_lse_kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    g_clusters[dev] = n;
    g_attr[dev] = true;
  }
  return g_clusters[dev];
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

KVS_API size_t kvs_lm_head_logprobs_scratch_bytes(int32_t n_rows, int32_t vocab) {
  if (n_rows <= 0 || vocab <= 0) return 0;
  const size_t tiles = (size_t)(vocab + BN - 1) / BN;
  return 256 + 2 * align256(tiles * n_rows * 4) + align256((size_t)n_rows * 4);
}

KVS_API int kvs_lm_head_logprobs_supported(int32_t hidden) {
  if (hidden <= 0 || hidden % BK) return 0;
  return encode_fn() != nullptr && max_pairs() > 0 ? 1 : 0;
}

KVS_API int kvs_lm_head_logprobs(const void* h, int64_t ld_h, const void* w, int64_t ld_w, int32_t n_rows,
                                 int32_t vocab, int32_t hidden, const int64_t* targets, double temperature,
                                 float* logp, float* lse, void* scratch, size_t scratch_bytes, kvs_stream_t stream) {
  if (!h || !w || !targets || !logp || !lse || !scratch || n_rows < 0 || vocab <= 0 || hidden <= 0 ||
      !(temperature > 0) || ld_h < hidden || ld_w < hidden)
    return KVS_E_ARG;
  if (n_rows == 0) return KVS_OK;
  if (hidden % BK || ld_h % 8 || ld_w % 8 || (reinterpret_cast<uintptr_t>(h) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15))
    return KVS_E_UNSUPPORTED;
  if (scratch_bytes < kvs_lm_head_logprobs_scratch_bytes(n_rows, vocab)) return KVS_E_SCRATCH;
  const int pairs_max = max_pairs();
  if (pairs_max <= 0) return KVS_E_UNSUPPORTED;
  CUtensorMap mh, mw;
  if (!make_rows_map(&mh, h, hidden, n_rows, ld_h) || !make_rows_map(&mw, w, hidden, vocab, ld_w))
    return KVS_E_UNSUPPORTED;
  const int n_tiles = (vocab + BN - 1) / BN;
  const int mb = (n_rows + 2 * BM - 1) / (2 * BM);
  uint8_t* sp = static_cast<uint8_t*>(scratch);
  LmHeadParams p;
  p.error = reinterpret_cast<int32_t*>(sp);
  p.part_m = reinterpret_cast<float*>(sp + 256);
  p.part_l = reinterpret_cast<float*>(sp + 256 + align256((size_t)n_tiles * n_rows * 4));
  p.tlogit = reinterpret_cast<float*>(sp + 256 + 2 * align256((size_t)n_tiles * n_rows * 4));
  p.targets = targets;
  p.M = n_rows;
  p.N = vocab;
  p.n_kb = hidden / BK;
  p.mb = mb;
  p.n_units = n_tiles * mb;
  p.s = (float)(1.4426950408889634 / temperature);
  const cudaStream_t st = to_cuda(stream);
  // the error word, and the target logits as NaN (a target outside [0, vocab) stays NaN)
  if (cudaMemsetAsync(p.error, 0, 4, st) != cudaSuccess ||
      cudaMemsetAsync(p.tlogit, 0xff, (size_t)n_rows * 4, st) != cudaSuccess)
    return KVS_E_LAUNCH;
  const int pairs = min(pairs_max, p.n_units);
  lmhead_lse_kernel<<<2 * pairs, NT, SMEM_BYTES, st>>>(mh, mw, p);
  int rc = launch_rc();
  if (rc) return rc;
  lmhead_merge_kernel<<<(n_rows + 255) / 256, 256, 0, st>>>(p.part_m, p.part_l, p.tlogit, p.error, n_rows, n_tiles,
                                                           (float)(1.0 / temperature), logp, lse);
  return launch_rc();
}
