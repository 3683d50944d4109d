// Entry points that choose between the tensor-core kernels and the exact SIMT
// kernels by dtype and shape (all kernels are this library's own sm_100a code).
#include "kvs_common.cuh"

int kvs_decode_generic(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a, cudaStream_t st);
size_t kvs_decode_bf16_scratch(const kvs_cache* c, int num_seqs, int grid);
bool kvs_decode_bf16_supported(const kvs_cache* c, const kvs_batch* b, int n_heads);
int kvs_decode_bf16_grid(int override_ctas);
int kvs_decode_bf16_launch(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a, int grid,
                           cudaStream_t st);
int kvs_rope_append(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a, cudaStream_t st);
size_t kvs_prefill_tc_scratch(int num_seqs);
bool kvs_prefill_tc_capable(const kvs_cache* c, int n_heads);
int kvs_prefill_tc_launch(const kvs_cache* c, const kvs_batch* b, int layer, void* qo, int n_heads, double scale,
                          void* scratch, cudaStream_t st);
int kvs_replay_generic(const kvs_replay_args* a, cudaStream_t st);
size_t kvs_replay_tc_scratch(int B, int T);
bool kvs_replay_tc_supported(const kvs_replay_args* a);
int kvs_replay_tc_launch(const kvs_replay_args* a, cudaStream_t st);

using namespace kvs;

#include <atomic>

static std::atomic<long long> g_launches{0};
void kvs::count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

KVS_API long long kvs_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

// Scratch of one kvs_paged_decode call: the decode kernel's region (partial rows and
// zeroed arrival counters), then the chunked-prefill region (per-sequence query-tile offsets).
static size_t decode_region_bytes(const kvs_cache* c, int num_seqs, int n_heads, int grid_ctas) {
  const kvs_batch probe = {nullptr, nullptr, num_seqs, num_seqs};
  if (!kvs_decode_bf16_supported(c, &probe, n_heads)) return 0;
  return kvs_decode_bf16_scratch(c, num_seqs, kvs_decode_bf16_grid(grid_ctas));
}

KVS_API size_t kvs_decode_scratch_bytes(const kvs_cache* c, int32_t num_seqs, int32_t n_heads,
                                        int32_t grid_ctas) {
  if (!c || num_seqs <= 0 || n_heads <= 0) return 0;
  size_t bytes = decode_region_bytes(c, num_seqs, n_heads, grid_ctas);
  if (kvs_prefill_tc_capable(c, n_heads)) bytes += kvs_prefill_tc_scratch(num_seqs);
  return bytes;
}

// Kernels one call over a batch of sequences runs (no mixed step): KVS_PATH_FUSED_DECODE,
// KVS_PATH_TC_PREFILL or KVS_PATH_EXACT.
static int single_path(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a) {
  // the tensor-core kernels store outputs with 16-byte vector writes
  const bool out_aligned = (reinterpret_cast<uintptr_t>(a->out) & 15) == 0;
  // the fused bf16 decode kernel also reads q / k_new / v_new / inv_freq with 16-byte loads
  const bool in_aligned = ((reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k_new) |
                            reinterpret_cast<uintptr_t>(a->v_new) | reinterpret_cast<uintptr_t>(a->inv_freq)) &
                           15) == 0 &&
                          a->q_stride % 8 == 0 && a->kv_stride % 8 == 0;
  if (out_aligned && in_aligned && kvs_decode_bf16_supported(c, b, a->n_heads)) return KVS_PATH_FUSED_DECODE;
  if (b->cu_tokens != nullptr && out_aligned && kvs_prefill_tc_capable(c, a->n_heads)) {
    const size_t off = decode_region_bytes(c, b->num_seqs, a->n_heads, a->grid_ctas);
    if (a->scratch && a->scratch_bytes >= off + kvs_prefill_tc_scratch(b->num_seqs)) return KVS_PATH_TC_PREFILL;
  }
  return KVS_PATH_EXACT;
}

static bool check_decode_args(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a) {
  if (!c || !b || !a || !a->q || !a->k_new || !a->v_new || !a->positions || !a->slot_blocks ||
      !a->slot_offsets || !a->inv_freq || !a->out)
    return false;
  if (b->cu_tokens == nullptr && b->total_tokens != b->num_seqs) return false;
  if (a->layer < 0 || a->layer >= c->n_layers || a->n_heads <= 0 || a->n_heads % c->n_kv_heads) return false;
  return true;
}

// A mixed step (chunks first, then tail_singles one-token sequences) as two sub-calls.
static bool split_mixed(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a, kvs_batch* bc,
                        kvs_decode_args* ac, kvs_batch* bs_, kvs_decode_args* as_) {
  const int ns = a->tail_singles, nc = b->num_seqs - ns, tok1 = b->total_tokens - ns;
  if (ns > b->num_seqs || tok1 < nc) return false;
  const size_t qrow = a->q_stride ? (size_t)a->q_stride : (size_t)a->n_heads * c->head_dim;
  const size_t kvrow = a->kv_stride ? (size_t)a->kv_stride : (size_t)c->n_kv_heads * c->head_dim;
  const size_t orow = (size_t)a->n_heads * c->head_dim;  // out is packed
  const size_t esz = c->dtype == KVS_F64 ? 8 : (c->dtype == KVS_F32 ? 4 : 2);
  *bs_ = {b->seq_slots + nc, nullptr, ns, ns};
  *as_ = *a;
  as_->q = static_cast<const uint8_t*>(a->q) + tok1 * qrow * esz;
  as_->k_new = static_cast<const uint8_t*>(a->k_new) + tok1 * kvrow * esz;
  as_->v_new = static_cast<const uint8_t*>(a->v_new) + tok1 * kvrow * esz;
  as_->positions = a->positions + tok1;
  as_->slot_blocks = a->slot_blocks + tok1;
  as_->slot_offsets = a->slot_offsets + tok1;
  as_->out = static_cast<uint8_t*>(a->out) + tok1 * orow * esz;
  as_->tail_singles = 0;
  // the chunks' prefill region of the scratch may cover where a stored plan of the singles
  // would lie: a mixed step computes its decode plan in every layer
  as_->plan = KVS_PLAN_NONE;
  *bc = {b->seq_slots, b->cu_tokens, nc, tok1};
  *ac = *a;
  ac->tail_singles = 0;
  return true;
}

KVS_API int kvs_paged_decode_path(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a) {
  if (!check_decode_args(c, b, a)) return KVS_E_ARG;
  if (b->num_seqs == 0) return 0;
  if (b->cu_tokens != nullptr && a->tail_singles > 0) {
    kvs_batch bc, bs_;
    kvs_decode_args ac, as_;
    if (!split_mixed(c, b, a, &bc, &ac, &bs_, &as_)) return KVS_E_ARG;
    return (bc.num_seqs > 0 ? single_path(c, &bc, &ac) : 0) | single_path(c, &bs_, &as_);
  }
  return single_path(c, b, a);
}

KVS_API int kvs_paged_decode(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a,
                             kvs_stream_t stream) {
  if (!check_decode_args(c, b, a)) return KVS_E_ARG;
  if (b->num_seqs == 0) return KVS_OK;
  const cudaStream_t st = to_cuda(stream);
  if (b->cu_tokens != nullptr && a->tail_singles > 0) {
    kvs_batch bc, bs_;
    kvs_decode_args ac, as_;
    if (!split_mixed(c, b, a, &bc, &ac, &bs_, &as_)) return KVS_E_ARG;
    if (bc.num_seqs > 0) {
      const int rc = kvs_paged_decode(c, &bc, &ac, stream);
      if (rc) return rc;
    }
    return kvs_paged_decode(c, &bs_, &as_, stream);
  }
  switch (single_path(c, b, a)) {
    case KVS_PATH_FUSED_DECODE:
      return kvs_decode_bf16_launch(c, b, a, kvs_decode_bf16_grid(a->grid_ctas), st);
    case KVS_PATH_TC_PREFILL: {
      // chunks (prefill): RoPE + append, then the tensor-core paged attention in place on `out`
      const size_t off = decode_region_bytes(c, b->num_seqs, a->n_heads, a->grid_ctas);
      int rc = kvs_rope_append(c, b, a, st);
      if (rc) return rc;
      uint8_t* region = static_cast<uint8_t*>(a->scratch) + off;
      rc = kvs_prefill_tc_launch(c, b, a->layer, a->out, a->n_heads, a->scale, region, st);
      if (rc) return rc;
      // the whole scratch buffer stays zero between calls: a later decode call with more
      // sequences finds its arrival counters where these tile offsets were
      return cudaMemsetAsync(region, 0, kvs_prefill_tc_scratch(b->num_seqs), st) == cudaSuccess ? KVS_OK
                                                                                       : KVS_E_LAUNCH;
    }
    default:
      return kvs_decode_generic(c, b, a, st);
  }
}

KVS_API size_t kvs_replay_scratch_bytes(int32_t batch, int32_t seq_len) {
  if (batch <= 0 || seq_len <= 0) return 0;
  return kvs_replay_tc_scratch(batch, seq_len);
}

KVS_API int kvs_replay_attention(const kvs_replay_args* a, kvs_stream_t stream) {
  if (!a || !a->q || !a->k || !a->v || !a->evicted_at || !a->lengths || !a->out || a->batch < 0 ||
      a->seq_len < 0 || a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads ||
      a->head_dim <= 0)
    return KVS_E_ARG;
  if (a->batch == 0 || a->seq_len == 0) return KVS_OK;
  if (!(a->flags & 1) && kvs_replay_tc_supported(a)) return kvs_replay_tc_launch(a, to_cuda(stream));
  return kvs_replay_generic(a, to_cuda(stream));
}
