// kvs_evict_positions_noalloc: the batched whole-block eviction of
// kvs_evict_positions, for callers that cannot allocate device memory.
//
// Who needs it: host programs that bind this library's C ABI directly (a Go,
// Java or plain C service over cgo / JNI / dlopen) often have no device
// allocator of their own, and latency-critical rollout loops must not call
// cudaMalloc between decode steps because it can synchronise the whole device.
// Both still own the cache and the input/output buffers; only the eviction's
// internal scratch (per-sequence counts, drop flags, dropped block ids) is taken
// from a fixed array compiled into the library instead of from the caller.
//
// The scratch lives in `g_evict_scratch`, a file-scope static __device__ array of
// kNoAllocScratchBytes (about 1.25 MiB).  Every GPU that loads the library holds
// one copy until the process exits.  Limits: at most kNoAllocMaxSeqs sequences
// per call and a cache whose tables hold at most kNoAllocMaxBlocks entries per
// sequence; larger requests return KVS_E_NOALLOC_LIMIT without launching.
//
// All calls on a device share the one array and it keeps the previous call's
// contents.  Nothing in it has to start at zero: the first eviction kernel
// writes every count, flag and snapshot before the second one reads it.  Calls
// whose kernels overlap on the GPU (different streams, or host threads racing
// on one device) use the same bytes and therefore race; serialise them.
//
// Host code must not pass `g_evict_scratch` itself to a kernel: in host code the
// name is only a host-side stand-in for the symbol.  The device address is
// obtained once per device with cudaGetSymbolAddress while that device is
// current, on the first call that runs on it; make that first call before any
// stream capture begins.  The address stays cached for the life of the process, so
// do not call cudaDeviceReset (or otherwise tear down the device's context) while
// the library is in use: the reloaded module may place the array elsewhere.
#include "kvs_common.cuh"

#include <mutex>

namespace {

constexpr int kNoAllocMaxSeqs = 256;
constexpr int kNoAllocMaxBlocks = 1024;
constexpr int kMaxDevices = 64;
// Same layout as kvs_evict_scratch_bytes(kNoAllocMaxSeqs, kNoAllocMaxBlocks):
// 256-byte aligned snapshot word, counts, drop flags, dropped block ids.
constexpr size_t kNoAllocScratchBytes = 256 + 2048 + 262144 + 1048576;

}  // namespace

static __device__ __align__(256) unsigned char g_evict_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_evict_scratch on the current device (set up once per device).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KVS_E_LAUNCH;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_evict_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return KVS_E_LAUNCH;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return KVS_OK;
}

}  // namespace

KVS_API int kvs_evict_positions_noalloc(const kvs_cache* c, const kvs_batch* b, const int32_t* cu_spans,
                                        const int64_t* span_start, const int64_t* span_end, int64_t* out_spans,
                                        int32_t* out_counts, int32_t span_cap, kvs_stream_t stream) {
  if (!c || !b || b->num_seqs < 0) return KVS_E_ARG;
  if (b->num_seqs > kNoAllocMaxSeqs || c->max_blocks > kNoAllocMaxBlocks) return KVS_E_NOALLOC_LIMIT;
  const size_t need = kvs_evict_scratch_bytes(b->num_seqs, c->max_blocks);
  if (need > kNoAllocScratchBytes) return KVS_E_NOALLOC_LIMIT;
  if (b->num_seqs == 0) return KVS_OK;
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != KVS_OK) return rc;
  return kvs_evict_positions(c, b, cu_spans, span_start, span_end, out_spans, out_counts, span_cap, scratch,
                             kNoAllocScratchBytes, stream);
}
