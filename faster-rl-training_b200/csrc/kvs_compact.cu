// Device-side compaction: the policy decision (compaction/policies.py:34-170), the in-place
// eviction (kvs_evict_positions) and the rollout bookkeeping (engine/base.py:260-308) for a
// batch of rollouts, without a host round trip.

#include <algorithm>

#include "kvs_common.cuh"

using namespace kvs;

namespace {

constexpr int kPlanThreads = 1024;
constexpr int kFlagProtected = 1, kFlagPartial = 2;

// live[i] = the cache's live entries of the slot + pending tokens; need[i] = step[i][1]
__global__ void compact_live_kernel(kvs_cache c, kvs_batch b, const int32_t* __restrict__ step,
                                    int32_t* __restrict__ live, int32_t* __restrict__ need) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= b.num_seqs) return;
  live[i] = c.lengths[b.seq_slots[i]] + step[3 * i];
  need[i] = step[3 * i + 1];
}

// CompactionPolicy.plan of one sequence (policies.py:34-170) in one pass over its segment
// table: the turn policies choose alive, whole, unprotected segments that are not among the
// keep_last most recent alive-and-whole ones (_evictable, :34-38), KeepRecentTurns stopping
// once the overflow is freed (:74-81); TokenSlidingWindow cuts from the end of the prompt to
// min(stream end - window, start of the last segment) (:146-158).  Spans arrive in stream
// order, so merge_spans (utils/spans.py:10-18) is a running merge.  Returns the span count.
__device__ int plan_one(const kvs_segments& s, int slot, int policy, int param, int budget, int live, int need,
                        int64_t* __restrict__ sp, int32_t* __restrict__ ch, int* n_chosen) {
  const int64_t base = (int64_t)slot * s.max_segs;
  const int n = min(s.count[slot], s.max_segs);
  const int32_t* st = s.start + base;
  const int32_t* en = s.end + base;
  const int32_t* ev = s.evicted_at + base;
  const int32_t* fl = s.flags + base;
  int ns = 0, nc = 0;
  auto add = [&](int a, int e) {
    if (e <= a) return;
    if (ns > 0 && a <= sp[2 * ns - 1]) {
      sp[2 * ns - 1] = max(sp[2 * ns - 1], (int64_t)e);
    } else {
      sp[2 * ns] = a;
      sp[2 * ns + 1] = e;
      ++ns;
    }
  };
  const int required = live + need;
  if (required > budget && n > 0) {
    if (policy == KVS_POLICY_TOKEN_WINDOW) {
      int prompt_end = 0;
      for (int j = 0; j < n; ++j)
        if (fl[j] & kFlagProtected) prompt_end = max(prompt_end, en[j]);
      const int cut = min(en[n - 1] - param, st[n - 1]);
      if (cut > prompt_end) {
        for (int j = 0; j < n; ++j)
          if (st[j] < cut && en[j] > prompt_end && ev[j] < 0) ch[nc++] = j;
        add(prompt_end, cut);
      }
    } else {
      int whole = 0;
      for (int j = 0; j < n; ++j) whole += (ev[j] < 0 && !(fl[j] & kFlagPartial)) ? 1 : 0;
      const int overflow = required - budget;
      int freed = 0, rank = 0;
      for (int j = 0; j < n; ++j) {
        if (ev[j] >= 0 || (fl[j] & kFlagPartial)) continue;
        const bool recent = rank >= whole - param;
        ++rank;
        if (recent || (fl[j] & kFlagProtected)) continue;
        if (policy == KVS_POLICY_KEEP_RECENT && freed >= overflow) break;
        ch[nc++] = j;
        freed += en[j] - st[j];
        add(st[j], en[j]);
      }
    }
  }
  *n_chosen = nc;
  return ns;
}

// One CTA: a thread per sequence, cu_spans by a block scan carried across rounds of
// kPlanThreads sequences.
__global__ void __launch_bounds__(kPlanThreads)
compact_plan_kernel(kvs_segments s, kvs_batch b, int policy, int param, int budget, const int32_t* __restrict__ live,
                    const int32_t* __restrict__ need, int64_t* __restrict__ spans, int32_t* __restrict__ n_spans,
                    int32_t* __restrict__ chosen, int32_t* __restrict__ n_chosen, int32_t* __restrict__ cu_spans,
                    int64_t* __restrict__ ss, int64_t* __restrict__ se) {
  __shared__ int scan[33];
  int carry = 0;
  for (int base = 0; base < b.num_seqs; base += blockDim.x) {
    const int i = base + threadIdx.x;
    int ns = 0;
    int64_t* sp = spans + (int64_t)i * s.max_segs * 2;
    if (i < b.num_seqs) {
      int nc = 0;
      ns = plan_one(s, b.seq_slots[i], policy, param, budget, live[i], need[i], sp,
                    chosen + (int64_t)i * s.max_segs, &nc);
      n_spans[i] = ns;
      n_chosen[i] = nc;
    }
    int tot = 0;
    const int pre = block_exclusive_scan(ns, scan, &tot);
    if (i < b.num_seqs) {
      cu_spans[i] = carry + pre;
      for (int k = 0; k < ns; ++k) {
        ss[carry + pre + k] = sp[2 * k];
        se[carry + pre + k] = sp[2 * k + 1];
      }
    }
    carry += tot;
  }
  if (threadIdx.x == 0) cu_spans[b.num_seqs] = carry;
}

// engine/base.py:275-308 after the eviction: event, stats and segment marks; a thread per sequence.
__global__ void compact_commit_kernel(kvs_cache c, kvs_segments s, kvs_batch b, int budget,
                                      const int32_t* __restrict__ step, const int32_t* __restrict__ live,
                                      const int64_t* __restrict__ spans, const int32_t* __restrict__ n_spans,
                                      const int32_t* __restrict__ chosen, const int32_t* __restrict__ n_chosen,
                                      const int64_t* __restrict__ out_spans, const int32_t* __restrict__ out_counts,
                                      int cap) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= b.num_seqs) return;
  const int slot = b.seq_slots[i];
  const int pend = step[3 * i], need = step[3 * i + 1], now = step[3 * i + 2];
  const int live_before = live[i];
  if (live_before + need <= budget) return;  // no compaction considered (base.py:264-265)
  const int live_after = c.lengths[slot] + pend;
  const int ne = min(out_counts[i], cap);
  int32_t* stats = s.stats + (int64_t)slot * 4;
  if (ne > 0) {
    const int64_t* evs = out_spans + (int64_t)i * cap * 2;
    stats[0] += 1;
    stats[1] += live_before - live_after;
    // the event (base.py:287-297)
    const int nr = n_spans[i], nc = n_chosen[i];
    const int e = s.ev_count[slot];
    int32_t* fill = s.ev_fill + (int64_t)slot * 2;
    if (e < s.max_events && fill[0] + nr + ne <= s.span_pool && fill[1] + nc <= s.seg_pool) {
      int32_t* m = s.ev_meta + ((int64_t)slot * s.max_events + e) * KVS_EV_FIELDS;
      m[KVS_EV_TIME] = now;
      m[KVS_EV_LIVE_BEFORE] = live_before;
      m[KVS_EV_LIVE_AFTER] = live_after;
      m[KVS_EV_CACHED_BEFORE] = live_before - pend;
      m[KVS_EV_N_REQUESTED] = nr;
      m[KVS_EV_N_EVICTED] = ne;
      m[KVS_EV_N_SEGMENTS] = nc;
      m[KVS_EV_SPAN_OFFSET] = fill[0];
      m[KVS_EV_SEG_OFFSET] = fill[1];
      int64_t* pool = s.ev_spans + ((int64_t)slot * s.span_pool + fill[0]) * 2;
      const int64_t* sp = spans + (int64_t)i * s.max_segs * 2;
      for (int k = 0; k < 2 * nr; ++k) pool[k] = sp[k];
      for (int k = 0; k < 2 * ne; ++k) pool[2 * nr + k] = evs[k];
      int32_t* sg = s.ev_segs + (int64_t)slot * s.seg_pool + fill[1];
      const int32_t* chs = chosen + (int64_t)i * s.max_segs;
      for (int k = 0; k < nc; ++k) sg[k] = chs[k];
      fill[0] += nr + ne;
      fill[1] += nc;
      s.ev_count[slot] = e + 1;
    } else {
      set_status(c.status, KVS_ST_LOG_CAPACITY, slot, e, fill[0]);
    }
    // segment marks (base.py:300-308)
    const int64_t base = (int64_t)slot * s.max_segs;
    const int n = min(s.count[slot], s.max_segs);
    for (int j = 0; j < n; ++j) {
      if (s.evicted_at[base + j] >= 0) continue;
      const int64_t a0 = s.start[base + j], e0 = s.end[base + j];
      int64_t covered = 0;
      for (int k = 0; k < ne; ++k) covered += max((int64_t)0, min(e0, evs[2 * k + 1]) - max(a0, evs[2 * k]));
      if (covered >= e0 - a0) {
        s.evicted_at[base + j] = now;
        s.flags[base + j] &= ~kFlagPartial;
      } else if (covered > 0) {
        s.flags[base + j] |= kFlagPartial;
      }
    }
  }
  if (live_after + need > budget) stats[2] += 1;  // base.py:274-275
}

struct CompactScratch {
  int32_t *live, *need, *n_spans, *chosen, *n_chosen, *cu, *out_counts;
  int64_t *spans, *ss, *se, *out_spans;
  void* evict;
  size_t evict_bytes;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t compact_layout(const kvs_cache* c, const kvs_segments* s, int n, void* base, CompactScratch* o) {
  const size_t S = (size_t)n, M = (size_t)s->max_segs, cap = (size_t)c->max_blocks;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align256(off + bytes);
    return at;
  };
  const size_t o_live = take(S * 4), o_need = take(S * 4), o_ns = take(S * 4), o_ch = take(S * M * 4),
               o_nc = take(S * 4), o_cu = take((S + 1) * 4), o_oc = take(S * 4), o_sp = take(S * M * 16),
               o_ss = take(S * M * 8), o_se = take(S * M * 8), o_os = take(S * cap * 16);
  const size_t ev_bytes = kvs_evict_scratch_bytes(n, c->max_blocks);
  const size_t o_ev = take(ev_bytes);
  if (o) {
    uint8_t* p = static_cast<uint8_t*>(base);
    o->live = reinterpret_cast<int32_t*>(p + o_live);
    o->need = reinterpret_cast<int32_t*>(p + o_need);
    o->n_spans = reinterpret_cast<int32_t*>(p + o_ns);
    o->chosen = reinterpret_cast<int32_t*>(p + o_ch);
    o->n_chosen = reinterpret_cast<int32_t*>(p + o_nc);
    o->cu = reinterpret_cast<int32_t*>(p + o_cu);
    o->out_counts = reinterpret_cast<int32_t*>(p + o_oc);
    o->spans = reinterpret_cast<int64_t*>(p + o_sp);
    o->ss = reinterpret_cast<int64_t*>(p + o_ss);
    o->se = reinterpret_cast<int64_t*>(p + o_se);
    o->out_spans = reinterpret_cast<int64_t*>(p + o_os);
    o->evict = p + o_ev;
    o->evict_bytes = ev_bytes;
  }
  return off;
}

bool segments_ok(const kvs_segments* s) {
  return s && s->start && s->end && s->evicted_at && s->flags && s->count && s->max_segs > 0;
}

}  // namespace

KVS_API int kvs_compact_plan(const kvs_segments* s, const kvs_batch* b, int32_t policy, int32_t param,
                             int32_t budget, const int32_t* live, const int32_t* need, int64_t* spans,
                             int32_t* n_spans, int32_t* chosen, int32_t* n_chosen, int32_t* cu_spans,
                             int64_t* span_start, int64_t* span_end, kvs_stream_t stream) {
  if (!segments_ok(s) || !b || b->num_seqs < 0 || policy < 0 || policy > KVS_POLICY_TOKEN_WINDOW || !live || !need ||
      !spans || !n_spans || !chosen || !n_chosen || !cu_spans || !span_start || !span_end)
    return KVS_E_ARG;
  if (policy != KVS_POLICY_TOKEN_WINDOW && param < 1) return KVS_E_ARG;  // keep_last >= 1 (policies.py:67)
  if (b->num_seqs == 0) return KVS_OK;
  compact_plan_kernel<<<1, kPlanThreads, 0, to_cuda(stream)>>>(*s, *b, policy, param, budget, live, need, spans, n_spans,
                                                              chosen, n_chosen, cu_spans, span_start, span_end);
  return launch_rc();
}

KVS_API size_t kvs_compact_scratch_bytes(const kvs_cache* c, const kvs_segments* s, int32_t num_seqs) {
  if (!c || !segments_ok(s) || num_seqs <= 0) return 0;
  return compact_layout(c, s, num_seqs, nullptr, nullptr);
}

KVS_API int kvs_compact(const kvs_cache* c, const kvs_batch* b, const kvs_segments* s, int32_t policy, int32_t param,
                        int32_t budget, const int32_t* step, void* scratch, size_t scratch_bytes,
                        kvs_stream_t stream) {
  if (!c || !segments_ok(s) || !s->ev_count || !s->ev_meta || !s->ev_spans || !s->ev_segs || !s->ev_fill ||
      !s->stats || !b || b->num_seqs < 0 || !step)
    return KVS_E_ARG;
  if (b->num_seqs == 0) return KVS_OK;
  CompactScratch x;
  if (!scratch || scratch_bytes < compact_layout(c, s, b->num_seqs, nullptr, nullptr)) return KVS_E_SCRATCH;
  compact_layout(c, s, b->num_seqs, scratch, &x);
  const cudaStream_t st = to_cuda(stream);
  const int grid = (b->num_seqs + 255) / 256;
  compact_live_kernel<<<grid, 256, 0, st>>>(*c, *b, step, x.live, x.need);
  int rc = launch_rc();
  if (rc) return rc;
  rc = kvs_compact_plan(s, b, policy, param, budget, x.live, x.need, x.spans, x.n_spans, x.chosen, x.n_chosen, x.cu,
                        x.ss, x.se, stream);
  if (rc) return rc;
  rc = kvs_evict_positions(c, b, x.cu, x.ss, x.se, x.out_spans, x.out_counts, c->max_blocks, x.evict, x.evict_bytes,
                           stream);
  if (rc) return rc;
  compact_commit_kernel<<<grid, 256, 0, st>>>(*c, *s, *b, budget, step, x.live, x.spans, x.n_spans, x.chosen,
                                              x.n_chosen, x.out_spans, x.out_counts, c->max_blocks);
  return launch_rc();
}
