/*
 * kvs_b200.h -- C ABI of the B200 (sm_100a) KV-streams paged-KV library.
 *
 * Every entry point takes plain device pointers and sizes plus a cudaStream_t,
 * never allocates device memory and never synchronises the stream.  Device-side
 * failures (pool exhausted, double free, invariant violations) are reported
 * through the int32 status words of the cache (`kvs_cache.status`) and read back
 * by the host at its next synchronisation point.  The return value of every
 * function is a host-side code: KVS_OK, or a negative KVS_E_* value for a bad
 * argument / unsupported shape / CUDA launch error (nothing was launched then).
 *
 * Reference interface each entry point replaces (thanhauco/faster-RL-training,
 * package kvstreams 0.2.0) is cited in the comment above it as file:line.
 *
 * Ordering contract for batched calls: a call over `num_seqs` sequences behaves
 * exactly as if the single-sequence reference method had been called once per
 * sequence, in the order of `seq_slots`.  Block ids popped from / pushed to the
 * free stack therefore come out in that canonical order (bit-exact with the
 * reference's LIFO list).
 */
#ifndef KVS_B200_H
#define KVS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kvs_stream_t; /* == cudaStream_t */

#define KVS_ABI_VERSION 4

/* element types of K/V pools and activations */
enum kvs_dtype { KVS_F32 = 0, KVS_F64 = 1, KVS_BF16 = 2, KVS_F16 = 3 };

/* host-side return codes */
enum kvs_rc {
  KVS_OK = 0,
  KVS_E_ARG = -1,         /* null pointer / size out of range */
  KVS_E_UNSUPPORTED = -2, /* shape or dtype the library has no kernel for */
  KVS_E_LAUNCH = -3,      /* cudaGetLastError() after the launch */
  KVS_E_SCRATCH = -4,     /* caller's scratch buffer too small */
  KVS_E_NOALLOC_LIMIT = -5 /* request larger than the built-in scratch of a *_noalloc entry point */
};

/* device-side status codes (status[0]; status[1..3] hold details) */
enum kvs_status {
  KVS_ST_OK = 0,
  KVS_ST_OUT_OF_BLOCKS = 1,    /* paged_cache.py:41-42  OutOfBlocksError */
  KVS_ST_DOUBLE_FREE = 2,      /* paged_cache.py:48-49  ValueError */
  KVS_ST_NOT_FULL_BLOCK = 3,   /* paged_cache.py:202-206 ValueError */
  KVS_ST_TABLE_OVERFLOW = 4,   /* table longer than max_blocks (no reference counterpart) */
  KVS_ST_TRUNCATE = 5,         /* paged_cache.py:247-248 ValueError */
  KVS_ST_INV_DUP_BLOCK = 6,    /* paged_cache.py:265-266 */
  KVS_ST_INV_TABLE_LEN = 7,    /* paged_cache.py:267-268 */
  KVS_ST_INV_HOLE = 8,         /* paged_cache.py:270-271 */
  KVS_ST_INV_ORDER = 9,        /* paged_cache.py:272-273 */
  KVS_ST_SPAN_CAPACITY = 10,   /* evicted-span output buffer too small */
  KVS_ST_OWNER = 11,           /* block freed by a sequence that does not own it */
  KVS_ST_KERNEL_TIMEOUT = 12,  /* a bounded wait inside a tensor-core kernel expired; its outputs
                                  are invalid (no reference counterpart) */
  KVS_ST_SEQ_TOO_LONG = 13,     /* a sequence is longer than the 32768 entries the tensor-core
                                  prefill attends over (no reference counterpart) */
  KVS_ST_LOG_CAPACITY = 14     /* a device compaction event did not fit the sequence's event log */
};

/* CacheStats counters (paged_cache.py:70-78), int64 each */
enum kvs_stat {
  KVS_STAT_WRITTEN_TOKENS = 0,
  KVS_STAT_EVICTED_TOKENS = 1,
  KVS_STAT_EVICTED_BLOCKS = 2,
  KVS_STAT_TRUNCATED_TOKENS = 3,
  KVS_STAT_PEAK_BLOCKS = 4,
  KVS_STAT_EVICTION_CALLS = 5,
  KVS_STAT_SHRUNK_TOKENS = 6,
  KVS_STAT_COUNT = 8
};

#define KVS_STATUS_WORDS 4
#define KVS_NEVER INT64_MAX /* events.py:20 NEVER */

/*
 * Device-resident paged KV cache (paged_cache.py:81-106).
 * Pool layout is the reference's: k, v = [n_layers][num_blocks][block_size][n_kv_heads][head_dim].
 * Sequences live in slots 0..max_seqs-1; table of slot s = tables[s*max_blocks .. +n_blocks[s]).
 * Free list: free_stack[0 .. *free_top) with the next block to hand out at free_stack[*free_top-1]
 * (the reference's `_free` list, popped from its end, paged_cache.py:37,43,51).
 */
typedef struct kvs_cache {
  void* k;
  void* v;
  int64_t* slot_pos;    /* [num_blocks][block_size] logical position, -1 = empty */
  int32_t* tables;      /* [max_seqs][max_blocks] */
  int32_t* n_blocks;    /* [max_seqs] table length */
  int32_t* lengths;     /* [max_seqs] live tokens */
  int32_t* free_stack;  /* [num_blocks] */
  int32_t* free_top;    /* [1] */
  int32_t* block_owner; /* [num_blocks] owning slot, -1 when free (the reference's `_used` set) */
  int64_t* stats;       /* [KVS_STAT_COUNT] */
  int32_t* status;      /* [KVS_STATUS_WORDS] */
  int32_t n_layers;
  int32_t num_blocks;
  int32_t block_size;
  int32_t n_kv_heads;
  int32_t head_dim;
  int32_t max_seqs;
  int32_t max_blocks;
  int32_t dtype; /* enum kvs_dtype of k and v */
} kvs_cache;

/* A batch of sequences processed in the given order.  cu_tokens may be NULL
 * when every sequence contributes exactly one token (decode). */
typedef struct kvs_batch {
  const int32_t* seq_slots; /* [num_seqs] */
  const int32_t* cu_tokens; /* [num_seqs+1] exclusive prefix sum of new tokens, or NULL */
  int32_t num_seqs;
  int32_t total_tokens;
} kvs_batch;

/* size of each public struct as compiled into the library (ABI check):
 * which = 0 kvs_cache, 1 kvs_batch, 2 kvs_decode_args, 3 kvs_replay_args, 4 kvs_segments */
size_t kvs_abi_struct_size(int which);
int kvs_abi_version(void);
/* number of SMs of the current device, cached per device (grid sizing) */
int kvs_device_sm_count(void);
/* kernels launched by this library in this process so far (for launch accounting) */
long long kvs_launch_count(void);

/* ------------------------------------------------------------------ cache state */

/* Reset all metadata to the freshly-constructed state: free stack [NB-1..0]
 * (paged_cache.py:37), slot_pos -1 (:100-102), empty tables, zero stats/status.
 * The K/V pool is not touched (the caller zero-initialises it at allocation). */
int kvs_cache_reset(const kvs_cache* c, kvs_stream_t stream);

/* PagedKVCache.append_slots (paged_cache.py:145-165), batched.
 * positions: [total_tokens] int64.  out_blocks/out_offsets: [total_tokens] int32
 * slot mapping (SlotMapping, paged_cache.py:62-67).  Allocates blocks on demand in
 * canonical order; if the pool cannot cover the whole batch nothing is changed and
 * status = KVS_ST_OUT_OF_BLOCKS. */
int kvs_append_slots(const kvs_cache* c, const kvs_batch* b, const int64_t* positions,
                     int32_t* out_blocks, int32_t* out_offsets, kvs_stream_t stream);

/* PagedKVCache.write (paged_cache.py:167-171): k,v [n_tokens][n_kv_heads][head_dim]
 * (dtype of the pool) stored at the slot mapping, for one layer. */
int kvs_write_kv(const kvs_cache* c, int32_t layer, const int32_t* blocks, const int32_t* offsets,
                 const void* k, const void* v, int32_t n_tokens, kvs_stream_t stream);

/* PagedKVCache.evict_positions (paged_cache.py:219-240), batched.
 * Spans of sequence i: [span_start[j], span_end[j]) for j in cu_spans[i]..cu_spans[i+1];
 * they must be sorted and non-overlapping (merge_spans, utils/spans.py:10-18).
 * Evicts every full block whose live tokens all fall inside the spans, joins the
 * table, resets slot_pos, pushes the freed blocks (ascending table index per
 * sequence, sequences in batch order) and updates CacheStats.
 * Output: the logical spans actually removed (positions_to_spans, spans.py:21-23)
 * for sequence i at out_spans[2*(i*span_cap + r)], r < out_counts[i].
 * scratch: >= kvs_evict_scratch_bytes(num_seqs, max_blocks) bytes of device memory. */
size_t kvs_evict_scratch_bytes(int32_t num_seqs, int32_t max_blocks);
int kvs_evict_positions(const kvs_cache* c, const kvs_batch* b, const int32_t* cu_spans,
                        const int64_t* span_start, const int64_t* span_end,
                        int64_t* out_spans, int32_t* out_counts, int32_t span_cap,
                        void* scratch, size_t scratch_bytes, kvs_stream_t stream);

/* No counterpart in the reference.  kvs_evict_positions for callers that cannot
 * allocate device memory (hosts binding this C ABI without a device allocator of
 * their own, or rollout loops that must not cudaMalloc between steps because it
 * can synchronise the device).  Same arguments and results as
 * kvs_evict_positions minus the scratch buffer: the scratch comes from one
 * ~1.25 MiB array compiled into the library (held by every GPU that loads it
 * until exit).  Limits: num_seqs <= 256 and c->max_blocks <= 1024, else
 * KVS_E_NOALLOC_LIMIT and nothing is launched.  Calls share that array, so calls
 * whose kernels overlap on the GPU race.  The first call on each device looks up
 * the array's device address (cudaGetSymbolAddress); make it before any stream
 * capture.  The address is cached until exit: do not cudaDeviceReset a device
 * while the library is in use.  Allocates nothing. */
int kvs_evict_positions_noalloc(const kvs_cache* c, const kvs_batch* b, const int32_t* cu_spans,
                                const int64_t* span_start, const int64_t* span_end,
                                int64_t* out_spans, int32_t* out_counts, int32_t span_cap,
                                kvs_stream_t stream);

/* PagedKVCache.evict_blocks (paged_cache.py:190-217), batched: drop_flags
 * [num_seqs][max_blocks] uint8 (1 = remove that table index; the host has already
 * checked that every flagged index is a full block).  Same join / free / stats as above. */
int kvs_evict_blocks(const kvs_cache* c, const kvs_batch* b, const uint8_t* drop_flags,
                     void* scratch, size_t scratch_bytes, kvs_stream_t stream);

/* PagedKVCache.truncate (paged_cache.py:242-260) when mode == 0 and
 * PagedKVCache.free_sequence (paged_cache.py:129-133) when mode == 1, batched.
 * new_lengths: [num_seqs] target live length (ignored for mode 1, which frees all). */
int kvs_release(const kvs_cache* c, const kvs_batch* b, const int32_t* new_lengths, int32_t mode,
                kvs_stream_t stream);

/* PagedKVCache.check_invariants (paged_cache.py:262-273), batched.
 * out_codes[i] = KVS_ST_OK or the first KVS_ST_INV_* violated by sequence i.
 * scratch: >= kvs_check_scratch_bytes(num_blocks) bytes. */
size_t kvs_check_scratch_bytes(int32_t num_blocks);
int kvs_check_invariants(const kvs_cache* c, const kvs_batch* b, int32_t* out_codes,
                         void* scratch, size_t scratch_bytes, kvs_stream_t stream);

/* ------------------------------------------------------------------ compute */

/* apply_rope (rope.py:42-46) with RotaryEmbedding angles (rope.py:30-34) at explicit
 * logical positions, in place: x [n_tokens][n_heads][head_dim] of `dtype`.
 * inv_freq: [head_dim/2] float (f32/bf16/f16 activations) or double (f64). */
int kvs_rope(void* x, int32_t dtype, const int64_t* positions, int32_t n_tokens, int32_t n_heads,
             int32_t head_dim, const void* inv_freq, kvs_stream_t stream);
/* The same rotation out of place, in one pass: src token rows src_stride elements apart, dst token
 * rows dst_stride apart (each row's [n_heads][head_dim] block dense; 0 = packed rows), e.g. q or k
 * read from / written to their column block of a fused q|k|v tensor.  Replaces the copy of q / k
 * out of the projection output followed by the in-place rotation (model.py:62-63), and in the
 * backward the assembly of the fused gradient from the rotated-back dq / dk. */
int kvs_rope_copy(const void* src, int64_t src_stride, void* dst, int64_t dst_stride, int32_t dtype,
                  const int64_t* positions, int32_t n_tokens, int32_t n_heads, int32_t head_dim, const void* inv_freq,
                  kvs_stream_t stream);

/* Paged attention of the new tokens of each sequence over its live cache entries
 * (Attention.forward in cached mode, model.py:50-75 with the kv_hook of
 * model.py:182-185 and the mask of model.py:175-176): query i of sequence s attends
 * to cache entries [0, lengths[s] - T_s + i].  q [total_tokens][n_heads][head_dim]
 * already rotated; out same shape.  Must run after the tokens were appended. */
int kvs_paged_attention(const kvs_cache* c, const kvs_batch* b, int32_t layer, const void* q,
                        void* out, int32_t n_heads, double scale, kvs_stream_t stream);

/* One layer of TinyLM.forward_cached (model.py:160-188) for the new tokens of a
 * batch of sequences: RoPE of q and k at `positions`, append of k and v at the
 * slot mapping produced by kvs_append_slots, and paged GQA attention of every new
 * query over the live entries it may see.  One token per sequence (decode,
 * cu_tokens NULL) runs the fused split-K kernel; prefill chunks (cu_tokens set)
 * run rope + append + the tensor-core paged prefill (bf16, head_dim 128, 16-token
 * blocks, even GQA group) or kvs_paged_attention.  A mixed step (cu_tokens set,
 * tail_singles > 0: the last tail_singles sequences have one token each) runs the
 * chunks and the single tokens as two launches of those kernels. */
typedef struct kvs_decode_args {
  const void* q;            /* [total_tokens] rows of [n_heads][head_dim], not yet rotated */
  const void* k_new;        /* [total_tokens] rows of [n_kv_heads][head_dim], not yet rotated */
  const void* v_new;        /* [total_tokens] rows of [n_kv_heads][head_dim] */
  const int64_t* positions; /* [total_tokens] */
  const int32_t* slot_blocks;  /* [total_tokens] from kvs_append_slots */
  const int32_t* slot_offsets; /* [total_tokens] */
  const void* inv_freq;     /* [head_dim/2] float, or double for f64 pools */
  void* out;                /* [total_tokens][n_heads][head_dim] */
  void* scratch;            /* split-K partials + per-sequence counters */
  size_t scratch_bytes;
  double scale;             /* head_dim**-0.5 (model.py:71) */
  int32_t layer;
  int32_t n_heads;
  int32_t grid_ctas;        /* CTAs of the fused decode kernel (0 = one per SM) */
  int32_t tail_singles;     /* with cu_tokens set: the last tail_singles sequences have
                               exactly one new token each (0: no such promise) */
  int64_t q_stride;         /* elements from one token's q row to the next (0: packed, n_heads*head_dim);
                               e.g. the q columns of a fused [tokens][q|k|v] projection output */
  int64_t kv_stride;        /* the same for k_new and v_new (0: packed, n_kv_heads*head_dim) */
  int32_t plan;             /* KVS_PLAN_*: the batch plan of a decode step (below) */
} kvs_decode_args;
/* The batch plan of the fused decode kernel (16-token blocks): how the step's groups of 16
 * live entries are split over the CTAs, and the block id of every group.  The layers of one
 * decode step all have the same plan, so the first layer's call can store it in the scratch
 * (KVS_PLAN_BUILD) and the later layers' calls read it back (KVS_PLAN_REUSE) instead of
 * recomputing it from the block tables.  REUSE is valid only while the batch, its sequences'
 * lengths and block tables and grid_ctas are those of the last BUILD call on the same scratch
 * (one decode step); a REUSE call whose stored plan has another batch size or grid computes
 * the plan itself.  No reference counterpart (the reference's decode recomputes nothing per
 * layer: it gathers every sequence's K/V in PyTorch). */
enum kvs_decode_plan { KVS_PLAN_NONE = 0, KVS_PLAN_BUILD = 1, KVS_PLAN_REUSE = 2 };
/* scratch of kvs_paged_decode: split partials and per-sequence arrival counters of the
 * fused decode kernel, then (bf16, head_dim 128, 16-token blocks, even GQA group) the
 * query-tile offsets of the tensor-core chunked prefill.  Zero it once when allocated:
 * every call leaves it zero, whatever the batch size of the previous call. */
size_t kvs_decode_scratch_bytes(const kvs_cache* c, int32_t num_seqs, int32_t n_heads,
                                int32_t grid_ctas);
int kvs_paged_decode(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a,
                     kvs_stream_t stream);
/* Which kernels kvs_paged_decode would run for these arguments, as an OR of KVS_PATH_* bits
 * (a mixed step reports both sub-batches), or KVS_E_ARG.  Launches nothing; no reference
 * counterpart (the reference has one attention path). */
enum kvs_decode_path {
  KVS_PATH_FUSED_DECODE = 1, /* fused RoPE + append + split-K paged decode (bf16, D 128, 32q/8kv, bs 16 or 1) */
  KVS_PATH_TC_PREFILL = 2,   /* RoPE + append, then the tensor-core paged prefill (bf16 chunks, bs 16) */
  KVS_PATH_EXACT = 4         /* the exact SIMT kernels (every dtype and shape) */
};
int kvs_paged_decode_path(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a);

/* CompactionLog.evicted_at (events.py:66-74), batched: for stream i, events are
 * triples (span_start, span_end, time) j in cu_spans[i]..cu_spans[i+1].
 * out [num_streams][t_stride] int64: min time over spans covering t, KVS_NEVER else;
 * entries t >= lengths[i] are KVS_NEVER. */
int kvs_evicted_at(const int32_t* cu_spans, const int64_t* span_start, const int64_t* span_end,
                   const int64_t* span_time, const int32_t* lengths, int32_t num_streams,
                   int32_t t_stride, int64_t* out, kvs_stream_t stream);

/* Masked replay attention (TinyLM.forward attention, model.py:71-74, with the
 * KV-streams mask of replay.py:55-63 and the collate padding of replay.py:221-222):
 *   visible(t, s) = s <= t && t < evicted_at[b][s]      for t < lengths[b]
 *   visible(t, s) = (s == t)                             for t >= lengths[b]
 * q [B][T][n_heads][head_dim], k,v [B][T][n_kv_heads][head_dim], already rotated;
 * out like q.  Fully masked 128x128 tiles are skipped using per-tile evicted_at bounds. */
typedef struct kvs_replay_args {
  const void* q;
  const void* k;
  const void* v;
  const int64_t* evicted_at; /* [B][T] */
  const int32_t* lengths;    /* [B] */
  void* out;
  void* scratch;
  size_t scratch_bytes;
  int32_t batch;
  int32_t seq_len;
  int32_t n_heads;
  int32_t n_kv_heads;
  int32_t head_dim;
  int32_t dtype;
  double scale;
  int32_t flags; /* bit 0: force the generic SIMT kernel; bit 1: tensor-core kernel
                    with one query head per CTA even when the GQA group size is even
                    (default there: two heads of the group share each K/V tile) */
  int32_t reserved;
  float* row_lse; /* optional [batch][n_heads][seq_len rounded up to 128], 16-byte aligned:
                     log2 of each query row's sum of 2^(scale*log2(e)*q.k) over its visible
                     keys.  Written by every forward path when non-NULL; the backward reads it
                     and, for bf16 with head_dim 128, then runs the tensor-core kernels (NULL
                     there selects the exact kernels). */
} kvs_replay_args;
size_t kvs_replay_scratch_bytes(int32_t batch, int32_t seq_len);
int kvs_replay_attention(const kvs_replay_args* a, kvs_stream_t stream);

/* Backward of kvs_replay_attention: what torch autograd computes for the reference's masked
 * attention (model.py:71-74 under the replay.py:62 mask) when the trainer differentiates
 * token_logprobs (training/logprobs.py:10-25).  Inputs as the forward (q and k rotated, the
 * forward's output in a->out) plus dout; writes dq, dk, dv in the layouts and dtype of q, k,
 * v (dk/dv summed over the query heads of each KV head); a->scratch holds
 * kvs_replay_backward_scratch_bytes.  bf16, head_dim 128 with a->row_lse as the forward left it:
 * tcgen05 kernels (P and dS rounded to bf16 as UMMA operands, fp32 accumulation, no atomics);
 * otherwise exact SIMT kernels (fp32 accumulation, fp64 for double). */
size_t kvs_replay_backward_scratch_bytes(int32_t batch, int32_t seq_len, int32_t n_heads, int32_t dtype);
int kvs_replay_attention_backward(const kvs_replay_args* a, const void* dout, void* dq, void* dk, void* dv,
                                  kvs_stream_t stream);
/* Which kernels kvs_replay_attention_backward runs for these arguments: 1 the tensor-core
 * ones, 0 the exact ones, negative a CUDA error (the first call on a device checks, once and
 * synchronously, that the tensor-core kernels fit it; no reference counterpart). */
int kvs_replay_backward_path(const kvs_replay_args* a, kvs_stream_t stream);

/* ---------------------------------------------------------------- device-side compaction
 * The reference decides compaction on the host, per rollout, before each turn
 * (engine/base.py:260-308 with compaction/policies.py:34-170 over compaction/segments.py).
 * kvs_compact runs that decision, the in-place eviction and its bookkeeping for a batch of
 * rollouts on the device, so a rollout loop needs no device round trip per compaction; the
 * segments, events and stats are read back once, when the rollouts end.  State per sequence
 * slot, all device arrays (zero-initialised; the caller appends segments as turns end):
 *   start, end        [max_seqs][max_segs] stream span of each segment
 *   evicted_at        [max_seqs][max_segs] stream length at the compaction that removed the
 *                     whole segment, -1 while (at least partly) alive
 *   flags             [max_seqs][max_segs] bit 0 protected (the prompt), bit 1 partially evicted
 *   count             [max_seqs] segments in use
 *   ev_count          [max_seqs] events logged
 *   ev_meta           [max_seqs][max_events][KVS_EV_FIELDS] (CompactionEvent, events.py:20-40)
 *   ev_spans          [max_seqs][span_pool][2] requested spans of each event, then evicted ones
 *   ev_segs           [max_seqs][seg_pool] segment indices chosen by each event
 *   ev_fill           [max_seqs][2] entries used in ev_spans / ev_segs
 *   stats             [max_seqs][4] compactions, evicted tokens, budget overflows, 0 */
typedef struct kvs_segments {
  int32_t* start;
  int32_t* end;
  int32_t* evicted_at;
  int32_t* flags;
  int32_t* count;
  int32_t* ev_count;
  int32_t* ev_meta;
  int64_t* ev_spans;
  int32_t* ev_segs;
  int32_t* ev_fill;
  int32_t* stats;
  int32_t max_seqs;
  int32_t max_segs;
  int32_t max_events;
  int32_t span_pool;
  int32_t seg_pool;
  int32_t reserved;
} kvs_segments;

enum kvs_event_field {
  KVS_EV_TIME = 0,          /* stream length when the compaction ran */
  KVS_EV_LIVE_BEFORE = 1,   /* live entries incl. pending tokens (engine/base.py:284) */
  KVS_EV_LIVE_AFTER = 2,
  KVS_EV_CACHED_BEFORE = 3, /* cache entries before the eviction (live_before without pending) */
  KVS_EV_N_REQUESTED = 4,
  KVS_EV_N_EVICTED = 5,
  KVS_EV_N_SEGMENTS = 6,
  KVS_EV_SPAN_OFFSET = 7,   /* first requested span in ev_spans; the evicted ones follow them */
  KVS_EV_SEG_OFFSET = 8,
  KVS_EV_FIELDS = 9
};

enum kvs_policy_code {
  KVS_POLICY_KEEP_RECENT = 0,  /* KeepRecentTurns(keep_last = param) */
  KVS_POLICY_MARKOVIAN = 1,    /* MarkovianPolicy(keep_last = param) */
  KVS_POLICY_SUMMARY = 2,      /* SummaryPolicy's spans (the summary turn itself is the caller's) */
  KVS_POLICY_TOKEN_WINDOW = 3  /* TokenSlidingWindow(window = param) */
};

/* CompactionPolicy.plan for every sequence of the batch whose live[i] + need[i] > budget
 * (engine/base.py:262-267; live incl. pending tokens, need = incoming + reserve), others get no
 * spans.  Per sequence i: spans[i][max_segs][2] merged sorted spans (merge_spans), n_spans[i];
 * chosen[i][max_segs] segment indices, n_chosen[i]; cu_spans[num_seqs+1] and span_start /
 * span_end [num_seqs*max_segs] in kvs_evict_positions' input form. */
int kvs_compact_plan(const kvs_segments* s, const kvs_batch* b, int32_t policy, int32_t param, int32_t budget,
                     const int32_t* live, const int32_t* need, int64_t* spans, int32_t* n_spans, int32_t* chosen,
                     int32_t* n_chosen, int32_t* cu_spans, int64_t* span_start, int64_t* span_end,
                     kvs_stream_t stream);

/* _maybe_compact + _compact (engine/base.py:260-308) for a batch: step [num_seqs][3] device
 * int32 = pending tokens, need (incoming + reserve), stream length.  Plans with live = the
 * cache's live entries + pending, evicts the planned spans (kvs_evict_positions), then for each
 * sequence whose eviction removed something appends the event, adds to its stats and marks its
 * segments (evicted_at = stream length when wholly covered, else partially evicted); a sequence
 * that was over budget and still is counts a budget overflow. */
size_t kvs_compact_scratch_bytes(const kvs_cache* c, const kvs_segments* s, int32_t num_seqs);
int kvs_compact(const kvs_cache* c, const kvs_batch* b, const kvs_segments* s, int32_t policy, int32_t param,
                int32_t budget, const int32_t* step, void* scratch, size_t scratch_bytes, kvs_stream_t stream);

/* token_logprobs' log-softmax + gather (training/logprobs.py:17-20) on lm_head logits
 * [n_rows][ld] (dtype KVS_F32 or KVS_F64, row stride ld >= vocab): logp[r] = x[r][t_r]/T -
 * log sum_v exp(x[r][v]/T) in one pass over each row (a target outside [0, vocab) gives NaN);
 * lse[r] (optional, same dtype) receives the log-sum-exp for the backward. */
int kvs_lse_gather(const void* logits, int64_t ld, int32_t n_rows, int32_t vocab, const int64_t* targets,
                   double temperature, int32_t dtype, void* logp, void* lse, kvs_stream_t stream);
/* Its gradient with respect to the logits for upstream grad[r] (same dtype as logits):
 * dlogits[r][v] = grad[r] * (onehot(t_r)[v] - exp(x[r][v]/T - lse[r])) / T, written in
 * out_dtype (KVS_F32 / KVS_BF16 / KVS_F16 from float logits, KVS_F64 from double ones) with row
 * stride ld_out; dlogits may be the logits buffer itself when the dtypes match. */
int kvs_lse_gather_backward(const void* logits, int64_t ld, int32_t n_rows, int32_t vocab, const int64_t* targets,
                            const void* lse, const void* grad, double temperature, int32_t dtype, void* dlogits,
                            int64_t ld_out, int32_t out_dtype, kvs_stream_t stream);

/* The same log-prob and log-sum-exp straight from the lm_head's inputs, the logits never
 * stored (training/logprobs.py:17-20 with model.py:110-114's lm_head): h [n_rows][ld_h] and
 * the lm_head weight w [vocab][ld_w], both bf16, give x = h w^T (float32 accumulation) and
 * logp[r] = x[r][t_r]/T - lse[r], lse[r] = log sum_v exp(x[r][v]/T), float32.  One tensor-core
 * GEMM (pairs of CTAs, M = 256 per MMA) reduces every 256-wide vocab tile of a row in its
 * epilogue; a second kernel merges the tiles.  Needs hidden % 64 == 0, ld_h and ld_w multiples
 * of 8, 16-byte aligned h and w (KVS_E_UNSUPPORTED otherwise), and scratch of
 * kvs_lm_head_logprobs_scratch_bytes(n_rows, vocab) bytes.  A target outside [0, vocab), or a
 * bounded wait inside the GEMM kernel that ran out, gives NaN.  kvs_lm_head_logprobs_supported
 * says whether this device can run it (0: use a GEMM and kvs_lse_gather). */
size_t kvs_lm_head_logprobs_scratch_bytes(int32_t n_rows, int32_t vocab);
int kvs_lm_head_logprobs_supported(int32_t hidden);
int kvs_lm_head_logprobs(const void* h, int64_t ld_h, const void* w, int64_t ld_w, int32_t n_rows, int32_t vocab,
                         int32_t hidden, const int64_t* targets, double temperature, float* logp, float* lse,
                         void* scratch, size_t scratch_bytes, kvs_stream_t stream);

/* The rollout's next-token step (engine/base.py:180-193: log_softmax(logits / T), then
 * multinomial or argmax, and the token's log-prob) for a batch of logits rows [n_rows][ld]
 * (KVS_F32 or KVS_F64) in one pass over each row.  greedy != 0: tokens[r] = the row's argmax
 * (lowest index among equal maxima).  Otherwise a sample of softmax(x[r] / T) by the Gumbel-max
 * rule, argmax_v x[r][v]/T - log(-log U_v), with U_v from a Philox4x32-10 stream (key = seed,
 * counter = (v / 4, r, offset low word, offset high word), word v % 4; U = ((bits >> 9) + 0.5)
 * * 2^-23): the same seed and offset give the same tokens, a new offset a new draw.
 * logp[r] (logits dtype) = log_softmax(x[r] / T)[tokens[r]].  A row of -inf / NaN only gives
 * tokens[r] = -1 and a NaN log-prob.  Replaces the per-row log_softmax + multinomial/argmax +
 * gather (about 17 launches per batch) with one launch of 4-CTA clusters per row. */
int kvs_sample(const void* logits, int64_t ld, int32_t n_rows, int32_t vocab, double temperature, int32_t dtype,
               int32_t greedy, uint64_t seed, uint64_t offset, int64_t* tokens, void* logp, kvs_stream_t stream);

/* The decoder layer's elementwise steps for half-precision models (KVS_BF16 / KVS_F16), one
 * pass each (model.py:29-36 RMSNorm, model.py:78-86 the MLP's silu(gate) * up):
 * y[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * weight in fp32 with one rounding (rstd[r], optional
 * float32, receives the row's rsqrt for a backward); out[r][j] = silu(gu[r][j]) * gu[r][f + j]
 * from the fused gate|up output, and its gradient dgu[r] = (d gate | d up).  Rows are ld_*
 * elements apart; dim / f and the row strides multiples of 8, pointers 16-byte aligned
 * (KVS_E_UNSUPPORTED otherwise). */
int kvs_rms_norm(const void* x, const void* weight, void* y, float* rstd, int64_t n_rows, int32_t dim, int64_t ld_x,
                 int64_t ld_y, double eps, int32_t dtype, kvs_stream_t stream);
/* Its backward with the forward's rstd: gx[r] = rstd[r] (gxn - xn mean_j(gxn xn)), xn = x[r] rstd[r],
 * gxn = gy[r] weight (fp32, one rounding of gx); gw (float32 [dim]) = sum_r gy[r] xn[r], summed per
 * CTA and then across CTAs in a fixed order (the bits do not depend on scheduling).  dim <= 8192;
 * scratch: kvs_rms_norm_backward_scratch_bytes(n_rows, dim) bytes, 16-byte aligned. */
size_t kvs_rms_norm_backward_scratch_bytes(int64_t n_rows, int32_t dim);
int kvs_rms_norm_backward(const void* x, const void* weight, const float* rstd, const void* gy, void* gx, float* gw,
                          int64_t n_rows, int32_t dim, int64_t ld_x, int64_t ld_gy, int64_t ld_gx, int32_t dtype,
                          void* scratch, size_t scratch_bytes, kvs_stream_t stream);
int kvs_silu_mul(const void* gu, void* out, int64_t n_rows, int32_t f, int64_t ld_gu, int64_t ld_out, int32_t dtype,
                 kvs_stream_t stream);
int kvs_silu_mul_backward(const void* gu, const void* grad, void* dgu, int64_t n_rows, int32_t f, int64_t ld_gu,
                          int64_t ld_grad, int64_t ld_dgu, int32_t dtype, kvs_stream_t stream);

/* Self-test of the tcgen05 path (no reference counterpart): c[128][128] f32 =
 * a[128][128] (bf16 row-major) x B, with B given as bt[128 n][128 k] (mode bit 0 = 0,
 * K-major operand) or b[128 k][128 n] (bit 0 = 1, MN-major operand); mode bit 1 = 1
 * stages A in TMEM (the operand form of the replay kernel's P V) instead of shared
 * memory.  *error is set non-zero if an internal wait timed out.  Validates the UMMA
 * descriptors, TMA swizzle and TMEM layouts that the replay kernel relies on. */
int kvs_selftest_umma(const void* a, const void* b, float* c, int32_t mode, int32_t* error,
                      kvs_stream_t stream);
/* Self-test of the bounded waits every kernel of this library uses on its mbarriers (no
 * reference counterpart): one warp waits, at most `limit` polls, on a barrier that nothing
 * arrives on (mode bit 1 = 0) or that one thread arrives on first (bit 1 = 1), with the
 * suspending wait (bit 0 = 0) or the fast one (bit 0 = 1).  out[0] = 1 if the wait gave up
 * (the kernels then record an error and wind down), 0 if it completed; out[1], out[2] = the
 * wait's SM cycles (low, high 32 bits).  A timeout leaves the context usable. */
int kvs_selftest_wait(int32_t mode, uint32_t limit, int32_t* out, kvs_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* KVS_B200_H */
