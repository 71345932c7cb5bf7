/*
 * C ABI of the B200-native SemanticLogKV flush-and-attend path.
 *
 * Plain pointers and sizes only.  Every device pointer is caller-owned CUDA
 * memory laid out exactly like the corresponding buffer of the reference's
 * LogStructuredKVCache (litgpt/log_kv_cache.py:907-1122): contiguous,
 * row-major, same shapes and dtypes.  All work is enqueued on the stream the
 * caller passes (a cudaStream_t as void*; NULL = legacy default stream); no
 * call allocates device memory, synchronizes, or reads device data back,
 * except the explicitly named *_read_status helper.  Scratch comes from a
 * caller-provided workspace sized by the matching *_workspace_bytes call.
 *
 * Return value: 0 on success, a negative LOGKV_E* code for invalid
 * arguments (nothing is launched then), or a CUDA error code > 0 when a
 * launch fails.
 */
#ifndef LOGKV_B200_H
#define LOGKV_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LOGKV_API __attribute__((visibility("default")))
#else
#define LOGKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LOGKV_OK 0
#define LOGKV_E_SHAPE (-1)      /* a size is out of the supported range      */
#define LOGKV_E_DTYPE (-2)      /* unsupported storage dtype code            */
#define LOGKV_E_WORKSPACE (-3)  /* workspace missing or too small            */
#define LOGKV_E_POINTER (-4)    /* a required pointer is NULL or misaligned  */
#define LOGKV_E_SMEM (-5)       /* the shape needs more shared memory        */
#define LOGKV_E_DEVICE (-6)     /* the state lives on another device than the current one */

#define LOGKV_DTYPE_F32 0
#define LOGKV_DTYPE_BF16 1

/* Routing of the archived tokens (logkv_layout_t.route). */
#define LOGKV_ROUTE_ATTACH 0    /* frozen-centre attach route (_alpha_route_flush :3984-3988)          */
#define LOGKV_ROUTE_UNIFIED 1   /* semantic_unified_route=True: _semantic_route_unified :3589-3688     */
#define LOGKV_UNIFIED_MAX_ROWS 4096  /* unified route: exact + flush tokens + clusters per lane, at most */

/* Static geometry of one layer's cache (LogStructuredKVCache.__init__, log_kv_cache.py:681-1133). */
typedef struct logkv_layout {
  int32_t batch;           /* B  : batch rows                                  */
  int32_t groups;          /* G  : KV groups (n_query_groups)                  */
  int32_t dim;             /* D  : head dim of K (pre-RoPE) and V              */
  int32_t clusters;        /* K  : cluster_k_max (<= 32)                       */
  int32_t levels;          /* L  : L_alloc                                     */
  int32_t slots;           /* B' : B_prime, slots per level                    */
  int32_t recent_capacity; /* 2 * recent_size                                  */
  int32_t exact;           /* P  : alpha_exact_tokens (> 0)                    */
  int32_t span_cap;        /* alpha_span_max_tokens                            */
  int32_t beta;            /* beta_novelty and beta_adaptive_merge (both on)   */
  int32_t dtype;           /* LOGKV_DTYPE_*: storage dtype of K/V buffers      */
  float eta;               /* seg_eta                                          */
  float g0;                /* seg_g0                                           */
  float lam;               /* cluster_lambda_rel                               */
  int32_t route;           /* LOGKV_ROUTE_*                                    */
  int32_t merge_passes;    /* semantic_merge_passes (>= 1; unified route)      */
} logkv_layout_t;

/*
 * Device state of one layer.  The first block are the reference's
 * named_buffers (log_kv_cache.py:907-1122); the alpha_span_* block is the
 * device form of the host lists _alpha_spans / _alpha_positions / alpha_count
 * (log_kv_cache.py:925-941), which this implementation keeps on the device so
 * a flush never waits for the host.
 */
typedef struct logkv_state {
  void* level_k;            /* [B,G,K,L,B',D] dtype */
  void* level_v;            /* [B,G,K,L,B',D] dtype */
  float* level_w;           /* [B,G,K,L,B']         */
  int64_t* level_p_lo;      /* [B,G,K,L,B']         */
  int64_t* level_p_hi;
  int64_t* level_sum_wp;
  int64_t* level_order;
  uint8_t* pad_mask;        /* bool                 */
  int16_t* level_count;     /* [B,G,K,L]            */
  float* centroid;          /* [B,G,K,D]            */
  float* n_eff;             /* [B,G,K]              */
  int32_t* n_total;         /* [B,G,K]              */
  int64_t* p_hi_c;          /* [B,G,K]              */
  int32_t* level0_phase;    /* [B,G,K]              */
  uint8_t* alive;           /* [B,G,K] bool         */
  float* s_h;               /* [B,G]                */
  void* recent_k;           /* [B,G,2R,D] dtype (post-RoPE)  */
  void* recent_k_raw;       /* [B,G,2R,D] dtype (pre-RoPE)   */
  void* recent_v;           /* [B,G,2R,D] dtype              */
  int64_t* recent_pos;      /* [B,2R]                        */
  uint8_t* recent_ends;     /* [B,2R] span-end flags (host list _recent_span_ends) */
  void* alpha_k_raw;        /* [B,G,P,D] dtype      */
  void* alpha_v;            /* [B,G,P,D] dtype      */
  int64_t* alpha_pos;       /* [B,P]                */
  uint8_t* alpha_valid;     /* [B,P] bool           */
  int32_t* alpha_span_len;  /* [B,P] lengths of the pool's spans, pool order */
  uint8_t* alpha_span_closed; /* [B,P]              */
  int32_t* alpha_nspans;    /* [B]                  */
  int32_t* alpha_rowcount;  /* [B] kept tokens per row                       */
  int32_t* alpha_count;     /* [1] max over rows (the reference's alpha_count) */
} logkv_state_t;

/*
 * Near-tie log (no reference counterpart).  Every decision of a flush whose two best candidates,
 * or whose value and threshold, lie within a relative gap |a - b| / max(|a|, |b|) < 1e-6 is
 * recorded in the workspace, so that a decision which a different floating-point summation
 * order could flip is logged, not waived silently.  Kinds and their fields:
 *   ATTACH_COST   frozen-centroid routing cost argmin (log_kv_cache.py:2649-2681): index = token
 *                 position, first / second = best / runner-up cluster, value = best cost;
 *   DIRECT        winner's semantic distance against lambda * s_h (:4597-4634): first = 1 if the
 *                 token joined directly, second = winner cluster, value = the distance;
 *   NEAREST       an orphan's exact-distance nearest live cluster (:4671-4677): clusters;
 *   SEED_PICK     farthest-point seed argmax (:4650-4668): index = pick number, first / second =
 *                 token positions of the best and runner-up;
 *   SEED_NEAREST  an orphan's nearest live-or-seeded cluster after seeding: clusters;
 *   BETA_CUT      Beta 4->2 cut costs (beta_log_kv.py:29-46) of groups decided in canonical
 *                 order: cluster = c, index = level * 65536 + group, first / second = cuts;
 *   ALPHA_ORDER   two span candidates of one batch row with near-equal densities
 *                 (alpha_log_kv.py:177-226 sorts by density): first / second = candidates;
 *   ALPHA_SWAP    the greedy's replacement test density * length > evicted loss: first =
 *                 candidate, second = 1 if the span was taken;
 *   WARD_MIN      unified route: a row's minimum Ward cost and the next cost of that row
 *                 (_UnifiedReduceTorch._scan, log_kv_cache.py:480-494, found by a full scan of the
 *                 row): cluster = pass (0 candidate, 1 global), index = row, first / second =
 *                 columns, value = the minimum cost;
 *   WARD_BUDGET   unified route: the last pair the round's budget takes and the first it leaves
 *                 (the stable cost order, :525-527): cluster = pass, first / second = their rows.
 * `flush` = flushes of this workspace before the logging one (0-based).
 */
#define LOGKV_TIE_ATTACH_COST 1
#define LOGKV_TIE_DIRECT 2
#define LOGKV_TIE_NEAREST 3
#define LOGKV_TIE_SEED_PICK 4
#define LOGKV_TIE_SEED_NEAREST 5
#define LOGKV_TIE_BETA_CUT 6
#define LOGKV_TIE_ALPHA_ORDER 7
#define LOGKV_TIE_ALPHA_SWAP 8
#define LOGKV_TIE_WARD_MIN 9
#define LOGKV_TIE_WARD_BUDGET 10
typedef struct logkv_tie {
  int32_t kind, flush, batch, group, cluster, index, first, second;
  float gap;    /* relative gap of the two values */
  float value;  /* the winning (or tested) value */
} logkv_tie_t;

/* Bytes of scratch one logkv_flush call needs for this layout and flush size. */
LOGKV_API size_t logkv_flush_workspace_bytes(const logkv_layout_t* layout, int32_t flush_tokens);

/*
 * One flush of the `flush_tokens` oldest window tokens of every batch row, then
 * the window shift.  Replaces LogStructuredKVCache._route_and_flush_batch for
 * the Alpha + attach route (log_kv_cache.py:5033-5128 -> _alpha_route_flush
 * :3903-4003) followed by the window shift of _semantic_flush_tokens
 * (:5640-5661): Alpha span cut/score/greedy choice and pool rewrite, attach
 * decisions with farthest-point seeding, new clusters, ordinary and delayed
 * joins, the per-cluster ladder append with pairwise or Beta merges, and the
 * ordered centroid update.  `recent_count` is the window fill before the flush.
 */
LOGKV_API int logkv_flush(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                          int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream);

/*
 * logkv_flush without a workspace argument, for callers that may not allocate
 * device memory themselves: serving hosts that carve all GPU memory into fixed
 * arenas at start-up and lock their allocator afterwards, and language bindings
 * that cannot pass a device buffer of their own across this C boundary.  (No
 * counterpart in the reference, which allocates freely through PyTorch.)
 *
 * The scratch is one region of 32 MiB compiled into the library: every GPU that
 * loads the library holds it until the process exits.  Layouts whose
 * logkv_flush_workspace_bytes exceeds 32 MiB are rejected with LOGKV_E_WORKSPACE
 * and nothing is launched.  The call itself allocates nothing (no cudaMalloc,
 * no allocating library call); it clears the region's status word and row
 * counters with cudaMemsetAsync before the flush.  The state must live on the
 * current device (else LOGKV_E_DEVICE, nothing launched).  The first call in
 * each CUDA context looks the region's device address up (with that device
 * current) and caches it for that context; make that first call before any
 * stream capture.  After a device reset the next call looks it up again.  All
 * calls share the one region, which keeps the last call's contents: two calls
 * whose work overlaps on the GPU (different streams, or different threads on
 * one device) race on it, so serialize them.  The flush's status word and row
 * counters stay readable in the region until the next static flush clears
 * them: logkv_read_status / logkv_read_counters with workspace = NULL read
 * them (current device).
 */
LOGKV_API int logkv_flush_static(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                 int32_t recent_count, void* stream);

/*
 * Append a chunk of n tokens to the recent window at rows [recent_count, recent_count + n): the
 * window write of LogStructuredKVCache._semantic_add_recent (log_kv_cache.py:5701-5704, and the
 * span-end flags of :5693).  k (post-RoPE), k_raw (pre-RoPE) and v are [B, G, n, D] in the cache's
 * storage dtype with the given element strides of their batch, group and token axes (the head dim
 * contiguous, every row 16-byte aligned); positions [B, n] int64 with strides, or NULL for the
 * consecutive positions pos0, pos0 + 1, ... of every row; ends [B, n] uint8 contiguous on the
 * device.  One kernel on `stream`; returns LOGKV_E_POINTER for misaligned rows.
 */
LOGKV_API int logkv_window_append(const logkv_layout_t* layout, const logkv_state_t* state, const void* k,
                                  const int64_t* k_strides, const void* k_raw, const int64_t* k_raw_strides,
                                  const void* v, const int64_t* v_strides, const int64_t* positions,
                                  const int64_t* pos_strides, int64_t pos0, const uint8_t* ends, int32_t n,
                                  int32_t recent_count, void* stream);

/* A chunk of n window rows as logkv_window_append takes them (same meaning and rules). */
typedef struct logkv_chunk {
  const void* k;
  int64_t k_strides[3];
  const void* k_raw;
  int64_t k_raw_strides[3];
  const void* v;
  int64_t v_strides[3];
  const int64_t* positions;   /* [B, n] int64, or NULL: pos0, pos0 + 1, ... */
  int64_t pos_strides[2];
  int64_t pos0;
  const uint8_t* ends;        /* [B, n] uint8, contiguous */
  int32_t n;
} logkv_chunk_t;

/*
 * _semantic_add_recent of a chunk whose append overflows the window by exactly one flush of
 * the flush_tokens oldest rows (log_kv_cache.py:5668-5718 with one pass of the flush loop),
 * when those rows are all rows already in the window: recent_count (the fill before the
 * chunk) in [flush_tokens, 2 * flush_tokens], recent_count + chunk->n <= recent_capacity.
 * The flush runs on the window as it is, and its final kernel writes the kept old rows and
 * the chunk's rows once, straight to their places after the shift (no separate append, no
 * second copy of the chunk).  The state afterwards is the state that
 * logkv_window_append(chunk, recent_count) followed by logkv_flush(flush_tokens,
 * recent_count + n) leaves; the workspace is logkv_flush's.  Other cases: LOGKV_E_SHAPE,
 * nothing launched.  logkv_flush_chunk_profiled adds logkv_flush_profiled's events (its last
 * stage is this window write).
 */
LOGKV_API int logkv_flush_chunk(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                int32_t recent_count, const logkv_chunk_t* chunk, void* workspace,
                                size_t workspace_bytes, void* stream);
LOGKV_API int logkv_flush_chunk_profiled(const logkv_layout_t* layout, const logkv_state_t* state,
                                         int32_t flush_tokens, int32_t recent_count, const logkv_chunk_t* chunk,
                                         void* workspace, size_t workspace_bytes, void* stream, void** events,
                                         int32_t n_events);

/*
 * KV-head sharding of one sequence (no reference counterpart: the reference runs a
 * layer's cache on one device).  Each rank's layout and state hold its own block of
 * `groups` KV groups (rank r: global groups [r * groups, (r + 1) * groups)).  Every
 * group is independent during a flush except the Alpha span score, which is the mean
 * over all groups of per-group parts (Beta: the mean of the top two groups)
 * (litgpt/alpha_log_kv.py:154-156, :173).  So a sharded flush is two calls around one
 * exchange:
 *   logkv_flush_scores  snapshot, span cut and this rank's per-group span parts;
 *   (caller)            all-gather the parts, [batch, candidates, groups, 2] float32 at
 *                       the address logkv_flush_partials gives, over the ranks in rank
 *                       order into one [ranks, batch, candidates, groups, 2] device buffer;
 *   logkv_flush_commit  the rest of the flush, reading the gathered parts in global group
 *                       order, so every rank makes the unsharded flush's span choice.
 * With ranks == 1 and partials_all == NULL the pair equals logkv_flush.
 */
LOGKV_API int logkv_flush_scores(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                 int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream);
LOGKV_API int logkv_flush_commit(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                 int32_t recent_count, void* workspace, size_t workspace_bytes,
                                 const float* partials_all, int32_t ranks, void* stream);
/*
 * logkv_flush_commit with rank r's parts at partials_all + r * rank_stride floats (rank_stride at
 * least the rank's part count): the layout of one all-gather of many layers' parts at once, where
 * each rank sends its layers' parts back to back.
 */
LOGKV_API int logkv_flush_commit_strided(const logkv_layout_t* layout, const logkv_state_t* state,
                                         int32_t flush_tokens, int32_t recent_count, void* workspace,
                                         size_t workspace_bytes, const float* partials_all, int32_t ranks,
                                         int64_t rank_stride, void* stream);
/*
 * Route overlap (replaces the side-stream route decisions of LOGKV_ROUTE_OVERLAP,
 * litgpt/log_kv_cache.py:3814-3849).  A flush's decisions (snapshot, span cut, span scores,
 * attach decisions, span choice, seeding, per-cluster plan) read only the flushed window rows,
 * the exact pool and the cluster state that the previous flush committed, and write only the
 * workspace; so they need not wait for readers of the cache (attention) queued since the
 * previous flush.  logkv_flush_decide enqueues them (on a side stream that waits for the end of
 * the previous flush); logkv_flush_apply enqueues the rest (ladder, pool rewrite, window shift)
 * on the caller's stream after the decisions.  The pair equals logkv_flush.  Valid when every
 * flushed row was in the window when the previous flush ended, and when nothing between the
 * two writes the rows or state the decisions read.
 */
LOGKV_API int logkv_flush_decide(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                 int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream);
LOGKV_API int logkv_flush_apply(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream);

/* Host-side address arithmetic only: where this workspace keeps the rank's span parts, and their float count. */
LOGKV_API int logkv_flush_partials(const logkv_layout_t* layout, int32_t flush_tokens, void* workspace,
                                   float** partials, size_t* count);

/*
 * Update tape (replaces the record / replay branches of route_and_flush_batch,
 * litgpt/log_kv_cache.py:4946-5031, with the _SemanticReplayUpdates store :111-137).
 * logkv_flush_record is logkv_flush that also writes, into a caller-owned device buffer of
 * logkv_tape_bytes (16-byte aligned): the flushed window rows (pre-RoPE K, V) as the flush
 * saw them, the kept / archived token lists, the new span table, the per-cluster plan and
 * every Beta cut of the cascade.  logkv_flush_replay applies such a record to a cache in the
 * state the recorded flush started from: the recorded rows replace the window's flushed rows,
 * nothing is routed, scored or chosen, and the cache ends exactly as the recorded flush left
 * it (buffers bit for bit).  The order of replays is the caller's to keep (the Python cache
 * checks it).  A KV-head-sharded rank records with logkv_flush_commit_record, the commit half of
 * its flush (logkv_flush_commit_strided's arguments; rank_stride 0 = the parts' own count) that
 * also writes its record; logkv_flush_replay of that record needs no exchange, since the record
 * holds the span choice the ranks made together.
 */
/*
 * Route op-log (replaces the op-log rows of _record_ops, litgpt/log_kv_cache.py:2043-2071,
 * recorded by the attach route and the joins).  After a flush (any of the entry points above,
 * same workspace, before the next flush), append that flush's rows to a caller-owned log
 * op_log [batch, groups, capacity, 4] int32 (16-byte aligned) with lengths op_log_len
 * [batch, groups] int32: per lane, NEW_CLUSTER (0, cluster, 0, position) for every cluster it
 * opened, in cluster order; then JOIN (2, cluster, 0, position) for the joined tokens of every
 * ordinary or new cluster, cluster by cluster, positions ascending; then JOIN rows for the new
 * tokens of delayed clusters.  A lane whose rows do not fit gets no rows and its length becomes
 * capacity + 1 (and stays there): the caller reports the overflow.
 */
LOGKV_API int logkv_flush_oplog_append(const logkv_layout_t* layout, int32_t flush_tokens, void* workspace,
                                       int32_t* op_log, int32_t* op_log_len, int32_t capacity, void* stream);

LOGKV_API size_t logkv_tape_bytes(const logkv_layout_t* layout, int32_t flush_tokens);
LOGKV_API int logkv_flush_record(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                 int32_t recent_count, void* workspace, size_t workspace_bytes, void* tape,
                                 size_t tape_bytes, void* stream);
LOGKV_API int logkv_flush_commit_record(const logkv_layout_t* layout, const logkv_state_t* state,
                                        int32_t flush_tokens, int32_t recent_count, void* workspace,
                                        size_t workspace_bytes, const float* partials_all, int32_t ranks,
                                        int64_t rank_stride, void* tape, size_t tape_bytes, void* stream);
LOGKV_API int logkv_flush_replay(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                 int32_t recent_count, void* workspace, size_t workspace_bytes, const void* tape,
                                 size_t tape_bytes, void* stream);

/*
 * Host-side helper for route overlap under CUDA-graph capture (no reference counterpart): *id = the
 * id of the capture `stream` takes part in, or 0 when it is not capturing.  A flush's decisions fork
 * to a side stream only after an event recorded in the same capture (or outside any capture).
 */
LOGKV_API int logkv_stream_capture_id(void* stream, unsigned long long* id);

/*
 * Copy the workspace status word to *out (synchronizes `stream`); nonzero = a capacity was
 * exceeded.  workspace = NULL reads the status of the last logkv_flush_static on the current
 * device.
 */
LOGKV_API int logkv_read_status(const void* workspace, int32_t* out, void* stream);

/*
 * Measurement helpers (no reference counterpart; the reference times stages
 * with host counters and optional CUDA events, litgpt/log_kv_timing.py:15-50).
 * logkv_flush_profiled is logkv_flush plus one cudaEventRecord (events are
 * cudaEvent_t as void*) before the first and after each of the
 * LOGKV_FLUSH_STAGES kernel stages: snapshot, span cut, span scores with attach
 * decisions, choose, seed + plan, prepare, cascade (merge and move kernels), pool
 * rewrite, window shift (logkv_flush_chunk: the window write of the kept rows and the
 * chunk).  (Events between the kernels end their programmatic
 * overlap, so a profiled flush is slower than a plain one.)
 */
#define LOGKV_FLUSH_STAGES 9
LOGKV_API int logkv_flush_profiled(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                   int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream,
                                   void** events, int32_t n_events);

/*
 * Copy up to n of the workspace's row counters (accumulated over every flush
 * since the workspace was zeroed) to out, synchronizing `stream`: [0] stored
 * level rows read, [1] incoming rows read, [2] survivor rows written, [3] rows
 * appended, [4] rows zeroed, [5] merged rows carried up, [6] rows gathered for
 * delayed re-inserts, [7] flushes, [8] Beta groups whose cut was a near tie and
 * was decided by the canonical sequential evaluation, [9] near-tie log entries,
 * [10] lanes whose ladder cascade took the sequential level walk.  The workspace must be
 * zero-filled once when it is allocated.  workspace = NULL reads the counters of
 * the last logkv_flush_static on the current device.
 */
LOGKV_API int logkv_read_counters(const void* workspace, uint64_t* out, int32_t n, void* stream);

/*
 * Unified route only: copy the per-(batch, group) lane words of the last flush made with this
 * workspace (16 int32 per lane, lane-major; up to n words) and synchronize `stream`.  Word 0..3:
 * candidate pass live count, active flag, merges, rounds; 4..7 the same for the global pass;
 * 8 global rows (live clusters + candidates), 9 live clusters before the flush, 10 candidates,
 * 11/12 exact-difference pair matrices in the candidate / global pass, 13 Ward merges.  No
 * reference counterpart: these are the host-side values the reference's route keeps in Python
 * (_semantic_route_unified, log_kv_cache.py:3589-3688), read here for diagnostics and tests.
 */
LOGKV_API int logkv_read_unified(const logkv_layout_t* layout, int32_t flush_tokens, const void* workspace,
                                 int32_t* out, int32_t n, void* stream);

/*
 * Copy the near-tie log to out (up to cap entries, in logging order) and the number of entries
 * requested since the log was last cleared to *total (entries beyond the log's 4096-entry
 * capacity are counted but not kept); with clear != 0 the log is emptied after the copy.
 * Synchronizes `stream`.  workspace = NULL reads the log of logkv_flush_static (current device).
 */
LOGKV_API int logkv_read_ties(void* workspace, logkv_tie_t* out, int32_t cap, int64_t* total, int32_t clear,
                              void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LOGKV_B200_H */
