/*
 * C ABI of the unified (Ward / radius) route operators.
 *
 * Replace the plugin functions of litgpt/log_kv_route_triton.py used by the reference's unified
 * route (_semantic_unified_pair_matrix / _semantic_unified_reduce_incremental,
 * litgpt/log_kv_cache.py:3185-3376): pair_distances (:585-607), mirror (:546-553) and
 * UnifiedReduce (:610-838), with the results of the reference's Torch reducer
 * _UnifiedReduceTorch (log_kv_cache.py:448-638).  Plain device pointers, row-major, float32;
 * every call is enqueued on `stream` and neither allocates nor synchronizes.
 */
#ifndef LOGKV_UNIFIED_H
#define LOGKV_UNIFIED_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LOGKV_UNIFIED_API __attribute__((visibility("default")))
#else
#define LOGKV_UNIFIED_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LOGKV_UNIFIED_E_SHAPE (-1)
#define LOGKV_UNIFIED_E_POINTER (-4)

/* In place: gram [lanes, size, size] (upper triangle read) becomes max((n_i + n_j) - 2 G_ij, 0),
 * symmetric; norm [lanes, size]. */
LOGKV_UNIFIED_API int logkv_pair_distances(float* gram, const float* norm, int32_t lanes, int32_t size,
                                           void* stream);
/* In place: copy the upper triangle of dist [lanes, size, size] onto the lower one. */
LOGKV_UNIFIED_API int logkv_mirror(float* dist, int32_t lanes, int32_t size, void* stream);

/*
 * Incremental mutual-nearest Ward rounds over `lanes` independent sets of `size` clusters
 * (size <= 4096).  Caller-owned device state, updated in place:
 *   dist [lanes, size, size]  squared centre distances (symmetric)
 *   mu [lanes, size, dim]     centres
 *   mass [lanes, size]        masses (0 = no cluster)
 *   limits [lanes] or NULL    radius limits (the candidate pass) or none (the global pass)
 *   status [2, lanes] int32   row 0: lane still active after the last round; row 1: live
 *                             clusters (set row 1 to the lanes' counts before logkv_unified_init)
 *   alive [lanes, size] u8, radius [lanes, size] f32, packed [lanes, size] i64 (8-byte aligned)
 *   merges [lanes] i32, stuck [lanes] u8, trace [lanes, size, 2] i32 (merge pairs, in round
 *   then (cost, left) order)
 *   target                    clusters to keep per lane
 * logkv_unified_init derives alive from the counts and scans every row; each
 * logkv_unified_step runs one round.  Only single-pass rounds (passes = 1).
 */
typedef struct logkv_unified {
  float* dist;
  float* mu;
  float* mass;
  const float* limits;
  int32_t* status;
  uint8_t* alive;
  float* radius;
  int64_t* packed;
  int32_t* merges;
  uint8_t* stuck;
  int32_t* trace;
  int32_t lanes;
  int32_t size;
  int32_t dim;
  int32_t target;
} logkv_unified_t;

LOGKV_UNIFIED_API int logkv_unified_init(const logkv_unified_t* u, void* stream);
LOGKV_UNIFIED_API int logkv_unified_step(const logkv_unified_t* u, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LOGKV_UNIFIED_H */
