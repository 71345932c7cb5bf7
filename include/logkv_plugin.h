/*
 * C ABI of the operator-level plugin functions: the functions the reference's
 * fused-kernel modules export (litgpt/log_kv_updates_triton.py and the attach entry
 * of litgpt/log_kv_route_triton.py), so the reference's own Python orchestration
 * (LogStructuredKVCache with _fused_on) can run them on sm_100a.  Same conventions as
 * logkv_b200.h.  Arithmetic is the reference's CPU order (feature sums left to right,
 * no fused multiply-adds), so results equal the reference's CPU path.
 */
#ifndef LOGKV_PLUGIN_H
#define LOGKV_PLUGIN_H

#include "logkv_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The eight first-order ladder fields of a block of rows (indices 0, 1, 2, 8-12 of the
 * reference's 13-field tuples): k [rows, dk], v [rows, dv], the rest [rows]. */
typedef struct logkv_rows {
  void* k;
  void* v;
  float* w;
  int64_t* p_lo;
  int64_t* p_hi;
  int64_t* sum_wp;
  int64_t* order;
  uint8_t* pad;      /* bool */
  int32_t kv_dtype;  /* LOGKV_DTYPE_* of k and v */
} logkv_rows_t;

/* fill (log_kv_updates_triton.py:79): fields[dst[i]] = stage[src[i]] for i < n (K/V cast to the fields' dtype). */
LOGKV_API int logkv_fill(const logkv_rows_t* fields, const logkv_rows_t* stage, const int64_t* src,
                         const int64_t* dst, int64_t n, int32_t dk, int32_t dv, void* stream);

/*
 * merge_scatter (log_kv_updates_triton.py:176).  The pool is stored rows fields[si[i]]
 * (i < ns) followed by staged rows stage[gi[i - ns]], cast to the fields' dtype.
 * beta_mode 0: pool rows pi[2j], pi[2j+1] merge pairwise into out[j] (count-weighted
 * mean, p_lo/p_hi over positive-weight sides, sum_wp added, order min, pad and);
 * beta_mode 1/2: Beta groups of four (layout rows {start, width, dest}, npi / 2 output
 * rows), the cut selected and written to beta_cuts (1) or read from it (2).  Then pool
 * rows vi[j] are written to fields[dst[j]] and fields[clear[j]] are zeroed.  `out`
 * (float32 K/V) holds npi / 2 + nv rows; its first npi / 2 rows are the carry.
 */
LOGKV_API int logkv_merge_scatter(const logkv_rows_t* fields, const logkv_rows_t* stage, const int64_t* si,
                                  int64_t ns, const int64_t* gi, const int64_t* pi, int64_t npi, const int64_t* vi,
                                  int64_t nv, const int64_t* dst, const int64_t* clear, int64_t nclear,
                                  const logkv_rows_t* out, const int64_t* beta_layout, int64_t ngroups,
                                  uint8_t* beta_cuts, int32_t beta_mode, int32_t dk, int32_t dv, void* stream);

/*
 * centroid / centroid_parallel (log_kv_updates_triton.py:268-283): for runs
 * [start, start + count) of metadata [5, runs] (cluster, -, begin, length, forget as
 * float32 bits): acc = sum of k rows [begin, begin + length); pre = n_eff * forget;
 * mu = pre > 0 ? (pre * mu + acc) / (pre + length) : acc / length; n_eff = pre + length.
 * All runs read the old state; `scratch` holds count * (dim + 1) floats.
 */
LOGKV_API int logkv_centroid(const void* k, int32_t k_dtype, int32_t dim, float* mu, float* n_eff,
                             const int64_t* metadata, int64_t runs, int64_t start, int64_t count, float* scratch,
                             void* stream);

/* alpha_partition (log_kv_updates_triton.py:313): copy kept rows into the exact pool and archived rows out. */
typedef struct logkv_partition {
  const void* k;          /* [batch, groups, tokens, dk] */
  const void* v;          /* [batch, groups, tokens, dv] */
  const int64_t* pos;     /* [batch, tokens]             */
  const int64_t* indices; /* [batch, exact + archive], -1 = empty */
  void* exact_k;          /* [batch, groups, exact, dk]  */
  void* exact_v;
  int64_t* exact_pos;     /* [batch, exact]              */
  uint8_t* exact_valid;   /* [batch, exact] bool         */
  void* archive_k;        /* [batch, groups, archive, dk] */
  void* archive_v;
  int64_t* archive_pos;   /* [batch, archive]            */
  int32_t batch, groups, tokens, exact, archive, dk, dv, dtype;
} logkv_partition_t;
LOGKV_API int logkv_alpha_partition(const logkv_partition_t* args, void* stream);

/*
 * attach_assign (log_kv_route_triton.py:894): per (batch, group) lane and token slot
 * t < counts[b] (token offset order[b, t]): semantic_c = max((|x|^2 + |mu_c|^2) - 2 x.mu_c, 0),
 * cost_c = semantic_c + eta * gap / (gap + g0) with gap = max(pos - p_hi_c, 0) over live
 * clusters; the winner if its semantic <= lam * s_h, else the nearest live cluster by
 * exact squared difference.  out [batch, groups, tokens] int8 (slots past counts untouched).
 */
typedef struct logkv_attach {
  const void* x;              /* k_raw, element (b, g, t, d) at b*x_stride_b + g*x_stride_g + t*x_stride_t + d */
  int64_t x_stride_b, x_stride_g, x_stride_t;
  const int64_t* positions;   /* element (b, t) at b * pos_stride_b + t */
  int64_t pos_stride_b;
  const int64_t* order;       /* [batch, tokens] */
  const int64_t* counts;      /* [batch]         */
  const float* centroid;      /* [batch, groups, clusters, dim] */
  const uint8_t* alive;       /* [batch, groups, clusters] bool */
  const int64_t* p_hi;        /* [batch, groups, clusters] */
  const float* s_h;           /* [batch, groups] */
  int8_t* out;                /* [batch, groups, tokens] */
  int32_t batch, groups, tokens, clusters, dim, dtype;
  float eta, g0, lam;
} logkv_attach_t;
LOGKV_API int logkv_attach_assign(const logkv_attach_t* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LOGKV_PLUGIN_H */
