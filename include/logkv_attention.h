/*
 * C ABI of the read side of the SemanticLogKV cache: mid-anchor attention plan,
 * packing and slot attention over [merged slots | exact pool | recent window |
 * current tokens].  Same conventions as logkv_b200.h: caller-owned device
 * memory in the reference's layouts, work enqueued on the caller's stream, no
 * allocation, no host synchronization, 0 / negative LOGKV_E_* / CUDA error.
 */
#ifndef LOGKV_ATTENTION_H
#define LOGKV_ATTENTION_H

#include "logkv_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Attention plan of one layer.  cap = clusters * levels * slots.  The first block
 * is the reference's plan (LogStructuredKVCache._semantic_mid_attention_plan,
 * litgpt/log_kv_cache.py:5979-6007): per (b, g) lane the occupied ladder entries,
 * cluster-major with the top level first, their mid anchors
 * floor((2 sum_wp + ww) / (2 ww)), ww = max(trunc(w), 1), and valid = w > 0.
 * Entries past a lane's width are 0 / 0 / false, which is what the reference's
 * [B, G, width_max] tensors hold there.  The second block is the same plan with
 * the invalid entries dropped, and the valid exact-pool rows per batch row.
 */
typedef struct logkv_plan {
  int64_t* idx;        /* [B,G,cap] physical entry (c * L + level) * B' + slot     */
  int64_t* anchor;     /* [B,G,cap]                                               */
  uint8_t* valid;      /* [B,G,cap]                                               */
  int32_t* width;      /* [B,G] occupied entries per lane                         */
  int32_t* width_max;  /* [1]                                                     */
  int32_t* vslot;      /* [B,G,cap] physical entries of valid slots, plan order    */
  int64_t* vanchor;    /* [B,G,cap] their anchors                                 */
  int32_t* nvalid;     /* [B,G]                                                   */
  int32_t* exact_rows; /* [B,P] valid rows among the first alpha_count pool rows  */
  int32_t* nexact;     /* [B]                                                     */
} logkv_plan_t;

/* LitGPT RoPE tables (cos_cache / sin_cache of the cache, litgpt/log_kv_position.py:74-101). */
typedef struct logkv_rope {
  const void* cos;  /* [rows, rope_n] */
  const void* sin;  /* [rows, rope_n] */
  int32_t rows;     /* positions in the tables; a larger anchor sets status bit 16 and is clamped */
  int32_t rope_n;   /* rotated leading features: even, <= dim (0 = no rotation) */
  int32_t dtype;    /* LOGKV_DTYPE_F32 or LOGKV_DTYPE_BF16 */
} logkv_rope_t;

/*
 * Packed frozen prefix for attention, rebuilt once per flush: per lane the valid
 * merged slots (plan order, keys rotated at their mid anchors) followed by the
 * valid exact-pool rows (keys rotated at alpha_pos), values as stored, and the
 * mass term log(max(w, 1)) rounded to the storage dtype (0 for exact rows).
 */
typedef struct logkv_prefix {
  void* k;           /* [B,G,capacity,D] storage dtype */
  void* v;           /* [B,G,capacity,D]               */
  float* mass;       /* [B,G,capacity]                 */
  int32_t* length;   /* [B,G]                          */
  int32_t capacity;  /* >= clusters * levels * slots + exact */
} logkv_prefix_t;

/* Plan of the current ladder state (reads level_count, level_w, level_sum_wp, alpha_valid, alpha_count). */
LOGKV_API int logkv_attention_plan(const logkv_layout_t* layout, const logkv_state_t* state,
                                   const logkv_plan_t* plan, void* stream);

/*
 * Pack the frozen prefix from a plan.  Replaces the pooled and exact parts of
 * the reference's packer (_pack_torch, litgpt/log_kv_pack.py:27-72) and the
 * reference's decode workspace reuse (_mid_chunk_attention, log_kv_cache.py:6770-6799).
 * `status` (device int32, may be NULL) gets bit 16 when an anchor is outside the tables.
 */
LOGKV_API int logkv_pack_prefix(const logkv_layout_t* layout, const logkv_state_t* state,
                                const logkv_plan_t* plan, const logkv_rope_t* rope,
                                const logkv_prefix_t* prefix, int32_t* status, void* stream);

/*
 * The reference's packed K/V for SDPA ([B,G,length,dim], dim >= D + 1), bit for bit
 * (log_kv_pack.pack_mid_kv with the torch backend, litgpt/log_kv_pack.py:27-72 and
 * :114-131): length = width + alpha_count + recent_count + tokens; K column D holds
 * log(max(w,1)) / 0 / -10000 in the storage dtype.  `width` and `alpha_count` are the
 * host values the output was sized with.  skip_pooled != 0 leaves the first
 * width + alpha_count rows untouched; rows before width + alpha_count + recent_start
 * are left untouched likewise (the reference's decode-buffer reuse).  k_new/v_new
 * are contiguous [B,G,tokens,D].
 */
LOGKV_API int logkv_pack_mid(const logkv_layout_t* layout, const logkv_state_t* state, const logkv_plan_t* plan,
                             const logkv_rope_t* rope, int32_t width, int32_t alpha_count, int32_t recent_count,
                             const void* k_new, const void* v_new, int32_t tokens, void* out_k, void* out_v,
                             int32_t dim, int32_t skip_pooled, int32_t recent_start, int32_t* status, void* stream);

/*
 * Slot attention over [prefix | recent window | the call's `tokens` new tokens]
 * for the query tokens [q_offset, q_offset + q_tokens) of the call:
 *   out = softmax(scale * (q . k_s + qx * mass_s)) v_s,
 * with causal != 0 new token j visible to query token t iff j <= t (the reference's
 * lower-right causal tail), else every new token visible; every other slot visible.
 * Replaces log_kv_chunk_attention (litgpt/log_kv_cache.py:6802-6864 ->
 * _mid_chunk_attention :6770-6799 -> Flash SDPA over the packed inputs of
 * _slot_sdpa_inputs :6439-6464).  qx is the query's mass coordinate, 1/scale
 * rounded to the storage dtype.
 *
 * Kernels: bf16 caches use tensor cores, a split-K decode kernel for up to 16 query
 * rows per lane (heads / groups * q_tokens in {1, 2, 4, 8, 16}) and a chunk kernel for
 * more (heads / groups a power of two <= 8, head dim <= 128); float32 caches use
 * CUDA cores for 1, 2, 4 or 8 query rows per lane (longer chunks take several calls).
 */
typedef struct logkv_attention_args {
  const void* q;        /* [B,H,q_stride,D] storage dtype, post-RoPE */
  const void* k_new;    /* [B,G,tokens,D] post-RoPE                */
  const void* v_new;    /* [B,G,tokens,D]                          */
  void* out;            /* [B,H,q_stride,D] storage dtype; rows [q_offset, q_offset + q_tokens) written */
  int32_t heads;        /* H, a multiple of groups                 */
  int32_t tokens;       /* new tokens (>= 1)                       */
  int32_t q_offset;     /* first query token of this call          */
  int32_t q_tokens;     /* query tokens of this call               */
  int32_t recent_count; /* window rows [0, recent_count) are attended */
  int32_t causal;       /* 1: causal tail over the new tokens, 0: none */
  float scale;
  float qx;
  int32_t q_stride;     /* query / output rows per head: 0 = tokens; fewer (causal 0 only) when the queries
                           are the first of the new tokens, e.g. a decode step whose single query sees a
                           pending token and itself (litgpt/model.py:1219-1226, causal_tail=0) */
} logkv_attention_args_t;

/* Scratch bytes of logkv_attention (zero-fill it once when allocated; calls leave it reusable). */
LOGKV_API size_t logkv_attention_workspace_bytes(const logkv_layout_t* layout, int32_t heads, int32_t q_tokens,
                                                 int32_t prefix_capacity);

LOGKV_API int logkv_attention(const logkv_layout_t* layout, const logkv_state_t* state,
                              const logkv_prefix_t* prefix, const logkv_attention_args_t* args,
                              void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LOGKV_ATTENTION_H */
