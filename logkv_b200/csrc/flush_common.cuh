// Geometry and workspace views shared by the flush kernels.
#pragma once

#include "common.cuh"

namespace logkv {

struct LevelPlan;

// Per-call constants (by value into every kernel).
struct Geo {
  int B, G, D, K, L, Bs;  // batch, KV groups, head dim, clusters, levels, slots per level
  int cap2R;              // recent capacity (2 * recent_size)
  int P;                  // exact pool capacity
  int span_cap;           // alpha_span_max_tokens
  int beta;               // Beta novelty + 4->2 merge
  int F;                  // tokens flushed now
  int NW;                 // token index space per batch row: P + F
  int NC;                 // candidate capacity per row: P + F
  int recent_count;       // window fill before the flush
  int S;                  // ladder scratch rows per buffer per (b, g): NW + K*L*B' + K*(L+2)
  int sort_cap;           // power of two >= L * Bs + NW (delayed re-insert sort)
  int seed_staged;        // seeding CTAs keep their token rows in shared memory (set per dtype at launch)
  int shard_ranks;        // KV-head sharding: ranks holding G groups each (1 = unsharded)
  long long gpart_stride; // KV-head sharding: floats between two ranks' span parts in gpart_all
  int tape;               // update tape: kTapeNone, kTapeRecord (save Beta cuts), kTapeReplay (use them)
  int route;              // LOGKV_ROUTE_ATTACH or LOGKV_ROUTE_UNIFIED
  int passes;             // unified route: semantic_merge_passes of the global pass
  int Mg;                 // unified route: rows per lane of its matrices (NW + K)
  float eta, g0, lam;
};

// Unified-route workspace (flush_unified.cuh), per (batch, group) lane; null for the attach route.
constexpr int kULaneWords = 16;
enum ULaneWord : int {
  kUCountC = 0, kUActiveC = 1, kUMergesC = 2, kURoundsC = 3,   // candidate pass: live count, active, merges, rounds
  kUCountG = 4, kUActiveG = 5, kUMergesG = 6, kURoundsG = 7,   // global pass
  kUGCount = 8, kUOld = 9, kUCand = 10,         // global rows, old clusters, candidates
  kUCdistC = 11, kUCdistG = 12,                 // the pass takes the exact-difference form (tile size <= 32)
  kUWard = 13,                                  // Ward merges of old clusters
};
struct UWork {
  float* dist;          // [B*G, Mg, Mg] squared centre distances
  float* mu_c;          // [B*G, NW, D] candidate pass centres (archived tokens, then candidates)
  float* mu_g;          // [B*G, Mg, D] global pass centres (live centroids, then candidates)
  float* mass;          // [B*G, Mg]
  float* radius;        // [B*G, Mg]
  uint8_t* alive;       // [B*G, Mg]
  uint8_t* stuck;       // [B*G, 2]
  long long* packed;    // [B*G, Mg]
  long long* restr;     // [B*G, Mg] frozen-centre sweep scratch
  int32_t* trace_c;     // [B*G, NW, 2]
  int32_t* trace_g;     // [B*G, Mg, 2]
  int32_t* label;       // [B*G, NW] candidate (compact) of every archived token
  int32_t* words;       // [B*G, kULaneWords]
  float* limit;         // [B*G] candidate pass radius limit
  int32_t* old;         // [B*G, K] live clusters before the flush, ascending
  int32_t* ward;        // [B*G, K, 2] Ward merges (keep, free) in trace order
};

// 16-byte asynchronous global -> shared copies (both addresses 16-byte aligned).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// TMA bulk copies (cp.async.bulk into this CTA's own shared memory) completing on an mbarrier.  Both
// addresses 16-byte aligned, sizes multiples of 16 bytes.
__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
               ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned done;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(done) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return done != 0;
}
// Bounded wait for phase `parity` of an mbarrier: false once kMbarWaitNs of device time (the
// global nanosecond timer) have passed without the phase completing.
constexpr unsigned long long kMbarWaitNs = 2000000000ull;
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kMbarWaitNs) return false;
  return true;
}
__device__ __forceinline__ void bulk_store(void* gdst, const void* smem_src, unsigned bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n"
               ::"l"(gdst), "r"(smem_u32(smem_src)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

enum TapeMode : int { kTapeNone = 0, kTapeRecord = 1, kTapeReplay = 2 };

enum JobType : int32_t { kJobNone = 0, kJobOrdinary = 1, kJobNew = 2, kJobLate = 3 };

// Traffic counters (rows) accumulated across flushes in the workspace.
enum Counter : int {
  kCntStorageRead = 0,   // stored level rows loaded for an overflowing level
  kCntStageRead = 1,     // incoming rows read (tokens, carries, staged re-inserts)
  kCntSurvivor = 2,      // survivor rows written
  kCntFill = 3,          // rows appended without overflow
  kCntClear = 4,         // rows zeroed (level tails, cleared clusters)
  kCntCarry = 5,         // merged rows written for the next level
  kCntGather = 6,        // rows gathered for delayed re-inserts
  kCntFlushes = 7,       // flush calls
  kCntExactCuts = 8,     // Beta groups whose cut needed the canonical-order evaluation (near ties)
  kCntTies = 9,          // near-tie log entries requested (entries beyond kTieCap are counted only)
  kCntSeqLanes = 10,     // lanes whose cascade took the sequential walk in the parallel cascade
  kNumCounters = 11,
};

// Near-tie log: every decision of a flush whose two best candidates (or whose value and
// threshold) lie within a relative gap of kTieRel is recorded, so a caller can see where a
// different summation order (the reference's vectorised CPU sums) could have decided the other
// way.  Entries live in the workspace right after the counters (byte offset kTieOffset), in the
// order the kernels reach them; the count is counters[kCntTies].  Layout = logkv_tie_t.
constexpr float kTieRel = 1e-6f;
constexpr int kTieCap = 4096;
constexpr size_t kTieOffset = 512;
struct TieEntry {
  int32_t kind, flush, b, g, c, index, first, second;
  float gap, value;
};
static_assert(sizeof(TieEntry) == sizeof(logkv_tie_t), "tie entry layout");

// Views into the caller's workspace (carved by the host in flush.cu).
struct Work {
  int32_t* status;
  unsigned long long* counters;  // [kNumCounters]
  TieEntry* ties;                // [kTieCap] near-tie log (workspace byte kTieOffset)
  void* snap_k;            // [B,G,P,D] T  old pool snapshot
  void* snap_v;
  int64_t* snap_pos;       // [B,P]
  int32_t* snap_rowcount;  // [B]
  int32_t* cand_s0;        // [B,NC] first token range (start, count) of a candidate
  int32_t* cand_n0;
  int32_t* cand_s1;        // second range (old unfinished span continued by new tokens)
  int32_t* cand_n1;
  uint8_t* cand_flags;     // bit0 old, bit1 closed
  int32_t* n_cand;         // [B]
  float* scores;           // [B,NC]
  float* gpart;            // [B,NC,G,2] per-group parts (Alpha: R_K, R_V; Beta: group score)
  const float* gpart_all;  // sharded: [ranks,B,NC,G,2] every rank's gpart in rank order, else null
  int32_t* keep_idx;       // [B,P]  token indices kept in the pool, candidate order
  int32_t* nkeep;          // [B]
  int32_t* arch_idx;       // [B,NW] archived token indices, position order
  int32_t* narch;          // [B]
  int32_t* span_len;       // [B,P] the pool's new span table, written by the choice, committed by K7
  uint8_t* span_closed;    // [B,P]
  int32_t* nspans;         // [B]
  int8_t* assign;          // [B,G,NW] cluster per archived token (archive rank order)
  int8_t* assign_tok;      // [B,G,NW] attach decision per token (token index order)
  uint8_t* orphan;         // [B,G,NW] token index order
  float* s_winner;         // [B,G,NW] token index order
  float* cnorm;            // [B,G,K] sum_d mu_d^2 of every centre (left to right), before the flush
  uint8_t* tape_cuts;      // update tape's Beta cuts [B,G,K,L,cut stride] (record / replay), else null
  long long tape_cut_lane; // >= 0: the cut slot a sequential walk uses instead of its lane (Ward merges)
  int64_t* tok_pos;        // [B,NW] position of every token of the flush's index space (written by K0)
  int32_t* tok_list;       // [B,G,NW] archive ranks grouped by cluster (stable)
  int32_t* plan_off;       // [B,G,K] offset into tok_list
  int32_t* plan_n;         // [B,G,K] tokens joining the cluster
  int32_t* plan_type;      // [B,G,K] JobType
  int32_t* plan_m0;        // [B,G,K] level-0 stage rows
  int32_t* plan_scr;       // [B,G,K] first scratch row of the cluster in its (b,g) region
  int32_t* lane_mode;      // [B,G,K] cascade of this flush: 0 none, 1 parallel kernels, 2 sequential walk
  struct LevelPlan* lane_plan;  // [B,G,K,L] what every level does in this flush (prepare kernel)
  int64_t* plan_base;      // [B,G,K] order of the first token row (level0_phase before the flush)
  // Ladder scratch: [B*G][2][S] rows, structure of arrays.
  void* sk;
  void* sv;
  float* sw;
  int64_t* slo;
  int64_t* shi;
  int64_t* sswp;
  int64_t* sord;
  uint8_t* spad;
  // Window staging for overlapping shifts: [B,G,2R,D] x3 + [B,2R] x2.
  void* wk;
  void* wkr;
  void* wv;
  int64_t* wpos;
  uint8_t* wends;
  UWork u;                 // unified route only
};

// Relative gap of two values: |a - b| / max(|a|, |b|) (0 when both are 0; NaN-safe: NaN gives
// a gap that is not below any threshold).
__device__ __forceinline__ float rel_gap(float a, float b) {
  const float den = fmaxf(fabsf(a), fabsf(b));
  return den > 0.f ? fdiv(fabsf(fsub(a, b)), den) : 0.f;
}
// Division-free test of rel_gap(a, b) < kTieRel (false for NaN); rel_gap is computed only when logging.
__device__ __forceinline__ bool near_tie(float a, float b) {
  return fabsf(fsub(a, b)) < fmul(kTieRel, fmaxf(fabsf(a), fabsf(b)));
}

// Append one near-tie entry (flush index = flushes counted so far, minus one).
__device__ __forceinline__ void log_tie(const Work& w, int kind, int b, int g, int c, int index, int first,
                                        int second, float gap, float value) {
  const unsigned long long slot = atomicAdd(&w.counters[kCntTies], 1ull);
  if (slot >= (unsigned long long)kTieCap) return;
  const unsigned long long flushes = *reinterpret_cast<volatile unsigned long long*>(&w.counters[kCntFlushes]);
  TieEntry e{kind, (int32_t)flushes - 1, b, g, c, index, first, second, gap, value};
  w.ties[slot] = e;
}

// 16-byte vectors of storage elements.
template <typename T>
struct Vec {
  static constexpr int N = 16 / sizeof(T);
};

__device__ __forceinline__ void unpack(const uint4& u, float* out, const float*) {
  const float* f = reinterpret_cast<const float*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) out[i] = f[i];
}
__device__ __forceinline__ void unpack(const uint4& u, float* out, const __nv_bfloat16*) {
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = __bfloat162float(h[i]);
}
__device__ __forceinline__ uint4 pack(const float* in, const float*) {
  uint4 u;
  float* f = reinterpret_cast<float*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) f[i] = in[i];
  return u;
}
__device__ __forceinline__ uint4 pack(const float* in, const __nv_bfloat16*) {
  uint4 u;
  __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = __float2bfloat16_rn(in[i]);
  return u;
}

// Position of token `src` of row b in [old pool | flush] index space.
__device__ __forceinline__ int64_t token_position(const Geo& g, const logkv_state_t& s, const Work& w, int b,
                                                  int src) {
  return src < g.P ? w.snap_pos[(size_t)b * g.P + src] : s.recent_pos[(size_t)b * g.cap2R + (src - g.P)];
}

// Pointer to the D features of token `src` of (b, group) for a [pool | window] pair of sources.
template <typename T>
__device__ __forceinline__ const T* token_row(const Geo& g, const T* snap, const T* recent, int b, int grp,
                                              int src) {
  if (src < g.P) return snap + (((size_t)b * g.G + grp) * g.P + src) * g.D;
  return recent + (((size_t)b * g.G + grp) * g.cap2R + (src - g.P)) * g.D;
}

}  // namespace logkv
