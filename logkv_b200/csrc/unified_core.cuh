// Mutual-nearest Ward rounds on one lane by one thread-block cluster: the device core of the
// unified (Ward / radius) route, shared by the operator-level API (unified.cu: one round per
// launch, the reference plugin's UnifiedReduce) and the flush-level route (flush_unified.cuh:
// every round of a pass in one persistent launch).
//
// Semantics of the reference's Torch reducer _UnifiedReduceTorch (litgpt/log_kv_cache.py:448-638):
// row minima of packed (Ward cost bits << 32 | row ^ col) keys, disjoint mutual pairs, exact
// radius verification when a limit is given, frozen-centre sweeps when passes > 1 (:564-588), a
// per-lane budget of count - target pairs by increasing cost, Lance-Williams row updates and
// rescans of rows whose best partner merged.  Every operation is float32, rounded as the
// reference writes it (the including translation units are compiled without fused
// multiply-adds); the exact squared distance of a candidate pair sums the features left to right.
//
// A cluster of 2 to kUCluster CTAs runs one round of one lane: the leader selects the pairs, all CTAs
// share the centre, Lance-Williams and rescan work; within a round every merge writes only its
// own row and column, which no other merge of the round reads.
#pragma once

#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/logkv_b200.h"

namespace logkv_ward {

namespace cg = cooperative_groups;

constexpr int kUThreads = 1024;
constexpr int kUCluster = 8;        // most CTAs per lane (one thread-block cluster)
constexpr int kUMaxSize = 4096;     // rows per lane (the pair sort runs in shared memory)
constexpr long long kInfKey = 0x7F800000LL << 32;

__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// (cost bits << 32) | key, with -0.0 written as +0.0 (_unified_pack, log_kv_cache.py:431-434).
__device__ __forceinline__ long long pack_key(float cost, long long key) {
  if (cost == 0.f) cost = 0.f;
  return ((long long)__float_as_int(cost) << 32) | key;
}

// Ward cost of joining clusters i and j, +inf when the pair is not allowed
// (_unified_pair_cost, log_kv_cache.py:437-445).
__device__ __forceinline__ float pair_cost(float d2, float mi, float mj, float ri, float rj, const float* limit,
                                           bool valid) {
  const float denom = fmaxf(fadd(mi, mj), 1.f);
  valid = valid && mi > 0.f && mj > 0.f;
  if (limit) {
    // Exact early out: with radii >= 0 and mi + mj >= 1, every rounding above leaves
    // max(b1, b2) >= sqrt(d2) (1 - 5u) / 2 (u = 2^-24), so d2 > 4.0001 limit^2 proves the pair
    // invalid without its divisions (an infinite or NaN limit never takes this branch).
    if (denom == fadd(mi, mj) && d2 > fmul(fmul(4.0001f, *limit), *limit)) return __int_as_float(0x7F800000);
    const float distance = __fsqrt_rn(d2);
    const float b1 = fadd(ri, fmul(fdiv(mj, denom), distance));
    const float b2 = fadd(rj, fmul(fdiv(mi, denom), distance));
    valid = valid && fmaxf(b1, b2) <= *limit;
  }
  return valid ? fmul(d2, fdiv(fmul(mi, mj), denom)) : __int_as_float(0x7F800000);
}

// A lower bound of pair_cost's finite value from a fast division: __fdividef is within 2 ulp of
// the quotient (denominators here lie in [1, 2^126]), so the bound is below the exact cost by at
// most ~4 ulp, and 2^-18 of slack covers it; tiny costs are never bounded (0 returned).  A pair
// whose bound exceeds a known key's cost cannot have the smaller key (keys order by cost bits
// first), so its exact evaluation can be skipped.
__device__ __forceinline__ float cost_lower_bound(float d2, float mi, float mj) {
  const float approx = __fmul_rn(d2, __fdividef(__fmul_rn(mi, mj), fmaxf(__fadd_rn(mi, mj), 1.f)));
  return approx > 1e-30f ? __fmul_rn(approx, 0.999996f) : 0.f;
}
__device__ __forceinline__ float key_cost(long long key) { return __int_as_float((int)(key >> 32)); }

// Where a lane's near ties go (the flush workspace's tie log), or nowhere (count null): a
// decision whose best and runner-up costs lie within a relative 1e-6 of each other, which the
// reference's own summation order could decide the other way.
struct TieSink {
  unsigned long long* count;          // entries requested (entries beyond cap are counted only)
  logkv_tie_t* log;
  const unsigned long long* flushes;  // flushes so far (the entry's flush index is this - 1)
  int cap, b, g;
};

__device__ __forceinline__ bool near_tie_cost(float a, float b) {
  return fabsf(fsub(a, b)) < fmul(1e-6f, fmaxf(fabsf(a), fabsf(b)));
}

__device__ inline void log_ward_tie(const TieSink& t, int kind, int pass, int index, int first, int second, float a,
                                    float b) {
  if (!t.count) return;
  const unsigned long long slot = atomicAdd(t.count, 1ull);
  if (slot >= (unsigned long long)t.cap) return;
  const float den = fmaxf(fabsf(a), fabsf(b));
  const float gap = den > 0.f ? fdiv(fabsf(fsub(a, b)), den) : 0.f;
  const unsigned long long f = *reinterpret_cast<const volatile unsigned long long*>(t.flushes);
  t.log[slot] = logkv_tie_t{kind, (int32_t)f - 1, t.b, t.g, pass, index, first, second, gap, a};
}

// One lane's device state.  Rows are [0, M); the live count, merge count, flags and trace are
// this lane's own words.
struct RunLane {
  float* dist;           // [M, M] squared centre distances (symmetric)
  float* mu;             // [M, D] centres
  float* mass;           // [M]
  float* radius;         // [M]
  uint8_t* alive;        // [M]
  long long* packed;     // [M] row minima
  long long* restricted; // [M] sweep scratch (passes > 1), else null
  const float* limit;    // radius limit or null
  int* count;            // live clusters
  int* active;           // lane still active after the last round
  int* merges;           // merges so far (= trace rows)
  uint8_t* stuck;        // a round had no proposal while above target
  int* trace;            // [M, 2] merge pairs in round order; within a round in (cost, left) order,
                         // or in row order when `cost_order` is 0 and the budget takes every pair
  int M, D, target, passes;
  int cost_order;        // sort every round's pairs by cost (the operator API's trace contract)
  int pass;              // 0 candidate pass, 1 global pass (tie log entries)
  TieSink ties;          // near-tie log of the row minima and the budget cut
};

// out[r] = min over columns of the row's packed keys; one warp per row.  Only live columns
// (`cols`, or [0, ncols) when cols is null) are visited: any other column's key is +inf with
// r ^ c > 0, never below the key of the row's own column, (+inf, 0), which starts the minimum.
// Columns whose `excluded` flag has bit `xbit` count as massless (the sweeps' restricted scans).
__device__ inline void scan_rows(const RunLane& l, const int* rows, int nrows, const int* cols, int ncols,
                                 long long* out, const uint8_t* excluded = nullptr, uint8_t xbit = 0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int M = l.M;
  constexpr int kBatch = 4;   // columns per lane whose loads are in flight together
  for (int i = warp; i < nrows; i += nwarps) {
    const int r = rows[i];
    const float* drow = l.dist + (size_t)r * M;
    const float mr = l.mass[r], rr = l.radius[r];
    long long best = kInfKey, second = kInfKey;   // the row's minimum key and the next one
    const bool tie_log = l.ties.count != nullptr;
    for (int kb = lane; kb < ncols; kb += 32 * kBatch) {
      int cv[kBatch];
      float dv[kBatch], mv[kBatch], rv[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int k = kb + 32 * j;
        cv[j] = k < ncols ? (cols ? cols[k] : k) : -1;
        const int c = cv[j] < 0 ? r : cv[j];
        dv[j] = drow[c];
        mv[j] = (excluded && (excluded[c] & xbit)) ? 0.f : l.mass[c];
        rv[j] = l.radius[c];
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        if (cv[j] < 0) continue;
        // With the tie log on, the runner-up is kept exactly while it lies within 4e-6 of the
        // minimum (beyond that it cannot be a near tie, and the bound skips it).
        const float bound = tie_log ? fminf(key_cost(second), fmul(key_cost(best), 1.000004f)) : key_cost(best);
        if (cost_lower_bound(dv[j], mr, mv[j]) > bound) continue;
        const float cost = pair_cost(dv[j], mr, mv[j], rr, rv[j], l.limit, cv[j] != r);
        const long long key = pack_key(cost, (long long)(r ^ cv[j]));
        if (key < best) {
          second = best;
          best = key;
        } else if (key < second) {
          second = key;
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const long long ob = __shfl_xor_sync(0xffffffffu, best, off), os = __shfl_xor_sync(0xffffffffu, second, off);
      second = min(min(second, os), max(best, ob));
      best = min(best, ob);
    }
    if (lane == 0) {
      out[r] = best;
      const float bc = key_cost(best), sc = key_cost(second);
      if (tie_log && bc < __int_as_float(0x7F800000) && sc < __int_as_float(0x7F800000) && near_tie_cost(bc, sc))
        log_ward_tie(l.ties, LOGKV_TIE_WARD_MIN, l.pass, r, (int)((best & 0xFFFFFFFFLL) ^ r),
                     (int)((second & 0xFFFFFFFFLL) ^ r), bc, sc);
    }
  }
}

// Every live row's minimum, at the lane's start; the rows are split over the cluster's CTAs
// (row r on CTA r % CL).  `rows` is an [M] int scratch of this CTA, n_sh a shared int.
__device__ inline void init_lane(const RunLane& l, int part, int CL, int* rows, int* n_sh) {
  const int M = l.M;
  const int count = *l.count;
  if (threadIdx.x == 0) *n_sh = 0;
  __syncthreads();
  for (int r = part + CL * (int)threadIdx.x; r < M; r += CL * blockDim.x) {
    const bool live = r < count;
    l.alive[r] = live;
    l.radius[r] = 0.f;
    l.packed[r] = kInfKey;
    if (live) rows[atomicAdd(n_sh, 1)] = r;
  }
  __syncthreads();
  scan_rows(l, rows, *n_sh, nullptr, count < M ? count : M, l.packed);
}

// Shared memory of one round (the same layout in every CTA of a lane's cluster).
struct RoundSmem {
  unsigned long long* sk;  // [S] sort keys (leader)
  long long* rowmin;       // [M/2 + 1] this CTA's row minima of the merged rows
  long long* colmin;       // [CW] this CTA's column minima
  int* best;               // [M]
  int* partner;            // [M] the mate of a kept row
  int* rows;               // [M] dirty rows of this CTA (every row's mate while the leader selects)
  int* pairs;              // [M/2 + 1] kept row of merge m, in merge order
  int* cols;               // [M] live columns after the merges, ascending
  float* bound;            // [M]
  float* pma;              // [M] masses of a merge's rows, at its kept row
  float* pmb;              // [M]
  float* alpha;            // [M] ma / total, mb / total and alpha * beta * d_ab of a merge, at its kept row
  float* beta;             // [M]
  float* shift;            // [M]
  uint8_t* flags;          // [M] 1 valid, 2 rejected, 4 keep, 8 merged, 16 matched (sweeps), 32 sweep pair
};

// Live columns per CTA of a cluster of CL, in whole warps.
__host__ __device__ inline int column_width(int M, int CL) { return ((M + CL - 1) / CL + 31) / 32 * 32; }

__host__ __device__ inline size_t round_smem_bytes(int M, int S, int CL) {
  const size_t half = (size_t)M / 2 + 1;
  return (size_t)S * 8 + half * 8 + (size_t)column_width(M, CL) * 8 + (size_t)M * 4 * 3 + half * 4 +
         (size_t)M * 4 * 7 + (size_t)M + 16;
}

// Sort width of a round: a power of two >= M / 2 (at most M / 2 disjoint pairs are sorted).
__host__ __device__ inline int sort_width(int M) {
  int p = 2;
  while (p < M / 2) p <<= 1;
  return p;
}

__device__ inline RoundSmem carve_round(void* base, int M, int S, int CL) {
  RoundSmem r;
  char* p = static_cast<char*>(base);
  const size_t half = (size_t)M / 2 + 1;
  r.sk = reinterpret_cast<unsigned long long*>(p);
  p += (size_t)S * 8;
  r.rowmin = reinterpret_cast<long long*>(p);
  p += half * 8;
  r.colmin = reinterpret_cast<long long*>(p);
  p += (size_t)column_width(M, CL) * 8;
  r.best = reinterpret_cast<int*>(p);
  p += (size_t)M * 4;
  r.partner = reinterpret_cast<int*>(p);
  p += (size_t)M * 4;
  r.rows = reinterpret_cast<int*>(p);
  p += (size_t)M * 4;
  r.pairs = reinterpret_cast<int*>(p);
  p += half * 4;
  r.cols = reinterpret_cast<int*>(p);
  p += (size_t)M * 4;
  r.bound = reinterpret_cast<float*>(p);
  p += (size_t)M * 4;
  r.pma = reinterpret_cast<float*>(p);
  p += (size_t)M * 4;
  r.pmb = reinterpret_cast<float*>(p);
  p += (size_t)M * 4;
  r.alpha = reinterpret_cast<float*>(p);
  p += (size_t)M * 4;
  r.beta = reinterpret_cast<float*>(p);
  p += (size_t)M * 4;
  r.shift = reinterpret_cast<float*>(p);
  p += (size_t)M * 4;
  r.flags = reinterpret_cast<uint8_t*>(p);
  return r;
}

__device__ __forceinline__ int key_partner(long long key, int r, int M) {
  const int p = (int)((key & 0xFFFFFFFFLL) ^ (long long)r);
  return p < 0 ? 0 : (p > M - 1 ? M - 1 : p);
}

// Frozen-centre sweeps (_UnifiedReduceTorch._sweeps, log_kv_cache.py:564-588), leader CTA, after
// the first mutual pairs: rows whose restricted partner was matched rescan the unmatched columns,
// then unmatched mutual pairs of the restricted minima pair up too (flag 32); sm.rows holds every
// row's mate.  Returns the extra proposals.
__device__ inline int sweeps(const RunLane& l, const RoundSmem& sm) {
  const int M = l.M, tid = threadIdx.x, nt = blockDim.x;
  __shared__ int n_scan, n_more;
  for (int r = tid; r < M; r += nt)
    if (sm.flags[r] & 1) sm.flags[r] |= 16;
  __syncthreads();
  // A valid row's partner is above it, never valid itself, and belongs to that pair only.
  for (int r = tid; r < M; r += nt)
    if (sm.flags[r] & 1) sm.flags[sm.best[r]] |= 16;
  for (int r = tid; r < M; r += nt) {
    l.restricted[r] = l.packed[r];
    sm.rows[r] = sm.best[r];
  }
  int extra = 0;
  for (int pass = 1; pass < l.passes; ++pass) {
    if (tid == 0) {
      n_scan = 0;
      n_more = 0;
    }
    __syncthreads();
    // Rows to rescan: live, unmatched, whose restricted partner is matched (as of the pass's start).
    for (int r = tid; r < M; r += nt) {
      if (!l.alive[r] || (sm.flags[r] & 16)) continue;
      if (sm.flags[key_partner(l.restricted[r], r, M)] & 16) sm.cols[atomicAdd(&n_scan, 1)] = r;
    }
    __syncthreads();
    scan_rows(l, sm.cols, n_scan, nullptr, M, l.restricted, sm.flags, 16);
    __syncthreads();
    // Unmatched mutual pairs of the restricted minima (matched as of the pass's start).
    for (int r = tid; r < M; r += nt) {
      if (!l.alive[r] || (sm.flags[r] & 16)) continue;
      const long long key = l.restricted[r];
      const int p = key_partner(key, r, M);
      const int pp = key_partner(l.restricted[p], p, M);
      const float cost = __int_as_float((int)(key >> 32));
      if (r < p && pp == r && cost < __int_as_float(0x7F800000) && !(sm.flags[p] & 16))
        sm.pairs[atomicAdd(&n_more, 1)] = r;
    }
    __syncthreads();
    const int nm = n_more;
    for (int i = tid; i < nm; i += nt) {
      const int r = sm.pairs[i];
      const int p = key_partner(l.restricted[r], r, M);
      sm.flags[r] |= 16 | 32;
      sm.flags[p] |= 16;
      sm.rows[r] = p;
    }
    extra += nm;
    __syncthreads();
  }
  return extra;
}

// Leader CTA: proposals, exact radius checks, sweeps, the pairs' cost order and budget, and the
// merged clusters' masses, liveness and radii; the trace and the lane's status.  Returns whether
// the lane stays active.
__device__ inline bool select_pairs(const RunLane& l, const RoundSmem& sm, int* n_ok_out) {
  const int M = l.M, D = l.D, tid = threadIdx.x, nt = blockDim.x;
  __shared__ int nprop, nvalid, nok;
  if (tid == 0) {
    nprop = 0;
    nvalid = 0;
  }
  const unsigned inf_bits = 0x7F800000u;
  for (int r = tid; r < M; r += nt) {
    sm.best[r] = key_partner(l.packed[r], r, M);
    sm.partner[r] = 0;
    sm.pma[r] = 1.f;
    sm.pmb[r] = 0.f;
    sm.bound[r] = 0.f;
  }
  __syncthreads();
  for (int r = tid; r < M; r += nt) {
    const long long p = l.packed[r];
    const float cost = __int_as_float((int)(p >> 32));
    const int b = sm.best[r];
    const bool v = l.alive[r] && r < b && sm.best[b] == r && cost < __int_as_float(inf_bits);
    sm.flags[r] = v ? 1 : 0;
    if (v) atomicAdd(&nprop, 1);
  }
  __syncthreads();
  if (l.limit) {
    for (int r = tid; r < M; r += nt) {
      if (!(sm.flags[r] & 1)) continue;
      const int o = sm.best[r];
      const float* xa = l.mu + (size_t)r * D;
      const float* xb = l.mu + (size_t)o * D;
      float exact2 = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) {
        const float df = fsub(xa[d], xb[d]);
        exact2 = fadd(exact2, fmul(df, df));
      }
      const float exact = __fsqrt_rn(exact2);
      const float ma = l.mass[r], mb = l.mass[o];
      const float denom = fmaxf(fadd(ma, mb), 1.f);
      const float verified =
          fmaxf(fadd(l.radius[r], fmul(fdiv(mb, denom), exact)), fadd(l.radius[o], fmul(fdiv(ma, denom), exact)));
      if (verified > *l.limit) {
        l.dist[(size_t)r * M + o] = exact2;
        l.dist[(size_t)o * M + r] = exact2;
        sm.flags[r] = 2;          // rejected, no longer valid
        sm.flags[o] |= 2;
      }
      sm.bound[r] = verified;
    }
  }
  __syncthreads();
  int extra = 0;
  const bool swept = l.passes > 1 && l.restricted;
  if (swept) extra = sweeps(l, sm);
  // Valid pairs (a row each, below its partner; finite costs) as (cost bits << 32 | row), in row
  // order; a sweep pair carries its restricted cost.  The reference takes them in stable cost
  // order up to the budget; when the budget takes them all, the order within the round changes
  // nothing (the round's pairs are disjoint), so the sort runs only when the budget cuts.
  {
    const int per = (M + nt - 1) / nt, lo = min(M, tid * per), hi = min(M, lo + per);
    int cnt = 0;
    for (int r = lo; r < hi; ++r) cnt += (sm.flags[r] & (1 | 32)) != 0;
    __shared__ int ws[kUThreads / 32];
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if ((tid & 31) >= off) incl += v;
    }
    if ((tid & 31) == 31) ws[tid >> 5] = incl;
    __syncthreads();
    if (tid < 32) {
      int w = tid < nt / 32 ? ws[tid] : 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, w, off);
        if (tid >= off) w += v;
      }
      if (tid < nt / 32) ws[tid] = w;
      if (tid == 31) nvalid = w;
    }
    __syncthreads();
    int at = incl - cnt + ((tid >> 5) ? ws[(tid >> 5) - 1] : 0);
    for (int r = lo; r < hi; ++r) {
      const uint8_t f = sm.flags[r];
      if (f & 1) sm.sk[at++] = ((unsigned long long)(l.packed[r] >> 32) << 32) | (unsigned)r;
      else if (f & 32) sm.sk[at++] = ((unsigned long long)(l.restricted[r] >> 32) << 32) | (unsigned)r;
    }
  }
  __syncthreads();
  const int nv = nvalid;
  const bool cut = l.cost_order || nv > M / 2 || nv > *l.count - l.target;
  int S = 1;
  while (cut && S < nv) S <<= 1;
  for (int i = nv + tid; i < S; i += nt) sm.sk[i] = ~0ull;
  __syncthreads();
  for (int k = 2; k <= S; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < S; i += nt) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = sm.sk[i], y = sm.sk[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) {
            sm.sk[i] = y;
            sm.sk[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  // Budget: the first min(valid, count - target, M / 2) pairs merge.
  const int count = *l.count;
  if (tid == 0) {
    int n = min(nv, M / 2);
    n = min(n, max(count - l.target, 0));
    nok = n;
    if (cut && n > 0 && n < nv) {
      const float a = __int_as_float((int)(sm.sk[n - 1] >> 32)), b = __int_as_float((int)(sm.sk[n] >> 32));
      if (near_tie_cost(a, b))
        log_ward_tie(l.ties, LOGKV_TIE_WARD_BUDGET, l.pass, n - 1, (int)(sm.sk[n - 1] & 0xFFFFFFFFull),
                     (int)(sm.sk[n] & 0xFFFFFFFFull), a, b);
    }
  }
  __syncthreads();
  const int n_ok = nok;
  const int trace0 = *l.merges;
  for (int m = tid; m < n_ok; m += nt) {
    const int a = (int)(sm.sk[m] & 0xFFFFFFFFull), b = swept ? sm.rows[a] : sm.best[a];
    sm.pairs[m] = a;
    sm.flags[a] |= 4 | 8;
    sm.flags[b] |= 8;
    sm.partner[a] = b;
    const float ma = l.mass[a], mb = l.mass[b];
    const float total = fadd(ma, mb);
    const float al = fdiv(ma, total), be = fdiv(mb, total);
    sm.pma[a] = ma;
    sm.pmb[a] = mb;
    sm.alpha[a] = al;
    sm.beta[a] = be;
    sm.shift[a] = fmul(fmul(al, be), l.dist[(size_t)a * M + b]);
    l.trace[(size_t)(trace0 + m) * 2] = a;
    l.trace[(size_t)(trace0 + m) * 2 + 1] = b;
  }
  __syncthreads();
  for (int m = tid; m < n_ok; m += nt) {
    const int a = sm.pairs[m], b = sm.partner[a];
    l.mass[a] = fadd(sm.pma[a], sm.pmb[a]);
    l.mass[b] = 0.f;
    l.alive[b] = 0;
    if (l.limit) l.radius[a] = sm.bound[a];
  }
  const int props = nprop + extra;
  const int left = count - n_ok;
  const bool remaining = left > l.target;
  if (tid == 0) {
    *l.count = left;
    *l.merges = trace0 + n_ok;
    if (remaining && props == 0) *l.stuck = 1;
    *l.active = remaining && props > 0;
  }
  *n_ok_out = n_ok;
  return remaining && props > 0;
}

// One round of one lane on its cluster.  The leader selects the pairs; every CTA copies the
// round's tables from the leader's shared memory, updates a share of the merged centres, the
// Lance-Williams values of its columns of every merged row, and rescans its dirty rows.  Within
// the round every merge writes only its own row and column, which no other merge reads, and the
// phases are separated by cluster barriers (which also order the global writes).  Returns the
// lane's active flag (every CTA): the leader publishes it in word `parity` of its two-word shared
// `act`, which the next round's other word keeps from being overwritten before every CTA read it.
__device__ inline bool run_round(cg::cluster_group& cluster, const RunLane& l, void* smem_raw, int S, int* act,
                                 int parity) {
  const int part = (int)cluster.block_rank(), CL = (int)cluster.num_blocks();
  const int M = l.M, D = l.D, tid = threadIdx.x, nt = blockDim.x;
  const RoundSmem sm = carve_round(smem_raw, M, S, CL);
  __shared__ int n_ok_s, ndirty;
  if (part == 0) {
    int n_ok;
    const bool a = select_pairs(l, sm, &n_ok);
    if (tid == 0) {
      n_ok_s = n_ok;
      act[parity] = a;
    }
  }
  cluster.sync();
  // ---- the round's tables, from the leader
  if (part != 0) {
    const RoundSmem lead = carve_round(cluster.map_shared_rank(smem_raw, 0), M, S, CL);
    if (tid == 0) n_ok_s = *cluster.map_shared_rank(&n_ok_s, 0);
    for (int r = tid; r < M; r += nt) {
      sm.best[r] = lead.best[r];
      sm.partner[r] = lead.partner[r];
      sm.pma[r] = lead.pma[r];
      sm.pmb[r] = lead.pmb[r];
      sm.alpha[r] = lead.alpha[r];
      sm.beta[r] = lead.beta[r];
      sm.shift[r] = lead.shift[r];
      sm.flags[r] = lead.flags[r];
    }
    __syncthreads();
    for (int m = tid; m < n_ok_s; m += nt) sm.pairs[m] = lead.pairs[m];
  }
  if (tid == 0) ndirty = 0;
  __syncthreads();
  const int n_ok = n_ok_s;
  // ---- merged centres: merge m goes to CTA m % CL
  for (int item = tid; item < ((n_ok - part + CL - 1) / CL) * D; item += nt) {
    const int m = part + CL * (item / D), d = item % D;
    const int a = sm.pairs[m], b = sm.partner[a];
    const float ma = sm.pma[a], mb = sm.pmb[a];
    const float total = fadd(ma, mb);
    float* ra = l.mu + (size_t)a * D;
    const float* rb = l.mu + (size_t)b * D;
    ra[d] = fdiv(fadd(fmul(ma, ra[d]), fmul(mb, rb[d])), fmaxf(total, 1.f));
  }
  // ---- live columns after the merges (ascending): a block scan of the alive flags
  __shared__ int wsum[kUThreads / 32], ncols_s;
  {
    const int per = (M + nt - 1) / nt, lo = tid * per, hi = min(M, lo + per);
    int cnt = 0;
    for (int c = lo; c < hi; ++c) cnt += l.alive[c] != 0;
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if ((tid & 31) >= off) incl += v;
    }
    if ((tid & 31) == 31) wsum[tid >> 5] = incl;
    __syncthreads();
    if (tid < 32) {
      int w = tid < nt / 32 ? wsum[tid] : 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, w, off);
        if (tid >= off) w += v;
      }
      if (tid < nt / 32) wsum[tid] = w;
      if (tid == 31) ncols_s = w;
    }
    __syncthreads();
    int at = incl - cnt + ((tid >> 5) ? wsum[(tid >> 5) - 1] : 0);
    for (int c = lo; c < hi; ++c)
      if (l.alive[c]) sm.cols[at++] = c;
  }
  __syncthreads();
  const int ncols = ncols_s;
  // ---- Lance-Williams: this CTA's share [k0, k0 + CW) of the live columns, every merged row,
  // as warp tasks of (merge, 32 columns); a merge's scalars were computed once by the leader.
  const int CW = column_width(ncols, CL), k0 = part * CW;
  for (int i = tid; i < n_ok; i += nt) sm.rowmin[i] = kInfKey;
  for (int i = tid; i < CW; i += nt) sm.colmin[i] = 0x7FFFFFFFFFFFFFFFLL;
  __syncthreads();
  constexpr int kChunks = 4;   // 32-column chunks per warp task, their loads in flight together
  const int lanew = tid & 31, nchunk = CW / 32, ngrp = (nchunk + kChunks - 1) / kChunks;
  const int ntask = k0 < ncols ? n_ok * ngrp : 0;
  for (int task = tid >> 5; task < ntask; task += nt >> 5) {
    const int m = task / ngrp, g0 = (task - m * ngrp) * kChunks;
    const int a = sm.pairs[m], b = sm.partner[a];
    const float alpha = sm.alpha[a], beta = sm.beta[a], shift = sm.shift[a];
    const float total = fadd(sm.pma[a], sm.pmb[a]), ra = l.radius[a];
    const float* rowa = l.dist + (size_t)a * M;
    const float* rowb = l.dist + (size_t)b * M;
    int cv[kChunks];
    float xaa[kChunks], xba[kChunks], mc[kChunks], rc[kChunks], pc[kChunks];
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const int k = k0 + (g0 + j) * 32 + lanew;
      cv[j] = (g0 + j < nchunk && k < ncols) ? sm.cols[k] : -1;
      const int c = cv[j] < 0 ? a : cv[j];
      xaa[j] = rowa[c];
      xba[j] = rowb[c];
      mc[j] = l.mass[c];
      rc[j] = l.radius[c];
      pc[j] = key_cost(l.packed[c]);
    }
    long long rkey = kInfKey;
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const int c = cv[j];
      if (c < 0) continue;
      const float x_aa = xaa[j], x_ba = xba[j];
      float nv = fsub(fadd(fmul(alpha, x_aa), fmul(beta, x_ba)), shift);
      const bool keep_c = sm.flags[c] & 4;
      if (keep_c) {
        // Both clusters merged this round: the lower keep index's order, so both owners agree.
        const int q = sm.partner[c];
        const float x_ab = rowa[q], x_bb = rowb[q];
        const float qal = sm.alpha[c], qbe = sm.beta[c], qsh = sm.shift[c];
        float v;
        if (a < c) {
          const float inner = fsub(fadd(fmul(alpha, x_ab), fmul(beta, x_bb)), shift);
          v = fsub(fadd(fmul(qal, nv), fmul(qbe, inner)), qsh);
        } else {
          const float t1 = fsub(fadd(fmul(qal, x_aa), fmul(qbe, x_ab)), qsh);
          const float t2 = fsub(fadd(fmul(qal, x_ba), fmul(qbe, x_bb)), qsh);
          v = fsub(fadd(fmul(alpha, t1), fmul(beta, t2)), shift);
        }
        nv = v;
      }
      nv = fmaxf(nv, 0.f);
      if (c == a) nv = 0.f;
      if (!keep_c) l.dist[(size_t)c * M + a] = nv;
      l.dist[(size_t)a * M + c] = nv;
      // The key matters only if it can lower the row's minimum or (a column that is not a merged
      // row) the column's current one; a column whose minimum went stale is rescanned anyway.
      const float lb = cost_lower_bound(nv, total, mc[j]);
      if (lb > key_cost(rkey) && (keep_c || lb > pc[j])) continue;
      const float cost = pair_cost(nv, total, mc[j], ra, rc[j], l.limit, c != a);
      const long long key = pack_key(cost, (long long)(a ^ c));
      if (cost < __int_as_float(0x7F800000) && !keep_c) atomicMin(&sm.colmin[(g0 + j) * 32 + lanew], key);
      rkey = min(rkey, key);
    }
    // A warp task covers columns of one merge only: one row-minimum atomic per task.
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) rkey = min(rkey, __shfl_xor_sync(0xffffffffu, rkey, off));
    if (lanew == 0) atomicMin(&sm.rowmin[m], rkey);
  }
  __syncthreads();
  // Columns this CTA owns take their new minima (non-merged columns only; an invalid key never lowers).
  for (int kl = tid; kl < CW && k0 + kl < ncols; kl += nt) {
    const int c = sm.cols[k0 + kl];
    if (!(sm.flags[c] & 4) && sm.colmin[kl] < l.packed[c]) l.packed[c] = sm.colmin[kl];
  }
  cluster.sync();
  // ---- merged rows: minimum over every CTA's columns (merge m on CTA m % CL)
  for (int m = part + CL * tid; m < n_ok; m += CL * nt) {
    long long v = sm.rowmin[m];
    for (int r = 1; r < CL; ++r)
      v = min(v, cluster.map_shared_rank(sm.rowmin, (part + r) % CL)[m]);
    l.packed[sm.pairs[m]] = v;
  }
  // ---- rows whose best partner merged (or that were rejected) rescan; row r on CTA r % CL
  for (int r = part + CL * tid; r < M; r += CL * nt) {
    const uint8_t f = sm.flags[r];
    if (l.alive[r] && !(f & 4) && ((sm.flags[sm.best[r]] & 8) || (f & 2))) sm.rows[atomicAdd(&ndirty, 1)] = r;
  }
  __syncthreads();
  scan_rows(l, sm.rows, ndirty, sm.cols, ncols, l.packed);
  cluster.sync();   // no CTA leaves while another may still read its row minima
  return cluster.map_shared_rank(act, 0)[parity] != 0;
}

}  // namespace logkv_ward
