// Per-cluster ladder commit: centroid update, new-cluster / delayed re-insert
// preparation, and the level cascade with pairwise or Beta 4->2 merges.
//
// Semantics of _semantic_append_entries_batched (litgpt/log_kv_cache.py:1756-1929):
// at a level holding c entries with m incoming rows, pool = stored[0:c] ++
// incoming.  If c + m <= B' the rows fill slots c.. .  Otherwise the first
// 2*ceil((c+m-B')/2) pool rows merge (compact :5217-5387, or Beta apply_cuts,
// litgpt/beta_log_kv.py:49-92) into the next level's incoming rows, the rest
// of the pool becomes slots 0.., and the tail slots are zeroed.  The top level
// folds its oldest entries (:1670-1728).  Merged K/V are rounded to the
// storage dtype when written, which is exactly when the reference rounds them
// (every consumer of a carried row casts it to the storage dtype first).
#pragma once

#include "flush_common.cuh"

namespace logkv {

struct Meta {
  float w;
  int64_t lo, hi, swp, ord;
  uint8_t pad;
};

__device__ __forceinline__ Meta merge_meta(const Meta& a, const Meta& b) {
  Meta o;
  o.w = fadd(a.w, b.w);
  const bool ra = a.w > 0.f, rb = b.w > 0.f;
  o.lo = (ra && rb) ? min(a.lo, b.lo) : (ra ? a.lo : b.lo);
  o.hi = (ra && rb) ? max(a.hi, b.hi) : (ra ? a.hi : b.hi);
  o.swp = a.swp + b.swp;
  o.ord = min(a.ord, b.ord);
  o.pad = a.pad & b.pad;
  return o;
}

// Incoming rows of one level: either the cluster's archived tokens or scratch rows.
struct Stage {
  int kind;   // 0 = tokens, 1 = scratch rows
  int buf;    // scratch buffer (kind 1)
  int m;      // rows
};

template <typename T>
struct LaneCtx {
  Geo g;
  logkv_state_t s;
  Work w;
  int b, grp, c;
  size_t lane, bg;
  int toff, scr;
  int64_t base_order;
  const int* arch;
  const int* toks;
  const T* snapk;
  const T* snapv;
  const T* reck;
  const T* recv;

  __device__ size_t scr_row(int buf, int i) const { return (bg * 2 + buf) * (size_t)g.S + scr + i; }
  __device__ int token_src(int i) const { return arch[toks[toff + i]]; }
  __device__ const T* stage_k(const Stage& st, int i) const {
    if (st.kind == 0) return token_row<T>(g, snapk, reck, b, grp, token_src(i));
    return static_cast<const T*>(w.sk) + scr_row(st.buf, i) * g.D;
  }
  __device__ const T* stage_v(const Stage& st, int i) const {
    if (st.kind == 0) return token_row<T>(g, snapv, recv, b, grp, token_src(i));
    return static_cast<const T*>(w.sv) + scr_row(st.buf, i) * g.D;
  }
  __device__ Meta stage_meta(const Stage& st, int i) const {
    Meta m;
    if (st.kind == 0) {
      const int64_t p = token_position(g, s, w, b, token_src(i));
      m.w = 1.f;
      m.lo = m.hi = m.swp = p;
      m.ord = base_order + i;
      m.pad = 0;
    } else {
      const size_t r = scr_row(st.buf, i);
      m.w = w.sw[r];
      m.lo = w.slo[r];
      m.hi = w.shi[r];
      m.swp = w.sswp[r];
      m.ord = w.sord[r];
      m.pad = w.spad[r];
    }
    return m;
  }
  __device__ void put_scratch(int buf, int i, const Meta& m) const {
    const size_t r = scr_row(buf, i);
    w.sw[r] = m.w;
    w.slo[r] = m.lo;
    w.shi[r] = m.hi;
    w.sswp[r] = m.swp;
    w.sord[r] = m.ord;
    w.spad[r] = m.pad;
  }
  __device__ size_t level_row(int ell, int slot) const { return (lane * g.L + ell) * (size_t)g.Bs + slot; }
  __device__ void put_level_meta(size_t row, const Meta& m) const {
    s.level_w[row] = m.w;
    s.level_p_lo[row] = m.lo;
    s.level_p_hi[row] = m.hi;
    s.level_sum_wp[row] = m.swp;
    s.level_order[row] = m.ord;
    s.pad_mask[row] = m.pad;
  }
};

template <typename T>
__device__ LaneCtx<T> make_ctx_at(const Geo& g, const logkv_state_t& s, const Work& w, int c, int grp, int b) {
  LaneCtx<T> x;
  x.g = g;
  x.s = s;
  x.w = w;
  x.c = c;
  x.grp = grp;
  x.b = b;
  x.bg = (size_t)x.b * g.G + x.grp;
  x.lane = x.bg * g.K + x.c;
  x.toff = w.plan_off[x.lane];
  x.scr = w.plan_scr[x.lane];
  x.base_order = w.plan_base[x.lane];
  x.arch = w.arch_idx + (size_t)x.b * g.NW;
  x.toks = w.tok_list + x.bg * g.NW;
  x.snapk = static_cast<const T*>(w.snap_k);
  x.snapv = static_cast<const T*>(w.snap_v);
  x.reck = static_cast<const T*>(s.recent_k_raw);
  x.recv = static_cast<const T*>(s.recent_v);
  return x;
}

// Lane of a (cluster, group, batch) grid.
template <typename T>
__device__ LaneCtx<T> make_ctx(const Geo& g, const logkv_state_t& s, const Work& w) {
  return make_ctx_at<T>(g, s, w, blockIdx.x, blockIdx.y, blockIdx.z);
}

// ---------------------------------------------------------------- cascade plan
// What every level of one lane does in this flush, from its counts and the lane's incoming row
// count: the sequential walk's control flow without touching a row.  In the steady state every
// level's merges read only that level's stored rows (level 0 also its incoming tokens), so the
// merges of all levels run at once (cascade_merge_kernel: carries of level l land in scratch
// buffer 1 as level l + 1's incoming rows) and then every level moves its survivors
// (cascade_move_kernel).  A level >= 1 whose merges would read incoming rows (carries of the
// level below) and the top level's fold need the levels in order: such lanes take the
// sequential walk.  The plan kernel writes the plan once per lane (the move kernel's CTAs update
// the level counts of their own levels, so the plan must not be recomputed from them).
enum LevelKind : int { kLvlNone = 0, kLvlFill = 1, kLvlMerge = 2, kLvlFold = 3 };
struct LevelPlan {
  int kind, cnt, m, npair, nsurv, in_off;  // in_off: the level's first incoming row in scratch buffer 1 (l >= 1)
};

// Returns 0 (no job), 1 (parallel kernels) or 2 (sequential walk).  One thread, from the lane's
// job type, incoming row count and level counts.
__device__ int plan_levels(const Geo& g, int type, int m0, const int* counts, LevelPlan* lp) {
  for (int l = 0; l < g.L; ++l) lp[l] = LevelPlan{kLvlNone, 0, 0, 0, 0, 0};
  if (type == kJobNone) return 0;
  int mode = 1, m = m0, off = 0;
  for (int l = 0; l < g.L && m > 0; ++l) {
    const int cnt = counts[l];
    LevelPlan p{kLvlFill, cnt, m, 0, cnt + m, off};
    int next = 0;
    if (cnt + m > g.Bs) {
      const int rem = cnt + m - g.Bs;
      if (l == g.L - 1) {
        p.kind = kLvlFold;
        mode = 2;
      } else {
        p.kind = kLvlMerge;
        p.npair = 2 * ((rem + 1) / 2);
        p.nsurv = cnt + m - p.npair;
        next = p.npair / 2;
        if (l > 0 && p.npair > cnt) mode = 2;
      }
    }
    lp[l] = p;
    if (l > 0) off += m;
    m = next;
  }
  return mode;
}

// The cascade plan of one lane, from the counts the cascade will start from (the prepare kernel
// clears new and delayed clusters), into the workspace.  One thread.
__device__ void write_lane_plan(const Geo& g, const logkv_state_t& s, const Work& w, size_t lane) {
  const int type = w.plan_type[lane];
  int counts[kMaxLevels];
  for (int l = 0; l < g.L; ++l)
    counts[l] = (type == kJobNew || type == kJobLate) ? 0 : s.level_count[lane * g.L + l];
  LevelPlan lp[kMaxLevels];
  w.lane_mode[lane] = plan_levels(g, type, w.plan_m0[lane], counts, lp);
  for (int l = 0; l < g.L; ++l) w.lane_plan[lane * g.L + l] = lp[l];
}

// ---------------------------------------------------------------- K6a: prepare
// Centroid and scalar updates of every cluster that receives tokens; new
// clusters and delayed (late) clusters are cleared, and a delayed cluster's
// entries plus its new tokens are staged in scratch buffer 0, stably sorted by
// p_lo with orders 0..n-1 (_alpha_commit_joins, log_kv_cache.py:3690-3788).
constexpr int kPrepRows = 64;  // token rows staged per pass of the centroid sum
constexpr int kPrepFeat = 4;   // features per thread of the centroid sum (D <= 1024, 256 threads)

template <typename T, int DC>
__global__ void __launch_bounds__(256) prepare_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  LaneCtx<T> x = make_ctx<T>(g, s, w);
  const int type = w.plan_type[x.lane];
  if (type == kJobNone) return;
  const int tid = threadIdx.x, nt = blockDim.x, D = DC ? DC : g.D;
  const int n = w.plan_n[x.lane];
  const float pre = s.n_eff[x.lane];
  float* mu = s.centroid + x.lane * D;
  extern __shared__ unsigned long long keys[];                       // [sort_cap] (delayed re-insert)
  int* srcs = reinterpret_cast<int*>(keys + g.sort_cap);             // [NW] token sources
  T* trows = reinterpret_cast<T*>(srcs + ((g.NW + 3) & ~3));         // [kPrepRows][D] staged token rows
  for (int i = tid; i < n; i += nt) srcs[i] = x.token_src(i);
  __syncthreads();
  // Centroid: per feature, a left-to-right sum over the lane's new tokens (a new cluster's
  // first token is kept apart, as the reference adds it after the others' sum).  Rows are
  // staged through shared memory kPrepRows at a time with 16-byte loads.
  constexpr int VN = Vec<T>::N;
  const int DV = D / VN;
  const int i0 = type == kJobNew ? 1 : 0;
  float sums[kPrepFeat];  // features tid, tid + nt, ... (D <= kPrepFeat * blockDim.x)
#pragma unroll
  for (int j = 0; j < kPrepFeat; ++j) sums[j] = 0.f;
  __shared__ const T* rowp[kPrepRows];  // source rows of the pass, resolved once per row
  for (int c0 = i0; c0 < n; c0 += kPrepRows) {
    const int cn = min(kPrepRows, n - c0);
    if (tid < cn) rowp[tid] = token_row<T>(g, x.snapk, x.reck, x.b, x.grp, srcs[c0 + tid]);
    __syncthreads();
    for (int item = tid; item < cn * DV; item += nt) {
      const int t = item / DV, v = item % DV;
      *reinterpret_cast<uint4*>(trows + t * D + v * VN) = *reinterpret_cast<const uint4*>(rowp[t] + v * VN);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kPrepFeat; ++j) {
      const int d = tid + j * nt;
      if (d < D) {
#pragma unroll 8
        for (int t = 0; t < cn; ++t) sums[j] = fadd(sums[j], Elem<T>::load(trows + t * D + d));
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < kPrepFeat; ++j) {
    const int d = tid + j * nt;
    if (d >= D) continue;
    if (type == kJobNew) {
      const float x0 = Elem<T>::load(token_row<T>(g, x.snapk, x.reck, x.b, x.grp, srcs[0]) + d);
      mu[d] = n == 1 ? x0 : fdiv(fadd(fmul(1.f, x0), sums[j]), fadd(1.f, (float)(n - 1)));
    } else {
      const float p = type == kJobOrdinary ? fmul(pre, 1.f) : pre;
      const float denom = fadd(p, (float)n);
      mu[d] = (type == kJobLate || p > 0.f) ? fdiv(fadd(fmul(p, mu[d]), sums[j]), denom) : fdiv(sums[j], (float)n);
    }
  }
  __shared__ int counts[kMaxLevels + 1];
  if (tid == 0) {
    int e = 0;
    for (int l = 0; l < g.L; ++l) {
      counts[l] = e;
      e += s.level_count[x.lane * g.L + l];
    }
    counts[g.L] = e;
  }
  __syncthreads();
  const int e = counts[g.L];
  const int64_t last_pos = token_position(g, s, w, x.b, x.token_src(n - 1));
  if (tid == 0) {
    if (type == kJobNew) {
      s.n_eff[x.lane] = n == 1 ? 1.f : fadd(1.f, (float)(n - 1));
      s.alive[x.lane] = 1;
      s.n_total[x.lane] = n;
      s.p_hi_c[x.lane] = last_pos;
      s.level0_phase[x.lane] = n;
    } else if (type == kJobOrdinary) {
      s.n_eff[x.lane] = fadd(fmul(pre, 1.f), (float)n);
      s.n_total[x.lane] += n;
      s.p_hi_c[x.lane] = last_pos;
      s.level0_phase[x.lane] += n;
    } else {
      s.n_eff[x.lane] = fadd(pre, (float)n);
      s.n_total[x.lane] += n;
      s.p_hi_c[x.lane] = max(s.p_hi_c[x.lane], last_pos);
      s.level0_phase[x.lane] = e + n;
      s.alive[x.lane] = 1;
    }
  }
  if (type == kJobOrdinary) return;
  if (type == kJobLate) {
    const int total = e + n;
    const int cap = g.sort_cap;
    for (int i = tid; i < cap; i += nt) {
      unsigned long long key = ~0ull;
      if (i < e) {
        int l = 0;
        while (l + 1 < g.L && counts[l + 1] <= i) ++l;
        const int64_t lo = s.level_p_lo[x.level_row(l, i - counts[l])];
        key = ((unsigned long long)lo << 14) | (unsigned long long)i;
      } else if (i < total) {
        const int64_t p = token_position(g, s, w, x.b, x.token_src(i - e));
        key = ((unsigned long long)p << 14) | (unsigned long long)i;
      }
      keys[i] = key;
    }
    __syncthreads();
    for (int k = 2; k <= cap; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < cap; i += nt) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const unsigned long long a = keys[i], bb = keys[ixj];
            const bool up = (i & k) == 0;
            if ((a > bb) == up) {
              keys[i] = bb;
              keys[ixj] = a;
            }
          }
        }
        __syncthreads();
      }
    }
    T* sk = static_cast<T*>(w.sk);
    T* sv = static_cast<T*>(w.sv);
    for (int item = tid; item < total * DV; item += nt) {
      const int r = item / DV, d = (item % DV) * VN;
      const int idx = (int)(keys[r] & 0x3FFFull);
      const size_t dst = x.scr_row(0, r) * D + d;
      const T *pk, *pv;
      if (idx < e) {
        int l = 0;
        while (l + 1 < g.L && counts[l + 1] <= idx) ++l;
        const size_t src = x.level_row(l, idx - counts[l]) * D + d;
        pk = static_cast<const T*>(s.level_k) + src;
        pv = static_cast<const T*>(s.level_v) + src;
      } else {
        const int src = srcs[idx - e];
        pk = token_row<T>(g, x.snapk, x.reck, x.b, x.grp, src) + d;
        pv = token_row<T>(g, x.snapv, x.recv, x.b, x.grp, src) + d;
      }
      *reinterpret_cast<uint4*>(sk + dst) = *reinterpret_cast<const uint4*>(pk);
      *reinterpret_cast<uint4*>(sv + dst) = *reinterpret_cast<const uint4*>(pv);
    }
    for (int r = tid; r < total; r += nt) {
      const int idx = (int)(keys[r] & 0x3FFFull);
      Meta m;
      if (idx < e) {
        int l = 0;
        while (l + 1 < g.L && counts[l + 1] <= idx) ++l;
        const size_t src = x.level_row(l, idx - counts[l]);
        m.w = s.level_w[src];
        m.lo = s.level_p_lo[src];
        m.hi = s.level_p_hi[src];
        m.swp = s.level_sum_wp[src];
        m.pad = s.pad_mask[src];
      } else {
        const int64_t p = token_position(g, s, w, x.b, x.token_src(idx - e));
        m.w = 1.f;
        m.lo = m.hi = m.swp = p;
        m.pad = 0;
      }
      m.ord = r;
      x.put_scratch(0, r, m);
    }
    __syncthreads();
  }
  // Clear every level of the lane (new clusters and delayed re-inserts).
  const size_t rows = (size_t)g.L * g.Bs;
  uint4* lk = reinterpret_cast<uint4*>(static_cast<T*>(s.level_k) + x.level_row(0, 0) * D);
  uint4* lv = reinterpret_cast<uint4*>(static_cast<T*>(s.level_v) + x.level_row(0, 0) * D);
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  for (size_t i = tid; i < rows * DV; i += nt) {
    lk[i] = zero;
    lv[i] = zero;
  }
  for (size_t r = tid; r < rows; r += nt) {
    const size_t row = x.level_row(0, 0) + r;
    s.level_w[row] = 0.f;
    s.level_p_lo[row] = 0;
    s.level_p_hi[row] = 0;
    s.level_sum_wp[row] = 0;
    s.level_order[row] = 0;
    s.pad_mask[row] = 0;
  }
  for (int l = tid; l < g.L; l += nt) s.level_count[x.lane * g.L + l] = 0;
  if (tid == 0) {
    atomicAdd(&w.counters[kCntClear], (unsigned long long)rows);
    if (type == kJobLate) atomicAdd(&w.counters[kCntGather], (unsigned long long)(e + n));
  }
}


}  // namespace logkv
