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
__device__ LaneCtx<T> make_ctx(const Geo& g, const logkv_state_t& s, const Work& w) {
  LaneCtx<T> x;
  x.g = g;
  x.s = s;
  x.w = w;
  x.c = blockIdx.x;
  x.grp = blockIdx.y;
  x.b = blockIdx.z;
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

// ---------------------------------------------------------------- K6a: prepare
// Centroid and scalar updates of every cluster that receives tokens; new
// clusters and delayed (late) clusters are cleared, and a delayed cluster's
// entries plus its new tokens are staged in scratch buffer 0, stably sorted by
// p_lo with orders 0..n-1 (_alpha_commit_joins, log_kv_cache.py:3690-3788).
template <typename T>
__global__ void __launch_bounds__(256) prepare_kernel(Geo g, logkv_state_t s, Work w) {
  LaneCtx<T> x = make_ctx<T>(g, s, w);
  const int type = w.plan_type[x.lane];
  if (type == kJobNone) return;
  const int tid = threadIdx.x, nt = blockDim.x, D = g.D;
  const int n = w.plan_n[x.lane];
  const float pre = s.n_eff[x.lane];
  float* mu = s.centroid + x.lane * D;
  for (int d = tid; d < D; d += nt) {
    if (type == kJobNew) {
      const float x0 = Elem<T>::load(token_row<T>(g, x.snapk, x.reck, x.b, x.grp, x.token_src(0)) + d);
      if (n == 1) {
        mu[d] = x0;
      } else {
        float sums = 0.f;
        for (int i = 1; i < n; ++i)
          sums = fadd(sums, Elem<T>::load(token_row<T>(g, x.snapk, x.reck, x.b, x.grp, x.token_src(i)) + d));
        mu[d] = fdiv(fadd(fmul(1.f, x0), sums), fadd(1.f, (float)(n - 1)));
      }
    } else {
      float sums = 0.f;
      for (int i = 0; i < n; ++i)
        sums = fadd(sums, Elem<T>::load(token_row<T>(g, x.snapk, x.reck, x.b, x.grp, x.token_src(i)) + d));
      const float p = type == kJobOrdinary ? fmul(pre, 1.f) : pre;
      const float denom = fadd(p, (float)n);
      mu[d] = (type == kJobLate || p > 0.f) ? fdiv(fadd(fmul(p, mu[d]), sums), denom) : fdiv(sums, (float)n);
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
    extern __shared__ unsigned long long keys[];  // [sort_cap]
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
    for (int item = tid; item < total * D; item += nt) {
      const int r = item / D, d = item % D;
      const int idx = (int)(keys[r] & 0x3FFFull);
      const size_t dst = x.scr_row(0, r) * D + d;
      if (idx < e) {
        int l = 0;
        while (l + 1 < g.L && counts[l + 1] <= idx) ++l;
        const size_t src = x.level_row(l, idx - counts[l]) * D + d;
        sk[dst] = static_cast<const T*>(s.level_k)[src];
        sv[dst] = static_cast<const T*>(s.level_v)[src];
      } else {
        const int src = x.token_src(idx - e);
        sk[dst] = token_row<T>(g, x.snapk, x.reck, x.b, x.grp, src)[d];
        sv[dst] = token_row<T>(g, x.snapv, x.recv, x.b, x.grp, src)[d];
      }
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
  T* lk = static_cast<T*>(s.level_k) + x.level_row(0, 0) * D;
  T* lv = static_cast<T*>(s.level_v) + x.level_row(0, 0) * D;
  for (size_t i = tid; i < rows * D; i += nt) {
    lk[i] = Elem<T>::zero();
    lv[i] = Elem<T>::zero();
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

// ---------------------------------------------------------------- K6b: cascade
constexpr int kBetaChunk = 64;  // Beta groups evaluated per pass

template <typename T, bool BETA>
__global__ void __launch_bounds__(256) cascade_kernel(Geo g, logkv_state_t s, Work w) {
  LaneCtx<T> x = make_ctx<T>(g, s, w);
  const int type = w.plan_type[x.lane];
  if (type == kJobNone) return;
  const int tid = threadIdx.x, nt = blockDim.x, D = g.D, Bs = g.Bs;
  extern __shared__ unsigned char smraw[];
  T* lk = reinterpret_cast<T*>(smraw);                       // [Bs*D]
  T* lv = lk + (size_t)Bs * D;                               // [Bs*D]
  Meta* lm = reinterpret_cast<Meta*>(lv + (size_t)Bs * D);   // [Bs] (aligned below by host padding)
  __shared__ float bloss[kBetaChunk][12];
  __shared__ float bener[kBetaChunk][2];
  __shared__ int bcut[kBetaChunk];
  T* LK = static_cast<T*>(s.level_k);
  T* LV = static_cast<T*>(s.level_v);
  T* SK = static_cast<T*>(w.sk);
  T* SV = static_cast<T*>(w.sv);
  Stage st;
  st.kind = type == kJobLate ? 1 : 0;
  st.buf = 0;
  st.m = w.plan_m0[x.lane];
  int nb = 1;
  for (int ell = 0; ell < g.L; ++ell) {
    const int m = st.m;
    if (m == 0) break;
    const int cnt = s.level_count[x.lane * g.L + ell];
    if (cnt + m <= Bs) {
      for (int item = tid; item < m * D; item += nt) {
        const int i = item / D, d = item % D;
        const size_t row = x.level_row(ell, cnt + i);
        LK[row * D + d] = x.stage_k(st, i)[d];
        LV[row * D + d] = x.stage_v(st, i)[d];
      }
      for (int i = tid; i < m; i += nt) x.put_level_meta(x.level_row(ell, cnt + i), x.stage_meta(st, i));
      if (tid == 0) {
        s.level_count[x.lane * g.L + ell] = (int16_t)(cnt + m);
        atomicAdd(&w.counters[kCntStageRead], (unsigned long long)m);
        atomicAdd(&w.counters[kCntFill], (unsigned long long)m);
      }
      break;
    }
    // Overflow: stage the stored rows, then rewrite the whole level.
    const size_t lrow0 = x.level_row(ell, 0);
    for (int item = tid; item < cnt * D; item += nt) {
      lk[item] = LK[lrow0 * D + item];
      lv[item] = LV[lrow0 * D + item];
    }
    for (int i = tid; i < cnt; i += nt) {
      const size_t row = lrow0 + i;
      lm[i] = Meta{s.level_w[row], s.level_p_lo[row], s.level_p_hi[row], s.level_sum_wp[row], s.level_order[row],
                   s.pad_mask[row]};
    }
    __syncthreads();
    auto pool_k = [&](int p, int d) -> T { return p < cnt ? lk[p * D + d] : x.stage_k(st, p - cnt)[d]; };
    auto pool_v = [&](int p, int d) -> T { return p < cnt ? lv[p * D + d] : x.stage_v(st, p - cnt)[d]; };
    auto pool_m = [&](int p) -> Meta { return p < cnt ? lm[p] : x.stage_meta(st, p - cnt); };
    const int rem = cnt + m - Bs;
    if (ell == g.L - 1) {
      // Top level: slot 0 = left fold of pool[0..rem], rounded after every step.
      for (int d = tid; d < D; d += nt) {
        const T t0k = pool_k(0, d), t0v = pool_v(0, d);
        float ak = Elem<T>::load(&t0k);
        float av = Elem<T>::load(&t0v);
        float aw = pool_m(0).w;
        for (int t = 1; t <= rem; ++t) {
          const float bw = pool_m(t).w;
          const float alpha = fdiv(aw, fmaxf(fadd(aw, bw), 1e-8f));
          const float beta = fsub(1.f, alpha);
          T tk = pool_k(t, d), tv = pool_v(t, d);
          ak = Elem<T>::round(fadd(fmul(alpha, ak), fmul(beta, Elem<T>::load(&tk))));
          av = Elem<T>::round(fadd(fmul(alpha, av), fmul(beta, Elem<T>::load(&tv))));
          aw = fadd(aw, bw);
        }
        Elem<T>::store(&LK[lrow0 * D + d], ak);
        Elem<T>::store(&LV[lrow0 * D + d], av);
      }
      if (tid == 0) {
        Meta acc = pool_m(0);
        for (int t = 1; t <= rem; ++t) acc = merge_meta(acc, pool_m(t));
        x.put_level_meta(lrow0, acc);
        s.level_count[x.lane * g.L + ell] = (int16_t)Bs;
        atomicAdd(&w.counters[kCntStorageRead], (unsigned long long)cnt);
        atomicAdd(&w.counters[kCntStageRead], (unsigned long long)m);
        atomicAdd(&w.counters[kCntSurvivor], (unsigned long long)Bs);
      }
      for (int item = tid; item < (Bs - 1) * D; item += nt) {
        const int slot = 1 + item / D, d = item % D;
        LK[(lrow0 + slot) * D + d] = pool_k(rem + slot, d);
        LV[(lrow0 + slot) * D + d] = pool_v(rem + slot, d);
      }
      for (int slot = 1 + tid; slot < Bs; slot += nt) x.put_level_meta(lrow0 + slot, pool_m(rem + slot));
      break;
    }
    const int npair = 2 * ((rem + 1) / 2);
    const int ncarry = npair / 2;
    const int nsurv = cnt + m - npair;
    if (!BETA) {
      for (int item = tid; item < ncarry * D; item += nt) {
        const int j = item / D, d = item % D;
        const float wa = pool_m(2 * j).w, wb = pool_m(2 * j + 1).w;
        const float alpha = fdiv(wa, fmaxf(fadd(wa, wb), 1e-8f));
        const float beta = fsub(1.f, alpha);
        T ka = pool_k(2 * j, d), kb = pool_k(2 * j + 1, d);
        T va = pool_v(2 * j, d), vb = pool_v(2 * j + 1, d);
        const size_t dst = x.scr_row(nb, j) * D + d;
        Elem<T>::store(&SK[dst], fadd(fmul(alpha, Elem<T>::load(&ka)), fmul(beta, Elem<T>::load(&kb))));
        Elem<T>::store(&SV[dst], fadd(fmul(alpha, Elem<T>::load(&va)), fmul(beta, Elem<T>::load(&vb))));
      }
      for (int j = tid; j < ncarry; j += nt) x.put_scratch(nb, j, merge_meta(pool_m(2 * j), pool_m(2 * j + 1)));
    } else {
      const int ngroups = (npair + 3) / 4;
      for (int q0 = 0; q0 < ngroups; q0 += kBetaChunk) {
        const int qn = min(kBetaChunk, ngroups - q0);
        // 14 sequential reductions per group: 12 (component, cut, side) losses, 2 energies.
        for (int item = tid; item < qn * 14; item += nt) {
          const int q = item / 14, k = item % 14;
          const int start = 4 * (q0 + q);
          const int width = min(4, npair - start);
          if (width != 4) continue;
          float wv[4];
          for (int i = 0; i < 4; ++i) wv[i] = pool_m(start + i).w;
          const int comp = k < 12 ? k / 6 : k - 12;
          if (k >= 12) {
            float e[4] = {0.f, 0.f, 0.f, 0.f};
            for (int d = 0; d < D; ++d)
              for (int i = 0; i < 4; ++i) {
                T t = comp == 0 ? pool_k(start + i, d) : pool_v(start + i, d);
                const float xv = Elem<T>::load(&t);
                e[i] = fadd(e[i], fmul(xv, xv));
              }
            float tot = 0.f, acc = 0.f;
            for (int i = 0; i < 4; ++i) tot = fadd(tot, wv[i]);
            tot = fmaxf(tot, 1e-12f);
            for (int i = 0; i < 4; ++i) acc = fadd(acc, fmul(e[i], wv[i]));
            bener[q][comp] = fmaxf(fdiv(acc, tot), 1e-12f);
          } else {
            const int j = (k % 6) / 2, side = k % 2;
            const int cut = j == 0 ? 2 : (j == 1 ? 1 : 3);
            float om[4];
            float wsum = 0.f;
            for (int i = 0; i < 4; ++i) {
              const bool in = side == 0 ? (i < cut) : (i >= cut);
              om[i] = fmul(wv[i], in ? 1.f : 0.f);
              wsum = fadd(wsum, om[i]);
            }
            const float den = fmaxf(wsum, 1e-12f);
            float r[4] = {0.f, 0.f, 0.f, 0.f};
            for (int d = 0; d < D; ++d) {
              float xv[4];
              float sacc = 0.f;
              for (int i = 0; i < 4; ++i) {
                T t = comp == 0 ? pool_k(start + i, d) : pool_v(start + i, d);
                xv[i] = Elem<T>::load(&t);
                sacc = fadd(sacc, fmul(xv[i], om[i]));
              }
              const float mean = fdiv(sacc, den);
              for (int i = 0; i < 4; ++i) {
                const float df = fsub(xv[i], mean);
                r[i] = fadd(r[i], fmul(df, df));
              }
            }
            float loss = 0.f;
            for (int i = 0; i < 4; ++i) loss = fadd(loss, fmul(r[i], om[i]));
            bloss[q][k] = loss;
          }
        }
        __syncthreads();
        for (int q = tid; q < qn; q += nt) {
          const int start = 4 * (q0 + q);
          const int width = min(4, npair - start);
          if (width != 4) {
            bcut[q] = 1;
            continue;
          }
          float costs[3] = {0.f, 0.f, 0.f};
          for (int comp = 0; comp < 2; ++comp)
            for (int j = 0; j < 3; ++j)
              for (int side = 0; side < 2; ++side)
                costs[j] = fadd(costs[j], fdiv(bloss[q][comp * 6 + j * 2 + side], bener[q][comp]));
          int best = 0;
          if (costs[1] < costs[best]) best = 1;
          if (costs[2] < costs[best]) best = 2;
          bcut[q] = best == 0 ? 2 : (best == 1 ? 1 : 3);
        }
        __syncthreads();
        // Apply: per output side, sum(w*x) over member rows in row order / max(mass, 1e-12).
        for (int item = tid; item < qn * 2 * D; item += nt) {
          const int q = item / (2 * D), side = (item / D) % 2, d = item % D;
          const int start = 4 * (q0 + q);
          const int width = min(4, npair - start);
          if (side == 1 && width != 4) continue;
          const int cut = bcut[q];
          float ks = 0.f, vs = 0.f, mass = 0.f;
          for (int i = 0; i < 4; ++i) {
            const bool valid = i < width;
            const bool in = valid && (width == 2 ? side == 0 : (side == 0 ? i < cut : i >= cut));
            const float wi = valid ? pool_m(start + i).w : 0.f;
            const float om = fmul(wi, in ? 1.f : 0.f);
            float kx = 0.f, vx = 0.f;
            if (valid) {
              T tk = pool_k(start + i, d), tv = pool_v(start + i, d);
              kx = Elem<T>::load(&tk);
              vx = Elem<T>::load(&tv);
            }
            mass = fadd(mass, om);
            ks = fadd(ks, fmul(kx, om));
            vs = fadd(vs, fmul(vx, om));
          }
          const float den = fmaxf(mass, 1e-12f);
          const size_t dst = x.scr_row(nb, start / 2 + side) * D + d;
          Elem<T>::store(&SK[dst], fdiv(ks, den));
          Elem<T>::store(&SV[dst], fdiv(vs, den));
        }
        for (int item = tid; item < qn * 2; item += nt) {
          const int q = item / 2, side = item % 2;
          const int start = 4 * (q0 + q);
          const int width = min(4, npair - start);
          if (side == 1 && width != 4) continue;
          const int cut = bcut[q];
          Meta o;
          float mass = 0.f;
          int64_t lo = INT64_MAX, hi = INT64_MIN, swp = 0, ord = INT64_MAX;
          uint8_t pad = 1;
          for (int i = 0; i < width; ++i) {
            const bool in = width == 2 ? side == 0 : (side == 0 ? i < cut : i >= cut);
            const Meta r = pool_m(start + i);
            mass = fadd(mass, fmul(r.w, in ? 1.f : 0.f));
            if (!in) continue;
            if (r.w > 0.f) {
              lo = min(lo, r.lo);
              hi = max(hi, r.hi);
            }
            swp += r.swp;
            ord = min(ord, r.ord);
            pad &= r.pad;
          }
          o.w = mass;
          o.lo = mass > 0.f ? lo : 0;
          o.hi = mass > 0.f ? hi : 0;
          o.swp = swp;
          o.ord = ord;
          o.pad = pad;
          x.put_scratch(nb, start / 2 + side, o);
        }
        __syncthreads();
      }
    }
    // Survivors shift to the front, tail slots are zeroed.
    for (int item = tid; item < Bs * D; item += nt) {
      const int slot = item / D, d = item % D;
      const size_t dst = (lrow0 + slot) * D + d;
      if (slot < nsurv) {
        LK[dst] = pool_k(npair + slot, d);
        LV[dst] = pool_v(npair + slot, d);
      } else {
        LK[dst] = Elem<T>::zero();
        LV[dst] = Elem<T>::zero();
      }
    }
    for (int slot = tid; slot < Bs; slot += nt) {
      if (slot < nsurv) {
        x.put_level_meta(lrow0 + slot, pool_m(npair + slot));
      } else {
        x.put_level_meta(lrow0 + slot, Meta{0.f, 0, 0, 0, 0, 0});
      }
    }
    if (tid == 0) {
      s.level_count[x.lane * g.L + ell] = (int16_t)nsurv;
      atomicAdd(&w.counters[kCntStorageRead], (unsigned long long)cnt);
      atomicAdd(&w.counters[kCntStageRead], (unsigned long long)m);
      atomicAdd(&w.counters[kCntSurvivor], (unsigned long long)nsurv);
      atomicAdd(&w.counters[kCntClear], (unsigned long long)(Bs - nsurv));
      atomicAdd(&w.counters[kCntCarry], (unsigned long long)ncarry);
    }
    __syncthreads();
    st.kind = 1;
    st.buf = nb;
    st.m = ncarry;
    nb = 1 - nb;
  }
}

}  // namespace logkv
