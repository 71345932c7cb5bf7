// Attach route on the device: frozen-centroid decisions, farthest-point seeding
// and the per-cluster commit plan.
//
// Follows _semantic_attach_decide / _semantic_attach_plan_torch
// (litgpt/log_kv_cache.py:4597-4680), _semantic_existing_assignments
// (:2649-2681) and the grouping of _semantic_attach_commit (:4682-4707) with
// the ordinary/delayed split of _alpha_commit_joins (:3690-3788).
#pragma once

#include "flush_common.cuh"

namespace logkv {

// ---------------------------------------------------------------- K4: attach decisions
// One thread per archived token (position rank); the block stages its 128
// token rows and the lane's centres in shared memory.  Every feature sum runs
// left to right in one thread.
template <typename T>
__global__ void __launch_bounds__(128) attach_kernel(Geo g, logkv_state_t s, Work w) {
  const int b = blockIdx.z, grp = blockIdx.y, tid = threadIdx.x;
  const int D = g.D, K = g.K;
  const int na = w.narch[b];
  const int r0 = blockIdx.x * 128;
  if (r0 >= na) return;
  extern __shared__ float sm[];
  float* mu = sm;            // [K][D]
  float* xs = mu + K * D;    // [128][D + 1]
  __shared__ float mm[kMaxClusters];
  __shared__ long long phi[kMaxClusters];
  __shared__ int alv[kMaxClusters];
  const size_t lane0 = ((size_t)b * g.G + grp) * K;
  for (int i = tid; i < K * D; i += blockDim.x) mu[i] = s.centroid[lane0 * D + i];
  if (tid < K) {
    alv[tid] = s.alive[lane0 + tid] != 0;
    phi[tid] = s.p_hi_c[lane0 + tid];
  }
  __syncthreads();
  if (tid < K) {
    float a = 0.f;
    for (int d = 0; d < D; ++d) a = fadd(a, fmul(mu[tid * D + d], mu[tid * D + d]));
    mm[tid] = a;
  }
  const T* snap = static_cast<const T*>(w.snap_k);
  const T* rec = static_cast<const T*>(s.recent_k_raw);
  const int* arch = w.arch_idx + (size_t)b * g.NW;
  const int nrow = min(128, na - r0);
  constexpr int VN = Vec<T>::N;
  const int DV = D / VN;
  for (int item = tid; item < nrow * DV; item += blockDim.x) {
    const int row = item / DV, v = item % DV;
    float xv[VN];
    unpack(*reinterpret_cast<const uint4*>(token_row<T>(g, snap, rec, b, grp, arch[r0 + row]) + v * VN), xv,
           (const T*)nullptr);
#pragma unroll
    for (int e = 0; e < VN; ++e) xs[row * (D + 1) + v * VN + e] = xv[e];
  }
  __syncthreads();
  if (tid >= nrow) return;
  const int r = r0 + tid;
  const int64_t pos = token_position(g, s, w, b, arch[r]);
  const float* x = xs + tid * (D + 1);
  float xx = 0.f;
  for (int d = 0; d < D; ++d) xx = fadd(xx, fmul(x[d], x[d]));
  const float thresh = fmul(g.lam, s.s_h[(size_t)b * g.G + grp]);
  float best_cost = INFINITY, s_win = 0.f, best_ex = INFINITY, sem0 = 0.f;
  int winner = 0, nearest = 0;
  bool any_alive = false;
  // Clusters in blocks of 16: 32 independent left-to-right accumulations per feature.
  constexpr int CB = 16;
  for (int cb = 0; cb < K; cb += CB) {
    float dot[CB], ex[CB];
#pragma unroll
    for (int j = 0; j < CB; ++j) dot[j] = ex[j] = 0.f;
    const int nc = min(CB, K - cb);
    for (int d = 0; d < D; ++d) {
      const float xd = x[d];
#pragma unroll
      for (int j = 0; j < CB; ++j) {
        if (j < nc) {
          const float m = mu[(cb + j) * D + d];
          dot[j] = fadd(dot[j], fmul(xd, m));
          const float df = fsub(xd, m);
          ex[j] = fadd(ex[j], fmul(df, df));
        }
      }
    }
#pragma unroll
    for (int j = 0; j < CB; ++j) {
      if (j >= nc) continue;
      const int c = cb + j;
      const float sem = fmaxf(fsub(fadd(xx, mm[c]), fmul(2.f, dot[j])), 0.f);
      if (c == 0) sem0 = sem;
      if (!alv[c]) continue;
      any_alive = true;
      const float gap = fmaxf((float)(pos - (int64_t)phi[c]), 0.f);
      const float cost = fadd(sem, fmul(g.eta, fdiv(gap, fadd(gap, g.g0))));
      if (cost < best_cost) {
        best_cost = cost;
        winner = c;
        s_win = sem;
      }
      const float dist = __fsqrt_rn(ex[j]);
      if (dist < best_ex) {
        best_ex = dist;
        nearest = c;
      }
    }
  }
  if (!any_alive) {
    winner = 0;
    s_win = sem0;
    nearest = 0;
  }
  const bool direct = any_alive && s_win <= thresh;
  const size_t o = ((size_t)b * g.G + grp) * g.NW + r;
  w.assign[o] = (int8_t)(direct ? winner : nearest);
  w.orphan[o] = direct ? 0 : 1;
  w.s_winner[o] = s_win;
}

// (value, index) argmax with the lowest index winning ties.
struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax argmax_better(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}
__device__ ArgMax block_argmax(ArgMax v, ArgMax* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    ArgMax o;
    o.v = __shfl_xor_sync(0xffffffffu, v.v, off);
    o.i = __shfl_xor_sync(0xffffffffu, v.i, off);
    v = argmax_better(v, o);
  }
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    ArgMax best = sh[0];
    for (int k = 1; k < nwarps; ++k) best = argmax_better(best, sh[k]);
    sh[0] = best;
  }
  __syncthreads();
  ArgMax out = sh[0];
  __syncthreads();
  return out;
}

// Left-to-right squared distance between a storage row (read 16 bytes at a time) and a float row.
template <typename T>
__device__ __forceinline__ float sq_dist_rows(const T* a, const float* b, int D) {
  constexpr int VN = Vec<T>::N;
  float acc = 0.f;
#pragma unroll 4
  for (int v = 0; v < D / VN; ++v) {
    float xa[VN];
    unpack(*reinterpret_cast<const uint4*>(a + v * VN), xa, (const T*)nullptr);
#pragma unroll
    for (int e = 0; e < VN; ++e) {
      const float df = fsub(xa[e], b[v * VN + e]);
      acc = fadd(acc, fmul(df, df));
    }
  }
  return acc;
}

// ---------------------------------------------------------------- K5: seeding + commit plan
// One block per (batch, group) lane.  Seeds: up to min(free slots, orphans)
// farthest-point picks among orphans; orphans then join the nearest live or
// seeded cluster.  Then a stable counting sort groups the archived tokens by
// cluster and each cluster's job (ordinary, new, delayed) and scratch range
// are planned.
template <typename T>
__global__ void __launch_bounds__(1024) plan_kernel(Geo g, logkv_state_t s, Work w) {
  const int b = blockIdx.y, grp = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const int D = g.D, K = g.K;
  const int na = w.narch[b];
  const size_t lane0 = ((size_t)b * g.G + grp) * K;
  const size_t row0 = ((size_t)b * g.G + grp) * g.NW;
  int8_t* asg = w.assign + row0;
  const uint8_t* orph = w.orphan + row0;
  const int* arch = w.arch_idx + (size_t)b * g.NW;
  const T* snap = static_cast<const T*>(w.snap_k);
  const T* rec = static_cast<const T*>(s.recent_k_raw);
  extern __shared__ float dist[];  // [NW]
  __shared__ ArgMax red[32];
  __shared__ int wsum[32];
  __shared__ int free_slots[kMaxClusters];
  __shared__ int picks[kMaxClusters];
  __shared__ int sh_nfree, sh_norph;
  __shared__ float prow[1024];  // pick row (D <= 1024)
  if (tid == 0) {
    int nf = 0;
    for (int c = 0; c < K; ++c)
      if (!s.alive[lane0 + c]) free_slots[nf++] = c;
    sh_nfree = nf;
    sh_norph = 0;
  }
  __syncthreads();
  int my_orph = 0;
  for (int t = tid; t < na; t += nt) my_orph += orph[t];
  atomicAdd(&sh_norph, my_orph);
  __syncthreads();
  const int n_use = min(sh_nfree, sh_norph);
  if (n_use > 0) {
    ArgMax a{-INFINITY, 0x7fffffff};
    for (int t = tid; t < na; t += nt) a = argmax_better(a, ArgMax{orph[t] ? w.s_winner[row0 + t] : -INFINITY, t});
    ArgMax best = block_argmax(a, red);
    int nxt = best.i;
    if (tid == 0) picks[0] = nxt;
    for (int d = tid; d < D; d += nt) prow[d] = Elem<T>::load(token_row<T>(g, snap, rec, b, grp, arch[nxt]) + d);
    __syncthreads();
    for (int t = tid; t < na; t += nt)
      dist[t] = orph[t] ? sq_dist_rows<T>(token_row<T>(g, snap, rec, b, grp, arch[t]), prow, D) : -INFINITY;
    __syncthreads();
    for (int i = 1; i < n_use; ++i) {
      if (tid == 0) dist[nxt] = -INFINITY;
      __syncthreads();
      ArgMax m{-INFINITY, 0x7fffffff};
      for (int t = tid; t < na; t += nt) m = argmax_better(m, ArgMax{dist[t], t});
      nxt = block_argmax(m, red).i;
      if (tid == 0) picks[i] = nxt;
      for (int d = tid; d < D; d += nt) prow[d] = Elem<T>::load(token_row<T>(g, snap, rec, b, grp, arch[nxt]) + d);
      __syncthreads();
      for (int t = tid; t < na; t += nt) {
        const float cur = dist[t];
        const float nd = sq_dist_rows<T>(token_row<T>(g, snap, rec, b, grp, arch[t]), prow, D);
        dist[t] = fminf(cur, nd);
      }
      __syncthreads();
    }
    // Orphans join the nearest live or seeded cluster (exact distance, lowest id on ties).
    // Candidate centres (live centroids, seed tokens for the opened slots) staged as float32.
    float* mus = dist + ((g.NW + 3) & ~3);  // [K][D]
    __shared__ int cand[kMaxClusters];
    if (tid < K) cand[tid] = s.alive[lane0 + tid] != 0;
    __syncthreads();
    for (int i = tid; i < K * D; i += nt) mus[i] = s.centroid[lane0 * D + i];
    __syncthreads();
    for (int i = 0; i < n_use; ++i) {
      const int c = free_slots[i];
      if (tid == 0) cand[c] = 1;
      for (int d = tid; d < D; d += nt)
        mus[c * D + d] = Elem<T>::load(token_row<T>(g, snap, rec, b, grp, arch[picks[i]]) + d);
    }
    __syncthreads();
    for (int t = tid; t < na; t += nt) {
      if (!orph[t]) continue;
      const T* x = token_row<T>(g, snap, rec, b, grp, arch[t]);
      float best_d = INFINITY;
      int best_c = 0;
      for (int c = 0; c < K; ++c) {
        if (!cand[c]) continue;
        const float dd = __fsqrt_rn(sq_dist_rows<T>(x, mus + c * D, D));
        if (dd < best_d) {
          best_d = dd;
          best_c = c;
        }
      }
      asg[t] = (int8_t)best_c;
    }
    __syncthreads();
    if (tid == 0)
      for (int i = 0; i < n_use; ++i) asg[picks[i]] = (int8_t)free_slots[i];
    __syncthreads();
  }
  // Stable counting sort of archive ranks by cluster.
  __shared__ int cl_count[kMaxClusters], cl_off[kMaxClusters];
  __shared__ int tot;
  int running = 0;
  for (int c = 0; c < K; ++c) {
    int carry = 0;
    for (int base = 0; base < na; base += nt) {
      const int t = base + tid;
      const int f = (t < na && asg[t] == c) ? 1 : 0;
      const int incl = block_inclusive_scan(f, wsum);
      if (f) w.tok_list[row0 + running + carry + incl - 1] = t;
      if (tid == nt - 1) tot = incl;
      __syncthreads();
      carry += tot;
      __syncthreads();
    }
    if (tid == 0) {
      cl_count[c] = carry;
      cl_off[c] = running;
    }
    running += carry;
  }
  __syncthreads();
  if (tid == 0) {
    int scr = 0;
    for (int c = 0; c < K; ++c) {
      const size_t lane = lane0 + c;
      const int n = cl_count[c];
      int type = kJobNone, m0 = 0;
      int64_t base_order = 0;
      if (n > 0) {
        if (!s.alive[lane]) {
          type = kJobNew;
          m0 = n;
        } else {
          const int64_t first_pos = token_position(g, s, w, b, arch[w.tok_list[row0 + cl_off[c]]]);
          if (first_pos < s.p_hi_c[lane]) {
            int e = 0;
            for (int l = 0; l < g.L; ++l) e += s.level_count[lane * g.L + l];
            type = kJobLate;
            m0 = e + n;
          } else {
            type = kJobOrdinary;
            m0 = n;
            base_order = s.level0_phase[lane];
          }
        }
      }
      w.plan_off[lane] = cl_off[c];
      w.plan_n[lane] = n;
      w.plan_type[lane] = type;
      w.plan_m0[lane] = m0;
      w.plan_scr[lane] = scr;
      w.plan_base[lane] = base_order;
      if (type != kJobNone) scr += m0 + 2;
    }
    if (scr > g.S) set_status(w.status, kStatusCarryOverflow);
  }
}

}  // namespace logkv
