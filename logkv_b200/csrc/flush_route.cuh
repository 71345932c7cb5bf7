// Attach route on the device: frozen-centroid decisions, farthest-point seeding
// and the per-cluster commit plan.
//
// Follows _semantic_attach_decide / _semantic_attach_plan_torch
// (litgpt/log_kv_cache.py:4597-4680), _semantic_existing_assignments
// (:2649-2681) and the grouping of _semantic_attach_commit (:4682-4707) with
// the ordinary/delayed split of _alpha_commit_joins (:3690-3788).
#pragma once

#include <cooperative_groups.h>

#include "flush_common.cuh"

namespace logkv {

// ---------------------------------------------------------------- K4: attach decisions
// Decisions for every token of the [old pool | flushed window] index space (the archive
// is a subset, picked later by the span choice; decisions depend only on the frozen
// cluster state).  One thread per (token, cluster): each computes the token's dot
// product and exact squared distance to one centre, left to right over the features;
// one thread per token then walks the clusters in index order for the decision
// (first-index argmin, as torch.argmin).  Token rows and centres are staged in shared
// memory with an odd word stride (conflict-free).  Outputs are indexed by token.
template <typename T>
__device__ void attach_body(const Geo& g, const logkv_state_t& s, const Work& w, int blk) {
  const int b = blockIdx.z, grp = blockIdx.y, tid = threadIdx.x;
  const int D = g.D, K = g.K;
  const int slots = K <= 16 ? 16 : 32;          // threads per token
  const int ntok = blockDim.x / slots;          // tokens per block
  const int r0 = blk * ntok;
  if (r0 >= g.NW) return;
  extern __shared__ float sm[];
  float* mu = sm;                                // [K][D+1]
  float* xs = mu + K * (D + 1);                  // [ntok][D+1]
  float* sem = xs + ntok * (D + 1);              // [ntok][K] semantic
  float* exd = sem + ntok * K;                   // [ntok][K] exact squared distance
  __shared__ float mm[kMaxClusters];
  __shared__ float xxs[32];
  __shared__ long long phi[kMaxClusters];
  __shared__ int alv[kMaxClusters];
  const size_t lane0 = ((size_t)b * g.G + grp) * K;
  for (int i = tid; i < K * D; i += blockDim.x) mu[(i / D) * (D + 1) + i % D] = s.centroid[lane0 * D + i];
  if (tid < K) {
    alv[tid] = s.alive[lane0 + tid] != 0;
    phi[tid] = s.p_hi_c[lane0 + tid];
  }
  const T* snap = static_cast<const T*>(w.snap_k);
  const T* rec = static_cast<const T*>(s.recent_k_raw);
  const int nrow = min(ntok, g.NW - r0);
  constexpr int VN = Vec<T>::N;
  const int DV = D / VN;
  for (int item = tid; item < nrow * DV; item += blockDim.x) {
    const int row = item / DV, v = item % DV;
    float xv[VN];
    unpack(*reinterpret_cast<const uint4*>(token_row<T>(g, snap, rec, b, grp, r0 + row) + v * VN), xv,
           (const T*)nullptr);
#pragma unroll
    for (int e = 0; e < VN; ++e) xs[row * (D + 1) + v * VN + e] = xv[e];
  }
  __syncthreads();
  if (tid < K) {
    float a = 0.f;
    for (int d = 0; d < D; ++d) a = fadd(a, fmul(mu[tid * (D + 1) + d], mu[tid * (D + 1) + d]));
    mm[tid] = a;
  }
  const int tok = tid / slots, c = tid % slots;
  if (tok < nrow) {
    const float* x = xs + tok * (D + 1);
    if (c < K) {
      const float* m = mu + c * (D + 1);
      float dot = 0.f, ex = 0.f;
      for (int d = 0; d < D; ++d) {
        dot = fadd(dot, fmul(x[d], m[d]));
        const float df = fsub(x[d], m[d]);
        ex = fadd(ex, fmul(df, df));
      }
      sem[tok * K + c] = dot;  // raw dot; the semantic distance needs |x|^2 and |mu|^2 below
      exd[tok * K + c] = ex;
    }
    if (c == (K < slots ? K : 0)) {
      float xx = 0.f;
      for (int d = 0; d < D; ++d) xx = fadd(xx, fmul(x[d], x[d]));
      xxs[tok] = xx;
    }
  }
  __syncthreads();
  if (c != 0 || tok >= nrow) return;
  const int r = r0 + tok;   // token index
  const int64_t pos = token_position(g, s, w, b, r);
  const float xx = xxs[tok];
  const float thresh = fmul(g.lam, s.s_h[(size_t)b * g.G + grp]);
  float best_cost = INFINITY, s_win = 0.f, best_ex = INFINITY, sem0 = 0.f;
  int winner = 0, nearest = 0;
  bool any_alive = false;
  for (int cc = 0; cc < K; ++cc) {
    const float semv = fmaxf(fsub(fadd(xx, mm[cc]), fmul(2.f, sem[tok * K + cc])), 0.f);
    if (cc == 0) sem0 = semv;
    if (!alv[cc]) continue;
    any_alive = true;
    const float gap = fmaxf((float)(pos - (int64_t)phi[cc]), 0.f);
    const float cost = fadd(semv, fmul(g.eta, fdiv(gap, fadd(gap, g.g0))));
    if (cost < best_cost) {
      best_cost = cost;
      winner = cc;
      s_win = semv;
    }
    const float dist = __fsqrt_rn(exd[tok * K + cc]);
    if (dist < best_ex) {
      best_ex = dist;
      nearest = cc;
    }
  }
  if (!any_alive) {
    winner = 0;
    s_win = sem0;
    nearest = 0;
  }
  const bool direct = any_alive && s_win <= thresh;
  const size_t o = ((size_t)b * g.G + grp) * g.NW + r;
  w.assign_tok[o] = (int8_t)(direct ? winner : nearest);
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

// ---------------------------------------------------------------- K5a: farthest-point seeding
// Runs only for lanes with free cluster slots and orphans (in practice the first
// flushes of a stream).  One thread-block cluster of kSeedCluster CTAs per
// (batch, group) lane: each CTA stages its share of the archived token rows in
// shared memory (odd 32-bit word stride, conflict-free), the per-pick argmax is
// exchanged through distributed shared memory, and the picks follow
// _semantic_attach_plan_torch (log_kv_cache.py:4636-4680): the first pick is the
// orphan with the largest semantic distance to its winner, every next pick the
// orphan farthest (by its minimum distance) from all picks so far; then every
// orphan joins the nearest live or seeded cluster.  Lanes without seeds exit at
// once (uniformly across the cluster).
constexpr int kSeedCluster = 8;

template <typename T>
__global__ void __cluster_dims__(kSeedCluster, 1, 1) __launch_bounds__(512) seed_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int grp = blockIdx.x / kSeedCluster, b = blockIdx.y, tid = threadIdx.x, nt = blockDim.x;
  const int D = g.D, K = g.K;
  const int na = w.narch[b];
  const size_t lane0 = ((size_t)b * g.G + grp) * K;
  const size_t row0 = ((size_t)b * g.G + grp) * g.NW;
  int8_t* asg = w.assign + row0;                 // archive rank order (written here)
  const int8_t* asg_tok = w.assign_tok + row0;   // token order (attach decisions)
  const uint8_t* orph_tok = w.orphan + row0;     // token order
  const float* swin_tok = w.s_winner + row0;     // token order
  const int* arch = w.arch_idx + (size_t)b * g.NW;
  auto orph = [&](int t) -> int { return orph_tok[arch[t]]; };
  const T* snap = static_cast<const T*>(w.snap_k);
  const T* rec = static_cast<const T*>(s.recent_k_raw);
  __shared__ int free_slots[kMaxClusters];
  __shared__ int picks[kMaxClusters];
  __shared__ int cand[kMaxClusters];
  __shared__ int sh_nfree, sh_norph, sh_pick;
  __shared__ ArgMax red[32];
  __shared__ ArgMax slot[2];
  if (tid == 0) {
    int nf = 0;
    for (int c = 0; c < K; ++c)
      if (!s.alive[lane0 + c]) free_slots[nf++] = c;
    sh_nfree = nf;
    sh_norph = 0;
  }
  __syncthreads();
  const int chunk = (na + kSeedCluster - 1) / kSeedCluster;
  const int t_lo = min(na, rank * chunk), t_hi = min(na, t_lo + chunk), nloc = t_hi - t_lo;
  // Decisions in archive rank order (orphans are overwritten below when seeds open).
  for (int t = t_lo + tid; t < t_hi; t += nt) asg[t] = asg_tok[arch[t]];
  int my = 0;
  for (int t = tid; t < na; t += nt) my += orph(t);
  atomicAdd(&sh_norph, my);
  __syncthreads();
  const int n_use = min(sh_nfree, sh_norph);
  if (n_use == 0) return;  // same decision in every CTA of the cluster
  // Dynamic shared memory: prow [D] f32 | mus [K][D+1] f32 | dist [chunk] f32 | cdist [chunk][K] f32 | rows.
  extern __shared__ float sm[];
  float* prow = sm;
  float* mus = prow + D;
  float* dist = mus + K * (D + 1);
  float* cdist = dist + chunk;
  const int rs = D + 4 / (int)sizeof(T);  // row stride in elements: an odd number of 32-bit words
  T* rows = reinterpret_cast<T*>(cdist + (size_t)chunk * K);
  const bool staged = g.seed_staged != 0;
  constexpr int VN = Vec<T>::N;
  if (staged) {
    for (int item = tid; item < nloc * (D / VN); item += nt) {
      const int t = item / (D / VN), v = item % (D / VN);
      const uint4 u = *reinterpret_cast<const uint4*>(token_row<T>(g, snap, rec, b, grp, arch[t_lo + t]) + v * VN);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < VN; ++j) rows[(size_t)t * rs + v * VN + j] = e[j];
    }
  }
  __syncthreads();
  auto xval = [&](int tl, int d) -> float {
    return staged ? Elem<T>::load(rows + (size_t)tl * rs + d)
                  : Elem<T>::load(token_row<T>(g, snap, rec, b, grp, arch[t_lo + tl]) + d);
  };
  for (int i = 0; i < n_use; ++i) {
    ArgMax a{-INFINITY, 0x7fffffff};
    for (int tl = tid; tl < nloc; tl += nt) {
      const int t = t_lo + tl;
      const float v = i == 0 ? (orph(t) ? swin_tok[arch[t]] : -INFINITY) : dist[tl];
      a = argmax_better(a, ArgMax{v, t});
    }
    a = block_argmax(a, red);
    if (tid == 0) slot[i & 1] = a;
    cluster.sync();
    if (tid == 0) {
      ArgMax best{-INFINITY, 0x7fffffff};
      for (int r = 0; r < kSeedCluster; ++r) best = argmax_better(best, *cluster.map_shared_rank(&slot[i & 1], r));
      sh_pick = best.i;
      picks[i] = best.i;
    }
    __syncthreads();
    const int pick = sh_pick;
    for (int d = tid; d < D; d += nt) prow[d] = Elem<T>::load(token_row<T>(g, snap, rec, b, grp, arch[pick]) + d);
    __syncthreads();
    for (int tl = tid; tl < nloc; tl += nt) {
      const int t = t_lo + tl;
      float acc = 0.f;
      for (int d = 0; d < D; ++d) {
        const float df = fsub(xval(tl, d), prow[d]);
        acc = fadd(acc, fmul(df, df));
      }
      float v = i == 0 ? (orph(t) ? acc : -INFINITY) : fminf(dist[tl], acc);
      if (t == pick) v = -INFINITY;  // a pick is never picked again
      dist[tl] = v;
    }
    __syncthreads();
  }
  // Orphans join the nearest live or seeded cluster: one (token, cluster) pair per thread.
  if (tid < K) cand[tid] = s.alive[lane0 + tid] != 0;
  for (int i = tid; i < K * D; i += nt) mus[(i / D) * (D + 1) + i % D] = s.centroid[lane0 * D + i];
  __syncthreads();
  for (int i = 0; i < n_use; ++i) {
    const int c = free_slots[i];
    if (tid == 0) cand[c] = 1;
    for (int d = tid; d < D; d += nt)
      mus[c * (D + 1) + d] = Elem<T>::load(token_row<T>(g, snap, rec, b, grp, arch[picks[i]]) + d);
  }
  __syncthreads();
  for (int item = tid; item < nloc * K; item += nt) {
    const int tl = item / K, c = item % K;
    float out = INFINITY;
    if (orph(t_lo + tl) && cand[c]) {
      float acc = 0.f;
      for (int d = 0; d < D; ++d) {
        const float df = fsub(xval(tl, d), mus[c * (D + 1) + d]);
        acc = fadd(acc, fmul(df, df));
      }
      out = __fsqrt_rn(acc);
    }
    cdist[item] = out;
  }
  __syncthreads();
  for (int tl = tid; tl < nloc; tl += nt) {
    if (!orph(t_lo + tl)) continue;
    float best = INFINITY;
    int bc = 0;
    for (int c = 0; c < K; ++c)
      if (cdist[tl * K + c] < best) {
        best = cdist[tl * K + c];
        bc = c;
      }
    asg[t_lo + tl] = (int8_t)bc;
  }
  __syncthreads();
  if (tid == 0)
    for (int i = 0; i < n_use; ++i)
      if (picks[i] >= t_lo && picks[i] < t_hi) asg[picks[i]] = (int8_t)free_slots[i];
  cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

// ---------------------------------------------------------------- K5b: commit plan
// One block per (batch, group) lane: a stable counting sort groups the archived
// tokens by cluster, then each cluster's job (ordinary, new, delayed) and scratch
// range are planned.
template <typename T>
__global__ void __launch_bounds__(1024) plan_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  const int b = blockIdx.y, grp = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const int K = g.K;
  const int na = w.narch[b];
  const size_t lane0 = ((size_t)b * g.G + grp) * K;
  const size_t row0 = ((size_t)b * g.G + grp) * g.NW;
  const int8_t* asg = w.assign + row0;
  const int* arch = w.arch_idx + (size_t)b * g.NW;
  __shared__ int wsum[32];
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
