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
#include "flush_ladder.cuh"

namespace logkv {

// ---------------------------------------------------------------- K4: attach decisions
// Decisions for every token of the [old pool | flushed window] index space (the archive
// is a subset, picked later by the span choice; decisions depend only on the frozen
// cluster state).  A warp takes 8 tokens; a token's 4 lanes each own CPL consecutive centres
// (lane q: centres q*CPL .. q*CPL+CPL-1) and compute, left to right over the features, the
// token's dot product with each of them and |x|^2, then the semantic distances and routing
// costs; the winner is the first-index argmin of the costs over live centres (as the
// reference's in-order scan / torch.argmin): first over the lane's centres in index order,
// then by a shuffle reduction over the token's 4 lanes.  Orphans then get exact distances to
// the live centres the same way (nearest = first-index argmin), in a second pass that a warp
// runs only when one of its tokens is an orphan.  Token rows (64 per block) and centres are
// staged in shared memory as float rows of D+4 words: the 8 token rows of a warp fall in
// distinct bank quads, and a centre load of a warp reads 4 rows (one per lane of a token),
// which for K <= 12 also fall in distinct bank quads, so every 16-byte shared load is one
// wavefront; a token row is read by 4 lanes and a centre row by 8 tokens' lanes at once,
// instead of once per (token, centre).  Centre norms come from the snapshot kernel.
// Outputs are indexed by token.  DC != 0 is a compile-time head dim.
constexpr int kAttachTokens = 64;   // tokens per 256-thread block: 8 warps x 8 tokens

// Best and runner-up (value, index) over the lane's centres, in index order: a later equal
// value never replaces the best (first index wins), so an exact tie becomes the runner-up.
template <int CPL>
__device__ __forceinline__ void lane_top2(const float (&v)[CPL], const bool (&ok)[CPL], int c0, float* bv, int* bi,
                                          float* sv, int* si, int none) {
  *bv = INFINITY;
  *bi = none;
  *sv = INFINITY;
  *si = none;
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    if (!ok[j]) continue;
    if (v[j] < *bv) {
      *sv = *bv;
      *si = *bi;
      *bv = v[j];
      *bi = c0 + j;
    } else if (v[j] < *sv) {
      *sv = v[j];
      *si = c0 + j;
    }
  }
}

// (value, index) best and runner-up over the 4 lanes of a token, lowest index on ties; `aux`
// follows the best.  The merge is symmetric, so both lanes of every exchange agree.
__device__ __forceinline__ void quad_top2(float* bv, int* bi, float* sv, int* si, float* aux) {
  auto better = [](float v1, int i1, float v2, int i2) { return v1 < v2 || (v1 == v2 && i1 < i2); };
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, *bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, *bi, off);
    const float osv = __shfl_xor_sync(0xffffffffu, *sv, off);
    const int osi = __shfl_xor_sync(0xffffffffu, *si, off);
    const float oa = __shfl_xor_sync(0xffffffffu, *aux, off);
    if (better(ov, oi, *bv, *bi)) {
      if (better(*bv, *bi, osv, osi)) {
        *sv = *bv;
        *si = *bi;
      } else {
        *sv = osv;
        *si = osi;
      }
      *bv = ov;
      *bi = oi;
      *aux = oa;
    } else if (better(ov, oi, *sv, *si)) {
      *sv = ov;
      *si = oi;
    }
  }
}

template <typename T, int DC, int CPL>
__device__ void attach_body(const Geo& g, const logkv_state_t& s, const Work& w, int blk) {
  const int b = blockIdx.z, grp = blockIdx.y, tid = threadIdx.x;
  const int D = DC ? DC : g.D, K = g.K;
  const int r0 = blk * kAttachTokens;
  if (r0 >= g.NW) return;
  const int nrow = min(kAttachTokens, g.NW - r0);
  extern __shared__ float4 sm4[];
  const int RS4 = D / 4 + 1;                     // row stride in float4: D + 4 words
  float4* mu4 = sm4;                             // [K][RS4]
  float4* xs4 = sm4 + K * RS4;                   // [kAttachTokens][RS4]
  __shared__ float cn_s[kMaxClusters];
  __shared__ long long phi_s[kMaxClusters];
  __shared__ uint8_t alv_s[kMaxClusters];
  __shared__ int any_alive_s;
  const size_t lane0 = ((size_t)b * g.G + grp) * K;
  if (tid == 0) any_alive_s = 0;
  __syncthreads();
  for (int cc = tid; cc < K; cc += blockDim.x) {
    cn_s[cc] = w.cnorm[lane0 + cc];
    phi_s[cc] = s.p_hi_c[lane0 + cc];
    alv_s[cc] = s.alive[lane0 + cc] != 0;
    if (s.alive[lane0 + cc]) any_alive_s = 1;
  }
  const int D4 = D / 4;
  const float4* cent4 = reinterpret_cast<const float4*>(s.centroid + lane0 * D);
  for (int i = tid; i < K * D4; i += blockDim.x) mu4[(i / D4) * RS4 + i % D4] = cent4[i];
  const T* snap = static_cast<const T*>(w.snap_k);
  const T* rec = static_cast<const T*>(s.recent_k_raw);
  constexpr int VN = Vec<T>::N;
  const int DV = D / VN;
  for (int i = tid; i < nrow * DV; i += blockDim.x) {
    const int row = i / DV, v = i % DV;
    float xv[VN];
    unpack(*reinterpret_cast<const uint4*>(token_row<T>(g, snap, rec, b, grp, r0 + row) + v * VN), xv,
           (const T*)nullptr);
#pragma unroll
    for (int e = 0; e < VN; e += 4)
      xs4[row * RS4 + (v * VN + e) / 4] = make_float4(xv[e], xv[e + 1], xv[e + 2], xv[e + 3]);
  }
  __syncthreads();
  const int lane = tid & 31, q = lane & 3;
  const int t = (tid >> 5) * 8 + (lane >> 2);   // token slot in the block
  const bool live_tok = t < nrow;
  const int c0 = q * CPL;
  int cj[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j) cj[j] = min(c0 + j, K - 1);   // spare slots read a real row
  const float4* x = xs4 + t * RS4;
  // Pass 1: dot products with the lane's centres and |x|^2, left to right.
  float dot[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j) dot[j] = 0.f;
  float xx = 0.f;
#pragma unroll(DC ? 4 : 1)
  for (int d4 = 0; d4 < D4; ++d4) {
    const float4 xv = x[d4];
    xx = fadd(xx, fmul(xv.x, xv.x));
    xx = fadd(xx, fmul(xv.y, xv.y));
    xx = fadd(xx, fmul(xv.z, xv.z));
    xx = fadd(xx, fmul(xv.w, xv.w));
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const float4 mv = mu4[cj[j] * RS4 + d4];
      dot[j] = fadd(dot[j], fmul(xv.x, mv.x));
      dot[j] = fadd(dot[j], fmul(xv.y, mv.y));
      dot[j] = fadd(dot[j], fmul(xv.z, mv.z));
      dot[j] = fadd(dot[j], fmul(xv.w, mv.w));
    }
  }
  // Semantic distances and routing costs of the lane's centres.
  const int r = r0 + t;   // token index
  const int64_t pos = live_tok ? token_position(g, s, w, b, r) : 0;
  float semv[CPL], cost[CPL];
  bool ok[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int c = cj[j];
    semv[j] = fmaxf(fsub(fadd(xx, cn_s[c]), fmul(2.f, dot[j])), 0.f);
    const float gap = fmaxf((float)(pos - (int64_t)phi_s[c]), 0.f);
    cost[j] = fadd(semv[j], fmul(g.eta, fdiv(gap, fadd(gap, g.g0))));
    // Live centres with a cost below +inf compete (NaN and +inf never replace the initial +inf).
    ok[j] = c0 + j < K && alv_s[c] && cost[j] < INFINITY;
  }
  float best_cost, second_cost, sem_win = 0.f;
  int wi, ri;
  lane_top2<CPL>(cost, ok, c0, &best_cost, &wi, &second_cost, &ri, kMaxClusters);
#pragma unroll
  for (int j = 0; j < CPL; ++j)
    if (c0 + j == wi) sem_win = semv[j];
  quad_top2(&best_cost, &wi, &second_cost, &ri, &sem_win);
  const bool any_alive = any_alive_s != 0;
  const int winner = wi < kMaxClusters ? wi : 0;
  // No live centre: winner 0 with cluster 0's semantic distance (the token is an orphan);
  // live centres but no finite cost: winner 0 with s = 0 (the scan's initial values).
  const float sem0 = __shfl_sync(0xffffffffu, semv[0], lane & ~3);
  const float s_win = !any_alive ? sem0 : (wi < kMaxClusters ? sem_win : 0.f);
  const size_t o = ((size_t)b * g.G + grp) * g.NW + r;
  const float thresh = fmul(g.lam, s.s_h[(size_t)b * g.G + grp]);
  const bool direct = any_alive && s_win <= thresh;
  const bool orphan = live_tok && any_alive && !direct;
  if (live_tok && q == 0) {
    w.orphan[o] = direct ? 0 : 1;
    w.s_winner[o] = s_win;
    if (!orphan) w.assign_tok[o] = (int8_t)winner;   // no live centre: 0
    if (any_alive && ri < kMaxClusters && near_tie(best_cost, second_cost))
      log_tie(w, LOGKV_TIE_ATTACH_COST, b, grp, -1, (int)pos, wi, ri, rel_gap(best_cost, second_cost), best_cost);
    if (any_alive && near_tie(s_win, thresh))
      log_tie(w, LOGKV_TIE_DIRECT, b, grp, -1, (int)pos, direct ? 1 : 0, winner, rel_gap(s_win, thresh), s_win);
  }
  if (!__any_sync(0xffffffffu, orphan)) return;
  // Pass 2 (warps with an orphan): exact distances to the lane's live centres, left to right;
  // nearest = first-index argmin (NaN and +inf never win; none: centre 0).
  float ex[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j) ex[j] = 0.f;
#pragma unroll(DC ? 4 : 1)
  for (int d4 = 0; d4 < D4; ++d4) {
    const float4 xv = x[d4];
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const float4 mv = mu4[cj[j] * RS4 + d4];
      float df = fsub(xv.x, mv.x);
      ex[j] = fadd(ex[j], fmul(df, df));
      df = fsub(xv.y, mv.y);
      ex[j] = fadd(ex[j], fmul(df, df));
      df = fsub(xv.z, mv.z);
      ex[j] = fadd(ex[j], fmul(df, df));
      df = fsub(xv.w, mv.w);
      ex[j] = fadd(ex[j], fmul(df, df));
    }
  }
  float dist[CPL];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    dist[j] = __fsqrt_rn(ex[j]);
    ok[j] = c0 + j < K && alv_s[cj[j]] && dist[j] < INFINITY;
  }
  float best_d, second_d, unused = 0.f;
  int ni, nri;
  lane_top2<CPL>(dist, ok, c0, &best_d, &ni, &second_d, &nri, kMaxClusters);
  quad_top2(&best_d, &ni, &second_d, &nri, &unused);
  if (orphan && q == 0) {
    w.assign_tok[o] = (int8_t)(ni < kMaxClusters ? ni : 0);
    if (nri < kMaxClusters && near_tie(best_d, second_d))
      log_tie(w, LOGKV_TIE_NEAREST, b, grp, -1, (int)pos, ni, nri, rel_gap(best_d, second_d), best_d);
  }
}

// (value, index) argmax with the lowest index winning ties, plus the runner-up (for the
// near-tie log).  merge() is symmetric, so every order of combining gives the same pair.
struct ArgMax {
  float v;
  int i;
  float v2;
  int i2;
};
__device__ __forceinline__ bool argmax_before(float v1, int i1, float v2, int i2) {
  return v1 > v2 || (v1 == v2 && i1 < i2);
}
__device__ __forceinline__ ArgMax argmax_none() { return ArgMax{-INFINITY, 0x7fffffff, -INFINITY, 0x7fffffff}; }
__device__ __forceinline__ ArgMax argmax_merge(ArgMax a, ArgMax b) {
  if (argmax_before(b.v, b.i, a.v, a.i)) {
    const ArgMax t = a;
    a = b;
    b = t;
  }
  // a holds the best head; the runner-up is the better of a's runner-up and b's head.
  if (argmax_before(b.v, b.i, a.v2, a.i2)) {
    a.v2 = b.v;
    a.i2 = b.i;
  }
  return a;
}
__device__ __forceinline__ ArgMax argmax_push(ArgMax a, float v, int i) {
  return argmax_merge(a, ArgMax{v, i, -INFINITY, 0x7fffffff});
}
__device__ ArgMax block_argmax(ArgMax v, ArgMax* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    ArgMax o;
    o.v = __shfl_xor_sync(0xffffffffu, v.v, off);
    o.i = __shfl_xor_sync(0xffffffffu, v.i, off);
    o.v2 = __shfl_xor_sync(0xffffffffu, v.v2, off);
    o.i2 = __shfl_xor_sync(0xffffffffu, v.i2, off);
    v = argmax_merge(v, o);
  }
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    ArgMax best = sh[0];
    for (int k = 1; k < nwarps; ++k) best = argmax_merge(best, sh[k]);
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
    ArgMax a = argmax_none();
    for (int tl = tid; tl < nloc; tl += nt) {
      const int t = t_lo + tl;
      const float v = i == 0 ? (orph(t) ? swin_tok[arch[t]] : -INFINITY) : dist[tl];
      a = argmax_push(a, v, t);
    }
    a = block_argmax(a, red);
    if (tid == 0) slot[i & 1] = a;
    cluster.sync();
    if (tid == 0) {
      ArgMax best = argmax_none();
      for (int r = 0; r < kSeedCluster; ++r) best = argmax_merge(best, *cluster.map_shared_rank(&slot[i & 1], r));
      if (rank == 0 && best.i2 < na && near_tie(best.v, best.v2))
        log_tie(w, LOGKV_TIE_SEED_PICK, b, grp, -1, i, (int)token_position(g, s, w, b, arch[best.i]),
                (int)token_position(g, s, w, b, arch[best.i2]), rel_gap(best.v, best.v2), best.v);
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
    float best = INFINITY, second = INFINITY;
    int bc = 0, sc = -1;
    for (int c = 0; c < K; ++c) {
      const float dv = cdist[tl * K + c];
      if (dv < best) {
        second = best;
        sc = best < INFINITY ? bc : -1;
        best = dv;
        bc = c;
      } else if (dv < second) {
        second = dv;
        sc = c;
      }
    }
    asg[t_lo + tl] = (int8_t)bc;
    if (sc >= 0 && near_tie(best, second))
      log_tie(w, LOGKV_TIE_SEED_NEAREST, b, grp, -1, (int)token_position(g, s, w, b, arch[t_lo + tl]), bc, sc,
              rel_gap(best, second), best);
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
  // Stable counting sort of archive ranks by cluster, in one pass: per 32-rank chunk and cluster
  // a ballot count, one block scan of those counts in (cluster, chunk) order, then each rank goes
  // to its (cluster, chunk) offset plus its lane rank among the chunk's ranks of that cluster.
  // NW <= 8192 ranks make at most 256 chunks; K <= kMaxClusters.
  __shared__ int cl_count[kMaxClusters], cl_off[kMaxClusters];
  __shared__ int cnt[(8192 / 32) * kMaxClusters];  // [chunk][cluster] counts, then offsets
  const int lane = tid & 31, warp = tid >> 5, nwarps = nt >> 5;
  const int nchunk = (na + 31) / 32;
  for (int ch = warp; ch < nchunk; ch += nwarps) {
    const int t = ch * 32 + lane;
    const int a = t < na ? asg[t] : -1;
    int mine = 0;
    for (int c = 0; c < K; ++c) {
      const int m = __popc(__ballot_sync(0xffffffffu, a == c));
      if (lane == c) mine = m;
    }
    if (lane < K) cnt[ch * K + lane] = mine;
  }
  __syncthreads();
  {
    // Exclusive scan of cnt in (cluster, chunk) order: thread tid owns q consecutive entries.
    const int n2 = K * nchunk, q = (n2 + nt - 1) / nt;
    const int j0 = min(n2, tid * q), j1 = min(n2, j0 + q);
    int local = 0;
    for (int j = j0; j < j1; ++j) local += cnt[(j % nchunk) * K + j / nchunk];
    const int incl = block_inclusive_scan(local, wsum);
    int run = incl - local;
    for (int j = j0; j < j1; ++j) {
      const int at = (j % nchunk) * K + j / nchunk;
      const int v = cnt[at];
      cnt[at] = run;
      run += v;
    }
  }
  __syncthreads();
  for (int ch = warp; ch < nchunk; ch += nwarps) {
    const int t = ch * 32 + lane;
    const int a = t < na ? asg[t] : -1;
    const unsigned same = __match_any_sync(0xffffffffu, a);
    if (t < na && a >= 0 && a < K) w.tok_list[row0 + cnt[ch * K + a] + __popc(same & ((1u << lane) - 1u))] = t;
  }
  if (tid < K) cl_off[tid] = nchunk ? cnt[tid] : 0;   // chunk 0's offset of cluster tid
  __syncthreads();
  if (tid < K) cl_count[tid] = (tid + 1 < K ? cl_off[tid + 1] : na) - cl_off[tid];
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
      // The lane's scratch range holds every level's incoming rows at once (the parallel cascade
      // keeps all levels' carries): at most m0 + L of them (each level carries at most half of
      // its incoming rows, rounded up).
      if (type != kJobNone) scr += m0 + g.L + 2;
    }
    if (scr > g.S) set_status(w.status, kStatusCarryOverflow);
  }
  __syncthreads();
  if (tid < K) write_lane_plan(g, s, w, lane0 + tid);
}

// Lane plans of a replayed flush (the replay copies the recorded per-cluster plan and skips this
// file's kernels): grid (G, B), one thread per cluster.
__global__ void lane_plan_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  if ((int)threadIdx.x < g.K) write_lane_plan(g, s, w, ((size_t)blockIdx.y * g.G + blockIdx.x) * g.K + threadIdx.x);
}

// ---------------------------------------------------------------- op-log append
// The route log rows of the last flush (_record_ops, litgpt/log_kv_cache.py:2043-2071), per
// (batch, group) lane in the reference's order: for the unified route first a WARD_MERGE row
// (op 3, keep, free, -1) per Ward merge of two old clusters, in merge order; a NEW_CLUSTER row (op 0, cluster, 0, position of
// the opening token) for every cluster the flush opened, in cluster order (_semantic_new_clusters
// :2276-2298); then JOIN rows (op 2, cluster, 0, position) for the joined tokens of every
// ordinary or newly opened cluster, cluster by cluster, positions ascending
// (_semantic_commit_joins_unsegmented :4158-4170); then JOIN rows for the new tokens of every
// delayed cluster (_alpha_commit_joins :3781-3788).  Reads the plan the flush left in its
// workspace; appends at op_len[lane] unless the log's capacity would be exceeded, in which case
// no row is written and op_len[lane] becomes capacity + 1 (sticky: later appends refuse too).

__global__ void __launch_bounds__(256) oplog_append_kernel(Geo g, Work w, int32_t* op_log, int32_t* op_len,
                                                           int cap) {
  const int b = blockIdx.y, grp = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const int K = g.K;
  const size_t bg = (size_t)b * g.G + grp, row0 = bg * K;
  __shared__ int off_new[kMaxClusters], off_join[kMaxClusters], off_late[kMaxClusters];
  __shared__ int sh_total, sh_new, sh_join, sh_len, sh_ward;
  if (tid == 0) {
    int nn = 0, nj = 0, nl = 0;
    // Unified route: the lane's Ward merges come first (_semantic_ward_merge_batch records them
    // before the new clusters and joins, log_kv_cache.py:2580).
    const int nw = (g.route == LOGKV_ROUTE_UNIFIED && w.narch[b] > 0) ? w.u.words[bg * kULaneWords + kUWard] : 0;
    sh_ward = nw;
    for (int c = 0; c < K; ++c) {
      const int type = w.plan_type[row0 + c], n = w.plan_n[row0 + c];
      off_new[c] = nn;
      off_join[c] = nj;
      off_late[c] = nl;
      if (type == kJobNew && n > 0) {
        nn += 1;
        nj += n - 1;
      } else if (type == kJobOrdinary) {
        nj += n;
      } else if (type == kJobLate) {
        nl += n;
      }
    }
    sh_new = nn;
    sh_join = nj;
    sh_total = nw + nn + nj + nl;
    sh_len = op_len[bg];
    if (sh_len > cap || sh_len + sh_total > cap) {
      op_len[bg] = cap + 1;
      sh_total = -1;
    }
  }
  __syncthreads();
  if (sh_total < 0) return;
  for (int i = tid; i < sh_ward; i += nt) {
    int4* wl = reinterpret_cast<int4*>(op_log) + bg * (size_t)cap;
    wl[sh_len + i] = make_int4(3, w.u.ward[(bg * K + i) * 2], w.u.ward[(bg * K + i) * 2 + 1], -1);
  }
  const int len0 = sh_len + sh_ward;
  const int* arch = w.arch_idx + (size_t)b * g.NW;
  const int* toks = w.tok_list + bg * g.NW;
  const int64_t* pos = w.tok_pos + (size_t)b * g.NW;
  int4* log = reinterpret_cast<int4*>(op_log) + bg * (size_t)cap;
  for (int c = 0; c < K; ++c) {
    const int type = w.plan_type[row0 + c], n = w.plan_n[row0 + c], toff = w.plan_off[row0 + c];
    if (type == kJobNone || n == 0) continue;
    for (int i = tid; i < n; i += nt) {
      const int p = (int)pos[arch[toks[toff + i]]];
      int at;
      int op = 2;
      if (type == kJobNew) {
        if (i == 0) {
          op = 0;
          at = len0 + off_new[c];
        } else {
          at = len0 + sh_new + off_join[c] + i - 1;
        }
      } else if (type == kJobOrdinary) {
        at = len0 + sh_new + off_join[c] + i;
      } else {
        at = len0 + sh_new + sh_join + off_late[c] + i;
      }
      log[at] = make_int4(op, c, 0, p);
    }
  }
  __syncthreads();
  if (tid == 0) op_len[bg] = sh_len + sh_total;
}

}  // namespace logkv
