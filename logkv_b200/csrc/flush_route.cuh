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
// cluster state).  A token owns 16 (K <= 16) or 32 consecutive lanes, one per centre: each
// computes the token's dot product with its centre left to right over the features, then
// the semantic distance and routing cost; the token's winner is the first-index argmin of
// the costs over live centres (as the reference's in-order scan / torch.argmin), found by a
// shuffle reduction over the token's lanes.  Orphans then get exact distances to the live
// centres the same way (nearest = first-index argmin).  Token rows and centres are staged
// in shared memory (16-byte rows, conflict-free); centre norms come from the snapshot
// kernel.  Outputs are indexed by token.  DC != 0 is a compile-time head dim.

// First-index argmin over the `width` lanes of a token (width 16 or 32, aligned): lanes with
// valid = false never win; returns the winning lane offset, or width if none is valid.
__device__ __forceinline__ int group_argmin(float v, bool valid, int c, int width, float* best_v) {
  float bv = valid ? v : INFINITY;
  int bi = valid ? c : width;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    if (off >= width) continue;
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ov < bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  *best_v = bv;
  return bi;
}

constexpr int kAttachRounds = 1;  // token rounds per block (the staged centres are reused)

template <typename T, int DC>
__device__ void attach_body(const Geo& g, const logkv_state_t& s, const Work& w, int blk) {
  const int b = blockIdx.z, grp = blockIdx.y, tid = threadIdx.x;
  const int D = DC ? DC : g.D, K = g.K;
  const int slots = K <= 16 ? 16 : 32;          // lanes per token
  const int ntok = blockDim.x / slots;          // tokens per round
  if (blk * kAttachRounds * ntok >= g.NW) return;
  extern __shared__ float4 sm4[];
  const int RS = D + 4;                          // row stride in floats: 16-byte rows, conflict-free
  float* mu = reinterpret_cast<float*>(sm4);     // [K][RS]
  float* xs = mu + K * RS;                       // [ntok][RS]
  __shared__ float xxs[32];
  __shared__ int orph_tok[32];
  __shared__ int n_orph;
  __shared__ float cn_s[kMaxClusters];
  __shared__ long long phi_s[kMaxClusters];
  __shared__ uint8_t alv_s[kMaxClusters];
  const size_t lane0 = ((size_t)b * g.G + grp) * K;
  if (tid == 0) n_orph = 0;
  for (int cc = tid; cc < K; cc += blockDim.x) {
    cn_s[cc] = w.cnorm[lane0 + cc];
    phi_s[cc] = s.p_hi_c[lane0 + cc];
    alv_s[cc] = s.alive[lane0 + cc] != 0;
  }
  const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
  const int D4 = D / 4;
  // Centres and token rows into shared memory: one row per warp at a time, 16-byte units.
  const float4* cent4 = reinterpret_cast<const float4*>(s.centroid + lane0 * D);
  for (int cc = warp; cc < K; cc += nwarps)
    for (int d4 = lane; d4 < D4; d4 += 32) reinterpret_cast<float4*>(mu + cc * RS)[d4] = cent4[cc * D4 + d4];
  const T* snap = static_cast<const T*>(w.snap_k);
  const T* rec = static_cast<const T*>(s.recent_k_raw);
  for (int round = 0; round < kAttachRounds; ++round) {
    const int r0 = (blk * kAttachRounds + round) * ntok;
    if (r0 >= g.NW) break;   // uniform across the block
    const int nrow = min(ntok, g.NW - r0);
    constexpr int VN = Vec<T>::N;
    const int DV = D / VN;
    for (int row = warp; row < nrow; row += nwarps) {
      const T* src = token_row<T>(g, snap, rec, b, grp, r0 + row);
      for (int v = lane; v < DV; v += 32) {
        float xv[VN];
        unpack(*reinterpret_cast<const uint4*>(src + v * VN), xv, (const T*)nullptr);
#pragma unroll
        for (int e = 0; e < VN; e += 4)
          *reinterpret_cast<float4*>(xs + row * RS + v * VN + e) = make_float4(xv[e], xv[e + 1], xv[e + 2], xv[e + 3]);
      }
    }
    __syncthreads();
    // Pass 1, one lane per (token, centre): the dot product, left to right over the features.
    // When a lane of the token's group is spare (K < slots), lane K runs the same loop against
    // the token itself, so its "dot" is |x|^2 (same operations).
    const int tok = tid / slots, c = tid % slots;
    const bool spare = K < slots;
    const bool live_tok = tok < nrow;
    float dot = 0.f;
    if (live_tok && c <= (spare ? K : K - 1)) {
      const float4* x = reinterpret_cast<const float4*>(xs + tok * RS);
      const float4* m = reinterpret_cast<const float4*>(c < K ? mu + c * RS : xs + tok * RS);
#pragma unroll(DC ? 8 : 1)
      for (int d4 = 0; d4 < D4; ++d4) {
        const float4 xv = x[d4], mv = m[d4];
        dot = fadd(dot, fmul(xv.x, mv.x));
        dot = fadd(dot, fmul(xv.y, mv.y));
        dot = fadd(dot, fmul(xv.z, mv.z));
        dot = fadd(dot, fmul(xv.w, mv.w));
      }
      if (c == K) xxs[tok] = dot;
    }
    if (!spare && live_tok && c == 0) {
      const float* x = xs + tok * RS;
      float xx = 0.f;
      for (int d = 0; d < D; ++d) xx = fadd(xx, fmul(x[d], x[d]));
      xxs[tok] = xx;
    }
    __syncthreads();
    // Pass 2, one lane per (token, centre): semantic distance and routing cost; then the
    // token's decision by a shuffle argmin over its lanes.
    const int r = r0 + tok;   // token index
    const bool mine = live_tok && c < K;
    const bool alive_c = mine && alv_s[c];
    float semv = 0.f, cost = INFINITY;
    if (mine) {
      const int64_t pos = token_position(g, s, w, b, r);
      semv = fmaxf(fsub(fadd(xxs[tok], cn_s[c]), fmul(2.f, dot)), 0.f);
      const float gap = fmaxf((float)(pos - (int64_t)phi_s[c]), 0.f);
      cost = fadd(semv, fmul(g.eta, fdiv(gap, fadd(gap, g.g0))));
    }
    const unsigned gmask = (slots == 32 ? 0xffffffffu : 0xffffu) << (lane & ~(slots - 1) & 31);
    const bool any_alive = (__ballot_sync(0xffffffffu, alive_c) & gmask) != 0u;
    float best_cost;
    // Live centres with a cost below +inf compete (NaN and +inf never replace the initial +inf).
    const int wi = group_argmin(cost, alive_c && cost < INFINITY, c, slots, &best_cost);
    const int winner = wi < slots ? wi : 0;
    const int src_lane = (lane & ~(slots - 1)) + winner;
    const float sem_win = __shfl_sync(0xffffffffu, semv, src_lane);
    // No live centre: winner 0 with cluster 0's semantic distance (the token is an orphan);
    // live centres but no finite cost: winner 0 with s = 0 (the scan's initial values).
    const float s_win = !any_alive ? sem_win : (wi < slots ? sem_win : 0.f);
    const size_t o = ((size_t)b * g.G + grp) * g.NW + r;
    if (live_tok && c == 0) {
      const float thresh = fmul(g.lam, s.s_h[(size_t)b * g.G + grp]);
      const bool direct = any_alive && s_win <= thresh;
      w.orphan[o] = direct ? 0 : 1;
      w.s_winner[o] = s_win;
      if (direct || !any_alive) w.assign_tok[o] = (int8_t)winner;   // no live centre: 0
      else orph_tok[atomicAdd(&n_orph, 1)] = tok;
    }
    __syncthreads();
    const int no = n_orph;
    if (no > 0) {
      // Exact distances of the queued orphans to the live centres: orphan j takes the lanes of
      // token slot j; nearest = first-index argmin (NaN and +inf never win; none: centre 0).
      const int j = tok;
      float dist = INFINITY;
      const bool act = j < no && c < K && alv_s[c];
      if (act) {
        const int t = orph_tok[j];
        const float4* x = reinterpret_cast<const float4*>(xs + t * RS);
        const float4* m = reinterpret_cast<const float4*>(mu + c * RS);
        float ex = 0.f;
#pragma unroll(DC ? 8 : 1)
        for (int d4 = 0; d4 < D4; ++d4) {
          const float4 xv = x[d4], mv = m[d4];
          float df = fsub(xv.x, mv.x);
          ex = fadd(ex, fmul(df, df));
          df = fsub(xv.y, mv.y);
          ex = fadd(ex, fmul(df, df));
          df = fsub(xv.z, mv.z);
          ex = fadd(ex, fmul(df, df));
          df = fsub(xv.w, mv.w);
          ex = fadd(ex, fmul(df, df));
        }
        dist = __fsqrt_rn(ex);
      }
      float best_d;
      const int ni = group_argmin(dist, act && dist < INFINITY, c, slots, &best_d);
      if (j < no && c == 0)
        w.assign_tok[((size_t)b * g.G + grp) * g.NW + r0 + orph_tok[j]] = (int8_t)(ni < slots ? ni : 0);
    }
    __syncthreads();  // token rows and the orphan queue are reused by the next round
    if (tid == 0) n_orph = 0;
  }
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

// ---------------------------------------------------------------- op-log append
// The route log rows of the last flush (_record_ops, litgpt/log_kv_cache.py:2043-2071), per
// (batch, group) lane in the reference's order: a NEW_CLUSTER row (op 0, cluster, 0, position of
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
  __shared__ int sh_total, sh_new, sh_join, sh_len;
  if (tid == 0) {
    int nn = 0, nj = 0, nl = 0;
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
    sh_total = nn + nj + nl;
    sh_len = op_len[bg];
    if (sh_len > cap || sh_len + sh_total > cap) {
      op_len[bg] = cap + 1;
      sh_total = -1;
    }
  }
  __syncthreads();
  if (sh_total < 0) return;
  const int len0 = sh_len;
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
  if (tid == 0) op_len[bg] = len0 + sh_total;
}

}  // namespace logkv
