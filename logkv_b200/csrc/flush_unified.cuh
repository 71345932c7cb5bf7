// Unified (Ward / radius) route of a flush on the device (semantic_unified_route=True).
//
// Follows _semantic_route_unified (litgpt/log_kv_cache.py:3589-3688) for every (batch, group)
// lane that archives tokens:
//   candidate pass  the lane's archived keys as unit-mass float32 centres, mutual-nearest Ward
//                   rounds with the radius limit sqrt(cluster_lambda_rel * s_h) down to 1
//                   (_semantic_unified_reduce_device :3246-3299);
//   labels          every token's candidate by pointer jumping over the merge forest
//                   (_semantic_unified_labels_batch :3544-3568);
//   global pass     [live centroids (mass n_total), candidates (mass = tokens)] reduced to K
//                   clusters without radius limits, with frozen-centre sweeps when
//                   semantic_merge_passes > 1;
//   route           a candidate whose root is an old cluster joins it, other roots open new
//                   clusters in the free slots (ascending), merges of two old clusters become Ward
//                   merges, applied in trace order before anything joins
//                   (_semantic_ward_merge_batch :2517-2593: the keep and free entries re-appended
//                   to the cleared keep cluster in _semantic_ward_entry_index order :2450-2474).
// The decisions land in the attach route's plan format (a cluster per archived token), so the
// per-cluster plan, prepare and cascade kernels commit them unchanged.
//
// The pair matrices take the reference's two forms (_semantic_unified_pair_matrix :3185-3221):
// exact differences, rooted and squared (cdist), when the widest active lane of the lane's tile
// has at most 32 rows, else a Gram product of the centres centred on each lane's first row.  The
// tile is the reference's CPU tile (_semantic_unified_tile :3578-3587, 64 MiB of float32 distances
// per tile).  Gram products (one fused multiply-add per feature) and difference sums run left to
// right over the features in float32; nothing else contracts (this file is compiled with
// -fmad=false).
#pragma once

#include "flush_cascade.cuh"
#include "flush_ladder.cuh"
#include "unified_core.cuh"

namespace logkv {

constexpr long long kUTileBytes = 64ll << 20;   // the CPU reference's distance budget per lane tile
constexpr int kGramTile = 128;                  // Gram output tile (rows x columns) per CTA
constexpr int kGramChunk = 32;                  // features staged per pass of the Gram tile

__device__ __forceinline__ size_t ulane(const Geo& g, int b, int grp) { return (size_t)b * g.G + grp; }
__device__ __forceinline__ int32_t* uwords(const Work& w, size_t bg) { return w.u.words + bg * kULaneWords; }

// The lane's reducer state for one pass (0 = candidates, 1 = global).
__device__ inline logkv_ward::RunLane urun(const Geo& g, const Work& w, size_t bg, int pass) {
  const size_t Mg = g.Mg;
  logkv_ward::RunLane l;
  l.dist = w.u.dist + bg * Mg * Mg;
  l.mu = pass ? w.u.mu_g + bg * Mg * g.D : w.u.mu_c + bg * (size_t)g.NW * g.D;
  l.mass = w.u.mass + bg * Mg;
  l.radius = w.u.radius + bg * Mg;
  l.alive = w.u.alive + bg * Mg;
  l.packed = w.u.packed + bg * Mg;
  l.restricted = w.u.restr + bg * Mg;
  l.limit = pass ? nullptr : w.u.limit + bg;
  int32_t* words = uwords(w, bg);
  l.count = words + (pass ? kUCountG : kUCountC);
  l.active = words + (pass ? kUActiveG : kUActiveC);
  l.merges = words + (pass ? kUMergesG : kUMergesC);
  l.stuck = w.u.stuck + bg * 2 + pass;
  l.trace = pass ? w.u.trace_g + bg * Mg * 2 : w.u.trace_c + bg * (size_t)g.NW * 2;
  l.M = (int)Mg;
  l.D = g.D;
  l.target = pass ? g.K : 1;
  l.passes = pass ? g.passes : 1;
  l.cost_order = 0;
  l.pass = pass;
  l.ties = logkv_ward::TieSink{&w.counters[kCntTies], reinterpret_cast<logkv_tie_t*>(w.ties), &w.counters[kCntFlushes],
                               kTieCap, (int)(bg / g.G), (int)(bg % g.G)};
  return l;
}

// Rows of a lane's pass: archived tokens (candidate pass) or live clusters + candidates.
__device__ __forceinline__ int upass_rows(const Geo& g, const Work& w, size_t bg, int b, int pass) {
  return pass ? uwords(w, bg)[kUGCount] : w.narch[b];
}

// ---------------------------------------------------------------- U0: the reference's lane tiles
// Lanes (b, g) of batch rows that archive tokens, in order, split into balanced tiles of at most
// 64 MiB / (4 * tokens^2) lanes (tokens = the widest row).  Per tile, the pass's matrix form
// follows from its widest active lane (rows > target): at most 32 rows -> exact differences.
// One block; dynamic shared memory B ints.
__global__ void __launch_bounds__(1024) unified_tile_kernel(Geo g, Work w, int pass) {
  pdl_entry();
  extern __shared__ int abatch[];   // [B] batch rows that archive tokens, in order
  __shared__ int nb, tokens;
  if (threadIdx.x == 0) {
    int n = 0, t = 0;
    for (int b = 0; b < g.B; ++b)
      if (w.narch[b] > 0) {
        abatch[n++] = b;
        t = max(t, w.narch[b]);
      }
    nb = n;
    tokens = t;
  }
  __syncthreads();
  const long long nl = (long long)nb * g.G;
  if (nl == 0) return;
  const long long tk = tokens;
  const long long widest = max(1ll, kUTileBytes / max(1ll, 4 * tk * tk));
  const long long tiles = (nl + widest - 1) / widest;
  const long long ts = max(1ll, (nl + max(tiles, 1ll) - 1) / max(tiles, 1ll));
  const int target = pass ? g.K : 1;
  for (long long t0 = (long long)threadIdx.x * ts; t0 < nl; t0 += (long long)blockDim.x * ts) {
    const long long t1 = min(nl, t0 + ts);
    int size = 0;
    for (long long j = t0; j < t1; ++j) {
      const int b = abatch[j / g.G], grp = (int)(j % g.G);
      const int rows = upass_rows(g, w, ulane(g, b, grp), b, pass);
      if (rows > target) size = max(size, rows);
    }
    for (long long j = t0; j < t1; ++j) {
      const int b = abatch[j / g.G], grp = (int)(j % g.G);
      uwords(w, ulane(g, b, grp))[pass ? kUCdistG : kUCdistC] = size > 0 && size <= 32;
    }
  }
}

// ---------------------------------------------------------------- U1: candidate pass inputs
// The lane's archived keys (archive rank order, = position order) as float32 centres of mass 1,
// its radius limit, and cleared lane words.  Grid (chunks, G, B).
template <typename T>
__global__ void __launch_bounds__(256) unified_load_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  const int b = blockIdx.z, grp = blockIdx.y, tid = threadIdx.x, nt = blockDim.x;
  const size_t bg = ulane(g, b, grp);
  const int n = w.narch[b], D = g.D, Mg = g.Mg;
  const int* arch = w.arch_idx + (size_t)b * g.NW;
  const T* snap = static_cast<const T*>(w.snap_k);
  const T* rec = static_cast<const T*>(s.recent_k_raw);
  float* mu = w.u.mu_c + bg * (size_t)g.NW * D;
  for (size_t item = (size_t)blockIdx.x * nt + tid; item < (size_t)n * D; item += (size_t)gridDim.x * nt) {
    const int t = (int)(item / D), d = (int)(item % D);
    mu[item] = Elem<T>::load(token_row<T>(g, snap, rec, b, grp, arch[t]) + d);
  }
  float* mass = w.u.mass + bg * Mg;
  for (int r = blockIdx.x * nt + tid; r < Mg; r += gridDim.x * nt) mass[r] = r < n ? 1.f : 0.f;
  if (blockIdx.x == 0 && tid < kULaneWords) {
    uwords(w, bg)[tid] = 0;
    if (tid == 0) {
      // float32(sqrt(lambda * s_h)), the root taken in double like the reference's host math.
      w.u.limit[bg] = (float)sqrt((double)g.lam * (double)s.s_h[bg]);
      w.u.stuck[bg * 2] = 0;
      w.u.stuck[bg * 2 + 1] = 0;
    }
  }
}

// ---------------------------------------------------------------- U2: pair matrix
// Upper-triangle output tiles of kGramTile x kGramTile (128 x 128) per CTA of 256 threads; the
// two centre panels are staged transposed ([kGramChunk][128] per feature chunk, c = x - x_0) and
// each thread owns 8 x 8 outputs (rows ty*4 + {0..3, 64..67}, columns tx*4 + {0..3, 64..67}, so a
// warp's 16-byte shared loads are conflict-free), accumulated over the features in order with one
// fused multiply-add each.  Norms n_i = sum_d c_id^2 run left to right across the chunks.
// Grid (tiles, tiles, B*G) x 256; dynamic shared memory: the output tile, 128 x 129 floats.
__global__ void __launch_bounds__(256) unified_dist_kernel(Geo g, Work w, int pass) {
  pdl_entry();
  const size_t bg = blockIdx.z;
  const int b = (int)(bg / g.G);
  const int n = upass_rows(g, w, bg, b, pass);
  const int ti = blockIdx.y, tj = blockIdx.x;
  if (n <= (pass ? g.K : 1) || ti > tj || ti * kGramTile >= n || tj * kGramTile >= n) return;
  const int D = g.D, Mg = g.Mg, tid = threadIdx.x;
  const float* mu = pass ? w.u.mu_g + bg * (size_t)Mg * D : w.u.mu_c + bg * (size_t)g.NW * D;
  float* dist = w.u.dist + bg * (size_t)Mg * Mg;
  const int i0 = ti * kGramTile, j0 = tj * kGramTile;
  if (uwords(w, bg)[pass ? kUCdistG : kUCdistC]) {
    // Exact differences (n <= 32: one tile): sqrt(sum (x - y)^2) rounded, then squared.
    for (int item = tid; item < n * n; item += blockDim.x) {
      const int i = item / n, j = item % n;
      if (i > j) continue;
      const float* xi = mu + (size_t)i * D;
      const float* xj = mu + (size_t)j * D;
      float acc = 0.f;
      for (int d = 0; d < D; ++d) {
        const float df = fsub(xi[d], xj[d]);
        acc = fadd(acc, fmul(df, df));
      }
      const float root = __fsqrt_rn(acc);
      const float v = fmul(root, root);
      dist[(size_t)i * Mg + j] = v;
      dist[(size_t)j * Mg + i] = v;
    }
    return;
  }
  // Gram form: c = x - x_0, n_i = sum_d c_id^2, d_ij = max((n_i + n_j) - 2 G_ij, 0).
  __shared__ __align__(16) float at[kGramChunk][kGramTile];   // rows i0.., chunk features
  __shared__ __align__(16) float bt[kGramChunk][kGramTile];   // rows j0..
  __shared__ float nrm[2][kGramTile];
  const float4* x0 = reinterpret_cast<const float4*>(mu);
  const int tx = tid & 15, ty = tid >> 4;
  float acc[8][8];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[r][c] = 0.f;
  float nacc = 0.f;   // thread t: the norm of row i0 + t (t < 128) or j0 + t - 128
  for (int d0 = 0; d0 < D; d0 += kGramChunk) {
    const int dn = min(kGramChunk, D - d0);   // a multiple of 4 (D % 4 == 0)
    // Stage: consecutive threads take consecutive rows (conflict-free transposed stores).
    for (int item = tid; item < kGramTile * (dn / 4); item += blockDim.x) {
      const int r = item % kGramTile, q = item / kGramTile;
      const int ri = i0 + r, rj = j0 + r;
      const float4 o = x0[d0 / 4 + q];
      const float4 a = ri < n ? reinterpret_cast<const float4*>(mu + (size_t)ri * D + d0)[q] : o;
      const float4 c = rj < n ? reinterpret_cast<const float4*>(mu + (size_t)rj * D + d0)[q] : o;
      at[4 * q + 0][r] = fsub(a.x, o.x);
      at[4 * q + 1][r] = fsub(a.y, o.y);
      at[4 * q + 2][r] = fsub(a.z, o.z);
      at[4 * q + 3][r] = fsub(a.w, o.w);
      bt[4 * q + 0][r] = fsub(c.x, o.x);
      bt[4 * q + 1][r] = fsub(c.y, o.y);
      bt[4 * q + 2][r] = fsub(c.z, o.z);
      bt[4 * q + 3][r] = fsub(c.w, o.w);
    }
    __syncthreads();
    {
      const float* col = tid < kGramTile ? &at[0][tid] : &bt[0][tid - kGramTile];
      for (int d = 0; d < dn; ++d) {
        const float v = col[d * kGramTile];
        nacc = fadd(nacc, fmul(v, v));
      }
    }
#pragma unroll 4
    for (int d = 0; d < dn; ++d) {
      const float4 a0 = *reinterpret_cast<const float4*>(&at[d][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&at[d][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&bt[d][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&bt[d][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[r][c] = __fmaf_rn(av[r], bv[c], acc[r][c]);
    }
    __syncthreads();
  }
  nrm[tid >> 7][tid & 127] = nacc;
  __syncthreads();
  // The finished tile through shared memory (row stride kGramTile + 1: a column read is
  // conflict-free), then both halves written with coalesced stores: rows i of columns j >= i, and
  // the mirror, rows j of columns i < j (the upper triangle's values, as the reference mirrors).
  extern __shared__ float tile[];   // [kGramTile][kGramTile + 1]
  constexpr int TS = kGramTile + 1;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int il = (r < 4 ? 0 : 64) + ty * 4 + (r & 3);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int jl = (c < 4 ? 0 : 64) + tx * 4 + (c & 3);
      tile[il * TS + jl] = fmaxf(fsub(fadd(nrm[0][il], nrm[1][jl]), fmul(2.f, acc[r][c])), 0.f);
    }
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  const int ni = min(kGramTile, n - i0), nj = min(kGramTile, n - j0);
  for (int il = warp; il < ni; il += 8) {
    const int i = i0 + il;
    for (int jl = lane; jl < nj; jl += 32)
      if (j0 + jl >= i) dist[(size_t)i * Mg + j0 + jl] = tile[il * TS + jl];
  }
  for (int jl = warp; jl < nj; jl += 8) {
    const int j = j0 + jl;
    for (int il = lane; il < ni; il += 32)
      if (i0 + il < j) dist[(size_t)j * Mg + i0 + il] = tile[il * TS + jl];
  }
}

// ---------------------------------------------------------------- U3: the rounds of one pass
// Every round of one lane in one launch, on a cluster of CL CTAs (unified_core.cuh; the cluster
// size is the launch's), until the lane has no proposal left or reaches its target.
// Grid (B*G * CL) x 1024.
__global__ void __launch_bounds__(logkv_ward::kUThreads) unified_reduce_kernel(Geo g, Work w, int pass, int S) {
  pdl_entry();
  namespace cg = cooperative_groups;
  extern __shared__ __align__(16) unsigned char usm[];
  __shared__ int act[2], n_sh;
  cg::cluster_group cluster = cg::this_cluster();
  const int part = (int)cluster.block_rank(), CL = (int)cluster.num_blocks();
  const size_t bg = blockIdx.x / CL;
  const int b = (int)(bg / g.G);
  const int n = upass_rows(g, w, bg, b, pass);
  const logkv_ward::RunLane l = urun(g, w, bg, pass);
  if (n <= l.target) return;   // the same in every CTA of the cluster
  if (part == 0 && threadIdx.x == 0) {
    *l.count = n;
    *l.active = 0;
    *l.merges = 0;
    *l.stuck = 0;
  }
  cluster.sync();
  logkv_ward::init_lane(l, part, CL, logkv_ward::carve_round(usm, l.M, S, CL).rows, &n_sh);
  cluster.sync();
  const int rounds = 2 * l.M + 7;   // every round but the last merges or pins a pair (a guard)
  int r = 0;
  while (r < rounds && logkv_ward::run_round(cluster, l, usm, S, act, r & 1)) ++r;
  if (part == 0 && threadIdx.x == 0) {
    uwords(w, bg)[pass ? kURoundsG : kURoundsC] = min(r + 1, rounds);
    if (pass == 1 && *l.stuck) set_status(w.status, kStatusBadCluster);
  }
  cluster.sync();   // the leader's flags stay readable until every CTA has read them
}

// Block-wide exclusive scan of one int per thread; returns the thread's offset and the total.
__device__ inline int ublock_scan(int v, int* total) {
  __shared__ int ws[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) ws[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < nw ? ws[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= off) s += y;
    }
    if (lane < nw) ws[lane] = s;
  }
  __syncthreads();
  const int excl = x - v + (warp ? ws[warp - 1] : 0);
  *total = ws[nw - 1];
  __syncthreads();
  return excl;
}

// Roots of a merge forest by pointer jumping: parent[right] = left for every trace pair (a right
// row is retired once, and its parent is a smaller row), then parent = parent[parent] until fixed.
// Survivors: rows [0, n) alive after the pass (every row when the pass did not run).  Writes
// comp[row] = compact index of the row's root among the survivors (ascending) and surv[k] = the
// k-th survivor; returns the survivor count.  Block-wide; parent, comp, surv are [n] shared.
__device__ inline int uforest(int n, const int32_t* trace, int merges, const uint8_t* alive, bool ran, int* parent,
                              int* comp, int* surv) {
  const int tid = threadIdx.x, nt = blockDim.x;
  __shared__ int changed;
  for (int r = tid; r < n; r += nt) parent[r] = r;
  __syncthreads();
  for (int m = tid; m < merges; m += nt) parent[trace[2 * m + 1]] = trace[2 * m];
  __syncthreads();
  // Every retired row's parent is a smaller row, so depths halve per step: 32 steps cover any
  // forest of fewer than 2^32 rows (the bound only guards against a malformed trace).
  for (int step = 0; step < 32; ++step) {
    if (tid == 0) changed = 0;
    __syncthreads();
    for (int r = tid; r < n; r += nt) {
      const int p = parent[r], pp = parent[p];
      if (pp != p) {
        parent[r] = pp;
        changed = 1;
      }
    }
    __syncthreads();
    if (!changed) break;
    __syncthreads();
  }
  // Compact survivor indices: per-thread contiguous row ranges, one block scan.
  const int per = (n + nt - 1) / nt, lo = min(n, tid * per), hi = min(n, lo + per);
  int cnt = 0;
  for (int r = lo; r < hi; ++r) cnt += !ran || alive[r];
  int total;
  int at = ublock_scan(cnt, &total);
  for (int r = lo; r < hi; ++r)
    if (!ran || alive[r]) {
      comp[r] = at;
      surv[at++] = r;
    }
  __syncthreads();
  for (int r = tid; r < n; r += nt) comp[r] = comp[parent[r]];
  __syncthreads();
  return total;
}

// ---------------------------------------------------------------- U4: candidate labels, global inputs
// Every archived token's candidate; the global pass's centres (live centroids, then the candidates'
// centres) and masses (n_total, then token counts).  Grid (G, B) x 1024; dynamic shared memory
// 3 * NW ints.
__global__ void __launch_bounds__(1024) unified_labels_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  const int b = blockIdx.y, grp = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const size_t bg = ulane(g, b, grp);
  const int n = w.narch[b], D = g.D, Mg = g.Mg, K = g.K;
  int32_t* words = uwords(w, bg);
  extern __shared__ int lsm[];
  int* parent = lsm;
  int* comp = parent + g.NW;
  int* surv = comp + g.NW;
  __shared__ int nold, olds[kMaxClusters];
  if (n == 0) {
    if (tid == 0) {
      words[kUGCount] = 0;
      words[kUOld] = 0;
      words[kUCand] = 0;
    }
    return;
  }
  const bool ran = n > 1;
  const int ncand = uforest(n, w.u.trace_c + bg * (size_t)g.NW * 2, ran ? words[kUMergesC] : 0,
                            w.u.alive + bg * Mg, ran, parent, comp, surv);
  int32_t* label = w.u.label + bg * g.NW;
  for (int t = tid; t < n; t += nt) label[t] = comp[t];
  if (tid == 0) {
    int c0 = 0;
    for (int c = 0; c < K; ++c)
      if (s.alive[bg * K + c]) olds[c0++] = c;
    nold = c0;
  }
  __syncthreads();
  // Token counts per candidate (parent[] reused as the histogram).
  for (int k = tid; k < ncand; k += nt) parent[k] = 0;
  __syncthreads();
  for (int t = tid; t < n; t += nt) atomicAdd(&parent[comp[t]], 1);
  __syncthreads();
  const int no = nold, gc = no + ncand;
  float* mu = w.u.mu_g + bg * (size_t)Mg * D;
  const float* muc = w.u.mu_c + bg * (size_t)g.NW * D;
  for (size_t item = tid; item < (size_t)gc * D; item += nt) {
    const int r = (int)(item / D), d = (int)(item % D);
    mu[item] = r < no ? s.centroid[(bg * K + olds[r]) * D + d] : muc[(size_t)surv[r - no] * D + d];
  }
  float* mass = w.u.mass + bg * Mg;
  for (int r = tid; r < Mg; r += nt)
    mass[r] = r < no ? (float)s.n_total[bg * K + olds[r]] : (r < gc ? (float)parent[r - no] : 0.f);
  int32_t* old = w.u.old + bg * K;
  for (int c = tid; c < K; c += nt) old[c] = c < no ? olds[c] : -1;
  if (tid == 0) {
    words[kUGCount] = gc;
    words[kUOld] = no;
    words[kUCand] = ncand;
  }
}

// ---------------------------------------------------------------- U5: route
// Global roots -> clusters: a root that is an old cluster keeps its slot, the other roots take the
// free slots (not alive, or freed by a Ward merge) in ascending order; merges of two old rows are
// the lane's Ward merges, in trace order.  Writes the cluster of every archived token in archive
// rank order (the plan kernel's input).  Grid (G, B) x 1024; dynamic shared memory 3 * Mg ints.
__global__ void __launch_bounds__(1024) unified_route_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  const int b = blockIdx.y, grp = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const size_t bg = ulane(g, b, grp);
  const int n = w.narch[b], K = g.K, Mg = g.Mg;
  int32_t* words = uwords(w, bg);
  if (n == 0) {
    if (tid == 0) words[kUWard] = 0;
    return;
  }
  extern __shared__ int rsm[];
  int* parent = rsm;
  int* comp = parent + Mg;
  int* surv = comp + Mg;
  __shared__ int target[kMaxClusters + 1];
  const int gc = words[kUGCount], no = words[kUOld];
  const bool ran = gc > K;
  const int32_t* trace = w.u.trace_g + bg * (size_t)Mg * 2;
  const int merges = ran ? words[kUMergesG] : 0;
  const int nroots = uforest(gc, trace, merges, w.u.alive + bg * Mg, ran, parent, comp, surv);
  const int32_t* old = w.u.old + bg * K;
  if (tid == 0) {
    int32_t* ward = w.u.ward + bg * (size_t)K * 2;
    unsigned freed = 0;
    int nw = 0;
    for (int m = 0; m < merges; ++m) {
      const int a = trace[2 * m], r = trace[2 * m + 1];
      if (r < no) {
        ward[2 * nw] = old[a];
        ward[2 * nw + 1] = old[r];
        ++nw;
        freed |= 1u << old[r];
      }
    }
    words[kUWard] = nw;
    int next = 0;   // next free slot candidate
    bool bad = nroots > K;
    for (int k = 0; k < nroots && k < K; ++k) {
      const int root = surv[k];
      if (root < no) {
        target[k] = old[root];
      } else {
        while (next < K && s.alive[bg * K + next] && !(freed >> next & 1u)) ++next;
        if (next >= K) {
          bad = true;
          target[k] = 0;
        } else {
          target[k] = next++;
        }
      }
    }
    if (bad) set_status(w.status, kStatusBadCluster);
  }
  __syncthreads();
  const int32_t* label = w.u.label + bg * g.NW;
  int8_t* asg = w.assign + bg * g.NW;
  for (int t = tid; t < n; t += nt) {
    const int k = comp[no + label[t]];
    asg[t] = (int8_t)(k < K ? target[k] : 0);
  }
}

// ---------------------------------------------------------------- U6: Ward merges
// The lane's Ward merges in order, one CTA per (batch, group): the keep and free clusters'
// entries (level by level, slots ascending) ordered like _semantic_ward_entry_index, staged in
// scratch buffer 0 with orders 0..n-1, both clusters cleared, the centroid the count-weighted
// mean of the two, and the entries appended to the empty keep ladder by the cascade's sequential
// walk.  Dynamic shared memory: the walk's (walk_bytes), then two sort arrays of cap entries.
template <typename T, bool BETA, int DC>
__global__ void __launch_bounds__(kCascadeThreads) unified_ward_kernel(Geo g, logkv_state_t s, Work w, int cap,
                                                                        size_t walk_bytes, uint8_t* ward_cuts) {
  pdl_entry();
  const int b = blockIdx.y, grp = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const size_t bg = ulane(g, b, grp);
  const int nw = w.narch[b] > 0 ? uwords(w, bg)[kUWard] : 0;
  if (nw == 0) return;
  extern __shared__ uint4 wsm4[];
  unsigned long long* k1 = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(wsm4) + walk_bytes);
  unsigned long long* k2 = k1 + cap;
  __shared__ int cnt[2][kMaxLevels + 1];
  const int K = g.K, L = g.L, D = DC ? DC : g.D;
  constexpr int VN = Vec<T>::N;
  const int DV = D / VN;
  auto bitonic = [&](unsigned long long* keys) {
    for (int k = 2; k <= cap; k <<= 1)
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < cap; i += nt) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const unsigned long long a = keys[i], c = keys[ixj];
            const bool up = (i & k) == 0;
            if ((a > c) == up) {
              keys[i] = c;
              keys[ixj] = a;
            }
          }
        }
        __syncthreads();
      }
  };
  for (int j = 0; j < nw; ++j) {
    const int keep = w.u.ward[(bg * K + j) * 2], free = w.u.ward[(bg * K + j) * 2 + 1];
    const size_t lk = bg * K + keep, lf = bg * K + free;
    if (tid < 2) {
      const size_t lane = tid ? lf : lk;
      int e = 0;
      for (int l = 0; l < L; ++l) {
        cnt[tid][l] = e;
        e += s.level_count[lane * L + l];
      }
      cnt[tid][L] = e;
    }
    __syncthreads();
    const int ek = cnt[0][L], n = ek + cnt[1][L];
    // Entry i: side (i >= ek), its level and slot, its ladder row.
    auto entry_row = [&](int i) -> size_t {
      const int side = i >= ek;
      const int e = side ? i - ek : i;
      int l = 0;
      while (l + 1 < L && cnt[side][l + 1] <= e) ++l;
      return ((side ? lf : lk) * L + l) * (size_t)g.Bs + (e - cnt[side][l]);
    };
    // 1. Each side stably sorted by level order (keys: side | order | entry).
    for (int i = tid; i < cap; i += nt)
      k1[i] = i < n ? ((unsigned long long)(i >= ek) << 62) | ((unsigned long long)s.level_order[entry_row(i)] << 16) |
                          (unsigned long long)i
                    : ~0ull;
    __syncthreads();
    bitonic(k1);
    // 2. Per side: effective key = p_lo of the next entry with mass at or after it (else its own
    // order), its running maximum; 3. the sides merged by it, keep side first on ties.
    if (tid < 2) {
      const int lo = tid ? ek : 0, hi = tid ? n : ek;
      long long next = -1;
      for (int p = hi - 1; p >= lo; --p) {
        const size_t row = entry_row((int)(k1[p] & 0xFFFFull));
        if (s.level_w[row] > 0.f) next = s.level_p_lo[row];
        k2[p] = (unsigned long long)(next >= 0 ? next : s.level_order[row]);
      }
      unsigned long long run = 0;
      for (int p = lo; p < hi; ++p) {
        run = p == lo ? k2[p] : max(run, k2[p]);
        k2[p] = (run << 16) | (unsigned long long)p;
      }
    }
    __syncthreads();
    for (int i = n + tid; i < cap; i += nt) k2[i] = ~0ull;
    __syncthreads();
    bitonic(k2);
    // 4. Stage the merged entries (orders 0..n-1) in scratch buffer 0 of this (b, g).
    T* SK = static_cast<T*>(w.sk);
    T* SV = static_cast<T*>(w.sv);
    const size_t srow0 = (bg * 2 + 0) * (size_t)g.S;
    for (int item = tid; item < n * DV; item += nt) {
      const int r = item / DV, v = item % DV;
      const size_t src = entry_row((int)(k1[k2[r] & 0xFFFFull] & 0xFFFFull));
      *reinterpret_cast<uint4*>(SK + (srow0 + r) * D + v * VN) =
          *reinterpret_cast<const uint4*>(static_cast<const T*>(s.level_k) + src * D + v * VN);
      *reinterpret_cast<uint4*>(SV + (srow0 + r) * D + v * VN) =
          *reinterpret_cast<const uint4*>(static_cast<const T*>(s.level_v) + src * D + v * VN);
    }
    for (int r = tid; r < n; r += nt) {
      const size_t src = entry_row((int)(k1[k2[r] & 0xFFFFull] & 0xFFFFull));
      const size_t dst = srow0 + r;
      w.sw[dst] = s.level_w[src];
      w.slo[dst] = s.level_p_lo[src];
      w.shi[dst] = s.level_p_hi[src];
      w.sswp[dst] = s.level_sum_wp[src];
      w.sord[dst] = r;
      w.spad[dst] = s.pad_mask[src];
    }
    // 5. Centroid and scalars (n_total as float32 weights, the reference's int64 -> float cast).
    const float nk = (float)s.n_total[lk], nf = (float)s.n_total[lf];
    for (int d = tid; d < D; d += nt) {
      float* mk = s.centroid + lk * D;
      const float* mf = s.centroid + lf * D;
      mk[d] = fdiv(fadd(fmul(nk, mk[d]), fmul(nf, mf[d])), fmaxf(fadd(nk, nf), 1.f));
    }
    __syncthreads();
    if (tid == 0) {
      s.n_eff[lk] = fadd(s.n_eff[lk], s.n_eff[lf]);
      s.n_eff[lf] = 0.f;
      s.n_total[lk] = s.n_total[lk] + s.n_total[lf];
      s.p_hi_c[lk] = max(s.p_hi_c[lk], s.p_hi_c[lf]);
      s.level0_phase[lk] = n;
      s.alive[lk] = 1;
      s.n_total[lf] = 0;
      s.p_hi_c[lf] = -1;
      s.level0_phase[lf] = 0;
      s.alive[lf] = 0;
      w.plan_type[lk] = kJobLate;
      w.plan_m0[lk] = n;
      w.plan_n[lk] = 0;
      w.plan_off[lk] = 0;
      w.plan_scr[lk] = 0;
      w.plan_base[lk] = 0;
    }
    // 6. Clear both clusters' levels.
    const size_t rows = (size_t)L * g.Bs;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    for (int side = 0; side < 2; ++side) {
      const size_t base = (side ? lf : lk) * L * (size_t)g.Bs;
      uint4* qk = reinterpret_cast<uint4*>(static_cast<T*>(s.level_k) + base * D);
      uint4* qv = reinterpret_cast<uint4*>(static_cast<T*>(s.level_v) + base * D);
      for (size_t i = tid; i < rows * DV; i += nt) {
        qk[i] = zero;
        qv[i] = zero;
      }
      for (size_t r = tid; r < rows; r += nt) {
        s.level_w[base + r] = 0.f;
        s.level_p_lo[base + r] = 0;
        s.level_p_hi[base + r] = 0;
        s.level_sum_wp[base + r] = 0;
        s.level_order[base + r] = 0;
        s.pad_mask[base + r] = 0;
      }
      for (int l = tid; l < L; l += nt) s.level_count[(side ? lf : lk) * L + l] = 0;
    }
    __syncthreads();
    // 7. Append the staged entries to the empty keep ladder (an update tape keeps this rebuild's
    // Beta cuts in its own slot, merge j of lane (b, g)).
    const LaneCtx<T> x = make_ctx_at<T>(g, s, w, keep, grp, b);
    Work wj = w;
    if (g.tape != kTapeNone) {
      wj.tape_cuts = ward_cuts;
      wj.tape_cut_lane = (long long)(bg * K + j);
    }
    cascade_walk<T, BETA, DC, kTileRows>(x, g, s, wj);
    __syncthreads();
  }
}

}  // namespace logkv
