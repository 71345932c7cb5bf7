// Alpha exact-span pool on the device: snapshot, span cut, span scores, greedy choice.
//
// Follows litgpt/alpha_log_kv.py (_new_runs :16-53, cut_spans :84-122,
// score_spans :125-174, choose_spans :177-226) and the pool rewrite of
// _alpha_route_flush (litgpt/log_kv_cache.py:3903-4003).  Token index space of
// one batch row: [0, P) = old pool rows (compacted, kept spans in pool order),
// [P, P + F) = the flushed window tokens.
#pragma once

#include "flush_common.cuh"

namespace logkv {

// ---------------------------------------------------------------- K0: snapshot
// Copies the old exact pool so the pool can be rewritten in place later, and
// resets the status word and the device alpha_count.
template <typename T>
__global__ void snapshot_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  const int b = blockIdx.z, grp = blockIdx.y;
  const size_t n = (size_t)g.P * g.D / Vec<T>::N;  // 16-byte units (rows are whole units)
  const uint4* ksrc = static_cast<const uint4*>(s.alpha_k_raw) + ((size_t)b * g.G + grp) * n;
  const uint4* vsrc = static_cast<const uint4*>(s.alpha_v) + ((size_t)b * g.G + grp) * n;
  uint4* kdst = static_cast<uint4*>(w.snap_k) + ((size_t)b * g.G + grp) * n;
  uint4* vdst = static_cast<uint4*>(w.snap_v) + ((size_t)b * g.G + grp) * n;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    kdst[i] = ksrc[i];
    vdst[i] = vsrc[i];
  }
  if (blockIdx.x == 0) {
    // Squared norms of the lane's frozen centres (attach and Beta novelty read them).
    const size_t lane0 = ((size_t)b * g.G + grp) * g.K;
    for (int c = threadIdx.x; c < g.K; c += blockDim.x) {
      const float4* mu = reinterpret_cast<const float4*>(s.centroid + (lane0 + c) * g.D);  // D % 4 == 0
      float mm = 0.f;
#pragma unroll 4
      for (int d4 = 0; d4 < g.D / 4; ++d4) {
        const float4 v = mu[d4];
        mm = fadd(mm, fmul(v.x, v.x));
        mm = fadd(mm, fmul(v.y, v.y));
        mm = fadd(mm, fmul(v.z, v.z));
        mm = fadd(mm, fmul(v.w, v.w));
      }
      w.cnorm[lane0 + c] = mm;
    }
  }
  if (grp == 0 && blockIdx.x == 0) {
    for (int i = threadIdx.x; i < g.P; i += blockDim.x) w.snap_pos[(size_t)b * g.P + i] = s.alpha_pos[(size_t)b * g.P + i];
    // Positions of the whole [old pool | flushed window] index space, as the flush starts.
    for (int i = threadIdx.x; i < g.NW; i += blockDim.x)
      w.tok_pos[(size_t)b * g.NW + i] =
          i < g.P ? s.alpha_pos[(size_t)b * g.P + i] : s.recent_pos[(size_t)b * g.cap2R + (i - g.P)];
    if (threadIdx.x == 0) {
      w.snap_rowcount[b] = s.alpha_rowcount[b];
      if (b == 0) {
        *w.status = 0;
        w.counters[kCntFlushes] += 1ull;
      }
    }
  }
}

// ---------------------------------------------------------------- K1: span cut
// One block (1024 threads) per batch row.  Candidates, in the reference's
// order: closed old spans (pool order), the old unfinished span if a
// position jump closed it, then the runs of the new tokens (the first one
// continuing the unfinished span), or the unfinished span alone when no new
// token arrived.
__global__ void __launch_bounds__(1024) alpha_cut_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  const int b = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const int P = g.P, F = g.F, cap = g.span_cap;
  __shared__ int wsum[32];
  __shared__ int sh_pend_idx, sh_n_closed, sh_nruns;
  extern __shared__ int run_end[];  // [F]
  const int nsp = s.alpha_nspans[b];
  if (tid == 0) sh_pend_idx = -1;
  __syncthreads();
  // Old spans: offsets and closed-candidate slots via block scans (chunked over P).
  int carry_off = 0, carry_closed = 0;
  for (int base = 0; base < nsp; base += nt) {
    const int i = base + tid;
    const int len = i < nsp ? s.alpha_span_len[(size_t)b * P + i] : 0;
    const int closed = i < nsp ? (int)s.alpha_span_closed[(size_t)b * P + i] : 0;
    const int off_incl = block_inclusive_scan(len, wsum);
    const int cl_incl = block_inclusive_scan(i < nsp && closed ? 1 : 0, wsum);
    if (i < nsp) {
      const int off = carry_off + off_incl - len;
      if (closed) {
        const int c = carry_closed + cl_incl - 1;
        w.cand_s0[(size_t)b * g.NC + c] = off;
        w.cand_n0[(size_t)b * g.NC + c] = len;
        w.cand_s1[(size_t)b * g.NC + c] = 0;
        w.cand_n1[(size_t)b * g.NC + c] = 0;
        w.cand_flags[(size_t)b * g.NC + c] = 3;  // old | closed
      } else {
        atomicMax(&sh_pend_idx, i);
      }
    }
    // broadcast the chunk totals
    __shared__ int tot_off, tot_cl;
    if (tid == nt - 1) {
      tot_off = off_incl;
      tot_cl = cl_incl;
    }
    __syncthreads();
    carry_off += tot_off;
    carry_closed += tot_cl;
    __syncthreads();
  }
  if (tid == 0) sh_n_closed = carry_closed;
  // Pending (unfinished) span: its offset is the sum of lengths before it.
  __shared__ int sh_pend_off, sh_pend_len;
  __shared__ long long sh_pend_pos;
  if (tid == 0) {
    sh_pend_off = 0;
    sh_pend_len = 0;
    sh_pend_pos = 0;
    const int pi = sh_pend_idx;
    if (pi >= 0) {
      int off = 0;
      for (int i = 0; i < pi; ++i) off += s.alpha_span_len[(size_t)b * P + i];
      sh_pend_off = off;
      sh_pend_len = s.alpha_span_len[(size_t)b * P + pi];
      if (sh_pend_len > 0) sh_pend_pos = w.snap_pos[(size_t)b * P + off + sh_pend_len - 1];
    }
  }
  __syncthreads();
  const int pend_len = sh_pend_len, pend_off = sh_pend_off;
  const int64_t* pos = s.recent_pos + (size_t)b * g.cap2R;
  const uint8_t* ends = s.recent_ends + (size_t)b * g.cap2R;
  const bool pclosed = pend_len > 0 && F > 0 && pos[0] != (int64_t)sh_pend_pos + 1;
  const int prefix = pclosed ? 0 : pend_len;
  // New runs: each thread owns a contiguous chunk of tokens.
  const int per = (F + nt - 1) / nt;
  const int lo = tid * per, hi = min(F, lo + per);
  // segment start = last token <= i that starts a segment (jump or boundary before it).
  int local_start = -1;
  for (int i = lo; i < hi; ++i) {
    const bool first = i == 0 || pos[i] != pos[i - 1] + 1 || ends[i - 1];
    if (first) local_start = i;
  }
  // inclusive max-scan over threads of local_start
  __shared__ int seg_carry[1024];
  seg_carry[tid] = local_start;
  __syncthreads();
  for (int off = 1; off < nt; off <<= 1) {
    int v = seg_carry[tid];
    if (tid >= off) v = max(v, seg_carry[tid - off]);
    __syncthreads();
    seg_carry[tid] = v;
    __syncthreads();
  }
  int seg_start = tid > 0 ? seg_carry[tid - 1] : -1;
  int nstops = 0;
  uint32_t stop_mask = 0, closed_mask = 0;
  for (int i = lo; i < hi; ++i) {
    const bool first = i == 0 || pos[i] != pos[i - 1] + 1 || ends[i - 1];
    if (first) seg_start = i;
    const bool seg0 = seg_start == 0;
    const int filled = i - seg_start + (seg0 ? prefix : 0) + 1;
    bool capc = filled % cap == 0;
    if (prefix >= cap && seg0) capc = false;
    const bool close = ends[i] != 0 || capc;
    const bool jump_next = i + 1 < F && pos[i + 1] != pos[i] + 1;
    const bool stop = close || jump_next || i == F - 1;
    if (stop) {
      stop_mask |= 1u << (i - lo);
      if (close || jump_next) closed_mask |= 1u << (i - lo);
      ++nstops;
    }
  }
  const int incl = block_inclusive_scan(nstops, wsum);
  int r = incl - nstops;
  int* run_closed = run_end + F;
  for (int i = lo; i < hi; ++i)
    if (stop_mask & (1u << (i - lo))) {
      run_closed[r] = (closed_mask >> (i - lo)) & 1u;
      run_end[r++] = i + 1;
    }
  if (tid == nt - 1) sh_nruns = incl;
  __syncthreads();
  const int nruns = sh_nruns;
  const int base = sh_n_closed + (pclosed ? 1 : 0);
  if (tid == 0 && pclosed) {
    const size_t c = (size_t)b * g.NC + sh_n_closed;
    w.cand_s0[c] = pend_off;
    w.cand_n0[c] = pend_len;
    w.cand_s1[c] = 0;
    w.cand_n1[c] = 0;
    w.cand_flags[c] = 2;  // closed, not old
  }
  // run -> candidate
  for (int rr = tid; rr < nruns; rr += nt) {
    const int stop = run_end[rr];
    const int start = rr == 0 ? 0 : run_end[rr - 1];
    const size_t c = (size_t)b * g.NC + base + rr;
    if (rr == 0 && pend_len > 0 && !pclosed) {
      w.cand_s0[c] = pend_off;
      w.cand_n0[c] = pend_len;
      w.cand_s1[c] = P + start;
      w.cand_n1[c] = stop - start;
    } else {
      w.cand_s0[c] = P + start;
      w.cand_n0[c] = stop - start;
      w.cand_s1[c] = 0;
      w.cand_n1[c] = 0;
    }
    w.cand_flags[c] = run_closed[rr] ? 2 : 0;
  }
  if (tid == 0) {
    int total = base + nruns;
    if (pend_len > 0 && !pclosed && nruns == 0) {
      const size_t c = (size_t)b * g.NC + base;
      w.cand_s0[c] = pend_off;
      w.cand_n0[c] = pend_len;
      w.cand_s1[c] = 0;
      w.cand_n1[c] = 0;
      w.cand_flags[c] = 0;
      total += 1;
    }
    w.n_cand[b] = total;
  }
}

// ---------------------------------------------------------------- K2: span scores
// One warp per (candidate, group) pair, no block-wide barriers.  The warp copies the span's
// K and V rows into its own shared memory, up to score_rows() tokens per pass (cp.async, all
// copies in flight at once; 16-byte chunks XOR-swizzled by token so that per-token and
// per-feature walks are conflict-free), then per component: the mean of every feature (lanes
// own 4 consecutive features and walk the tokens in order), the energy of every token (lanes
// own tokens and walk the features in order), their sum in token order, and the mean square
// of the mean vector; with Beta, the novelty of the key mean against every live centre (lanes
// own centres).  Every sum runs left to right, as the reference's CPU path.  Output per
// (row, candidate, group): Alpha parts (R_K, R_V) or Beta's per-group score.
__host__ __device__ inline int score_rows(int D, int esize) {
  // 24 rows of D = 128 bf16 per pass (a typical span in one pass) keep a block's staging
  // near 107 KB, so two 8-warp blocks share an SM.
  const int r = 6144 / (D * esize);
  return r < 1 ? 1 : (r > 32 ? 32 : r);
}
// Per-warp shared memory in floats: rows [2][rows][D] (storage dtype), means [2][D], token
// energies [2][32], centre distances [K].
__host__ __device__ inline int score_warp_floats(int D, int K, int esize) {
  return (2 * score_rows(D, esize) * D * esize / 4 + 2 * D + 64 + K + 3) & ~3;
}

// Four consecutive staged elements (8 or 16 bytes, aligned) as floats, in order.
__device__ __forceinline__ void load4(const float* p, float* out) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  out[0] = v.x;
  out[1] = v.y;
  out[2] = v.z;
  out[3] = v.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float* out) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  out[0] = __uint_as_float(v.x << 16);
  out[1] = __uint_as_float(v.x & 0xFFFF0000u);
  out[2] = __uint_as_float(v.y << 16);
  out[3] = __uint_as_float(v.y & 0xFFFF0000u);
}

template <typename T, int DC>
__device__ void score_pair(const Geo& g, const logkv_state_t& s, const Work& w, int b, int ci, int grp, int lane,
                           float* ws) {
  const int D = DC ? DC : g.D, K = g.K, G = g.G;
  constexpr int VN = Vec<T>::N;
  const int DV = D / VN;                                    // 16-byte chunks per row
  const int swz = (DV & (DV - 1)) == 0 ? min(DV, 16) - 1 : 0;  // chunk swizzle mask
  const int CR = score_rows(D, (int)sizeof(T));
  T* rows = reinterpret_cast<T*>(ws);                       // [2][CR][D]
  float* mean_s = ws + 2 * CR * D * (int)sizeof(T) / 4;    // [2][D] partial sums, then means
  float* etok_s = mean_s + 2 * D;                           // [2][32]
  float* cd_s = etok_s + 64;                                // [K]
  const size_t cix = (size_t)b * g.NC + ci;
  const int s0 = w.cand_s0[cix], n0 = w.cand_n0[cix], s1 = w.cand_s1[cix], n1 = w.cand_n1[cix];
  const int n = n0 + n1;
  const float fn = (float)n;
  const T* snapk = static_cast<const T*>(w.snap_k);
  const T* snapv = static_cast<const T*>(w.snap_v);
  const T* reck = static_cast<const T*>(s.recent_k_raw);
  const T* recv = static_cast<const T*>(s.recent_v);
  // Element (t, d) of staged component f: chunk d / VN of row t sits at chunk (d / VN) ^ (t & swz).
  float eacc[2] = {0.f, 0.f};
  for (int t0 = 0; t0 < n; t0 += CR) {
    const int cn = min(CR, n - t0);
    for (int item = lane; item < 2 * cn * DV; item += 32) {
      const int f = item >= cn * DV ? 1 : 0, r = item - f * cn * DV, t = r / DV, c = r % DV;
      const int tt = t0 + t;
      const int src = tt < n0 ? s0 + tt : s1 + (tt - n0);
      const T* row = f ? token_row<T>(g, snapv, recv, b, grp, src) : token_row<T>(g, snapk, reck, b, grp, src);
      cp_async16(rows + ((size_t)f * CR + t) * D + ((c ^ (t & swz)) * VN), row + c * VN);
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncwarp();
#pragma unroll
    for (int f = 0; f < 2; ++f) {
      // Mean partial sums: lane owns features f0 + 4 lane .. + 3, tokens in order.
      for (int f0 = 0; f0 < D; f0 += 128) {
        const int d = f0 + 4 * lane;
        if (d >= D) continue;
        float* ms = mean_s + f * D + d;
        float a0 = t0 ? ms[0] : 0.f, a1 = t0 ? ms[1] : 0.f, a2 = t0 ? ms[2] : 0.f, a3 = t0 ? ms[3] : 0.f;
        // 4 consecutive features never straddle a chunk: one 8- or 16-byte load per token.
        const T* fbase = rows + (size_t)f * CR * D + d % VN;
        const int dc = d / VN;
#pragma unroll 8
        for (int t = 0; t < cn; ++t) {
          float x4[4];
          load4(fbase + t * D + ((dc ^ (t & swz)) * VN), x4);
          a0 = fadd(a0, x4[0]);
          a1 = fadd(a1, x4[1]);
          a2 = fadd(a2, x4[2]);
          a3 = fadd(a3, x4[3]);
        }
        ms[0] = a0;
        ms[1] = a1;
        ms[2] = a2;
        ms[3] = a3;
      }
      // Energies: lane owns a token, features in order.
      if (lane < cn) {
        float e = 0.f;
#pragma unroll 4
        for (int c = 0; c < DV; ++c) {
          float x[VN];
          unpack(*reinterpret_cast<const uint4*>(rows + ((size_t)f * CR + lane) * D + ((c ^ (lane & swz)) * VN)), x,
                 (const T*)nullptr);
#pragma unroll
          for (int j = 0; j < VN; ++j) e = fadd(e, fmul(x[j], x[j]));
        }
        etok_s[f * 32 + lane] = fdiv(e, (float)D);
      }
    }
    __syncwarp();
    if (lane == 0)
      for (int f = 0; f < 2; ++f)
        for (int k = 0; k < cn; ++k) eacc[f] = fadd(eacc[f], etok_s[f * 32 + k]);
    __syncwarp();
  }
  for (int f = 0; f < 2; ++f)
    for (int d = 4 * lane; d < D; d += 128)
#pragma unroll
      for (int j = 0; j < 4; ++j) mean_s[f * D + d + j] = fdiv(mean_s[f * D + d + j], fn);
  __syncwarp();
  float part[2] = {0.f, 0.f}, ener0 = 0.f, kms = 0.f;
  if (lane == 0) {
#pragma unroll
    for (int f = 0; f < 2; ++f) {
      const float energy = fdiv(eacc[f], fn);
      const float* mc = mean_s + f * D;
      float ms = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) ms = fadd(ms, fmul(mc[d], mc[d]));
      ms = fdiv(ms, (float)D);
      part[f] = fdiv(fmaxf(fsub(energy, ms), 0.f), fmaxf(energy, 1e-12f));
      if (f == 0) {
        ener0 = energy;
        kms = ms;
      }
    }
  }
  float* out = w.gpart + (cix * G + grp) * 2;
  if (!g.beta) {
    if (lane == 0) {
      out[0] = part[0];
      out[1] = part[1];
    }
    return;
  }
  // Beta novelty: mean-square distance of the key mean to every live centre (lane owns a centre).
  kms = __shfl_sync(0xffffffffu, kms, 0);
  const size_t lane0 = ((size_t)b * G + grp) * K;
  for (int c = lane; c < K; c += 32) {
    float dist = INFINITY;
    if (s.alive[lane0 + c]) {
      const float4* mu = reinterpret_cast<const float4*>(s.centroid + (lane0 + c) * D);  // D % 4 == 0
      float dot = 0.f;
#pragma unroll 8
      for (int d4 = 0; d4 < D / 4; ++d4) {
        const float4 m = mu[d4];
        dot = fadd(dot, fmul(mean_s[4 * d4], m.x));
        dot = fadd(dot, fmul(mean_s[4 * d4 + 1], m.y));
        dot = fadd(dot, fmul(mean_s[4 * d4 + 2], m.z));
        dot = fadd(dot, fmul(mean_s[4 * d4 + 3], m.w));
      }
      dot = fdiv(dot, (float)D);
      dist = fmaxf(fsub(fadd(kms, fdiv(w.cnorm[lane0 + c], (float)D)), fmul(2.f, dot)), 0.f);
    }
    cd_s[c] = dist;
  }
  __syncwarp();
  if (lane == 0) {
    bool any = false;
    float nr = INFINITY;
    for (int c = 0; c < K; ++c) {
      any |= s.alive[lane0 + c] != 0;
      nr = fminf(nr, cd_s[c]);
    }
    if (!any) nr = 0.f;
    const float nov = fdiv(nr, fmaxf(ener0, 1e-12f));
    out[0] = fadd(fmul(fadd(part[0], part[1]), 0.5f), fdiv(nov, fadd(1.f, nov)));
  }
}

// ---------------------------------------------------------------- K3: greedy choice
// Sort helpers: the reference sorts Python tuples; ties are impossible because
// the index is part of every key.
__device__ __forceinline__ bool victim_less(double da, int ia, double db, int ib) {
  return da < db || (da == db && ia > ib);  // (density, -i) ascending
}
__device__ __forceinline__ bool ranked_less(double da, int ia, double db, int ib) {
  return da > db || (da == db && ia < ib);  // (-density, i) ascending
}
// Near tie of two float64 values (relative gap below the tie-log threshold), division-free.
__device__ __forceinline__ bool near_tie_d(double a, double b) {
  return fabs(a - b) < (double)kTieRel * fmax(fabs(a), fabs(b));
}
__device__ __forceinline__ float rel_gap_d(double a, double b) {
  const double den = fmax(fabs(a), fabs(b));
  return den > 0.0 ? (float)(fabs(a - b) / den) : 0.f;
}

__global__ void __launch_bounds__(1024) alpha_choose_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  const int b = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const int NC = g.NC, P = g.P;
  extern __shared__ unsigned char smraw[];
  const int VC = P + 1;                                      // victims never exceed P (each >= 1 token)
  double* dens = reinterpret_cast<double*>(smraw);           // [NC]
  double* vd = dens + NC;                                    // [2][VC] victim densities (ping-pong)
  int* size = reinterpret_cast<int*>(vd + 2 * VC);           // [NC]
  int* ranked = size + NC;                                   // [NC]
  int* vs = ranked + NC;                                     // [2][VC] victim sizes
  int* vi = vs + 2 * VC;                                     // [2][VC] victim candidate indices
  double* pls = reinterpret_cast<double*>(vi + 2 * VC);      // [VC] loss prefix, left to right
  int* psz = reinterpret_cast<int*>(pls + VC);               // [VC] inclusive size prefix
  double* swap_a = reinterpret_cast<double*>(psz + VC + (VC & 1));  // [NC] density * length of a swap test
  double* swap_b = swap_a + NC;                              // [NC] the victims' loss it was tested against
  int* uni = reinterpret_cast<int*>(swap_b + NC);            // [NC] closed candidates by (density, index)
  unsigned char* flags = reinterpret_cast<unsigned char*>(uni + NC);  // [NC]
  unsigned char* chosen = flags + NC;                        // [NC]
  unsigned char* swap_t = chosen + NC;                       // [NC] 0 untested, 1 rejected, 2 taken
  __shared__ int wsum[32];
  __shared__ int sh_nv, sh_nr, sh_room;
  if (tid == 0) {
    sh_nv = 0;
    sh_nr = 0;
    sh_room = P;
  }
  __syncthreads();
  const int n = w.n_cand[b];
  for (int i = tid; i < n; i += nt) {
    const size_t c = (size_t)b * NC + i;
    flags[i] = w.cand_flags[c];
    size[i] = w.cand_n0[c] + w.cand_n1[c];
    // Group parts in global group order: this rank's own, or all ranks' gathered parts.
    const int GT = g.G * g.shard_ranks;
    auto part = [&](int grp, int k) -> float {
      if (!w.gpart_all) return w.gpart[((size_t)c * g.G + grp) * 2 + k];
      const int r = grp / g.G, gl = grp % g.G;
      return w.gpart_all[(size_t)r * g.gpart_stride + (((size_t)b * NC + i) * g.G + gl) * 2 + k];
    };
    float sf;
    if (!g.beta) {
      float a = 0.f, v = 0.f;
      for (int grp = 0; grp < GT; ++grp) a = fadd(a, part(grp, 0));
      for (int grp = 0; grp < GT; ++grp) v = fadd(v, part(grp, 1));
      sf = fadd(fdiv(a, (float)GT), fdiv(v, (float)GT));
    } else {
      float v1 = -INFINITY, v2 = -INFINITY;
      for (int grp = 0; grp < GT; ++grp) {
        const float xg = part(grp, 0);
        if (xg > v1) {
          v2 = v1;
          v1 = xg;
        } else if (xg > v2) {
          v2 = xg;
        }
      }
      const int top = GT < 2 ? GT : 2;
      float acc = fadd(0.f, v1);
      if (top == 2) acc = fadd(acc, v2);
      sf = fdiv(acc, (float)top);
    }
    w.scores[c] = sf;
    const double sc = (double)sf;
    dens[i] = (flags[i] & 1) ? sc * 1.1 : sc * 1.0;
    chosen[i] = (!(flags[i] & 2)) || (flags[i] & 1);  // mandatory (open) or old
    swap_t[i] = 0;
  }
  __syncthreads();
  // room = budget - sizes of mandatory and old spans; victim count (integers, any order)
  for (int i = tid; i < n; i += nt) {
    if (chosen[i]) atomicSub(&sh_room, size[i]);
    if (chosen[i] && (flags[i] & 2)) atomicAdd(&sh_nv, 1);
  }
  // victims = chosen and not mandatory, sorted by (density, -i)
  for (int i = tid; i < n; i += nt) {
    if (chosen[i] && (flags[i] & 2)) {
      int rank = 0;
      for (int j = 0; j < n; ++j)
        if (j != i && chosen[j] && (flags[j] & 2) && victim_less(dens[j], j, dens[i], i)) ++rank;
      vd[rank] = dens[i];
      vs[rank] = size[i];
      vi[rank] = i;
    }
  }
  __syncthreads();
  // Make room for the bounded unfinished tail first (victims in order): remove the shortest
  // prefix of the sorted victims after which room >= 0 (one warp; exact integer prefix scan).
  if (tid < 32 && sh_room < 0) {
    const int lane = tid;
    const unsigned full = 0xffffffffu;
    const int nv = sh_nv;
    int acc = sh_room, k = nv;
    for (int c0 = 0; c0 < nv; c0 += 32) {
      const int j = c0 + lane;
      int incl = j < nv ? vs[j] : 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(full, incl, off);
        if (lane >= off) incl += y;
      }
      const unsigned hit = __ballot_sync(full, j < nv && acc + incl >= 0);
      if (hit) {
        const int f = __ffs(hit) - 1;
        k = c0 + f + 1;
        acc += __shfl_sync(full, incl, f);
        break;
      }
      acc += __shfl_sync(full, incl, 31);
    }
    for (int j = lane; j < k; j += 32) chosen[vi[j]] = 0;
    for (int j = lane; j < nv - k; j += 32) {   // victims [k, nv) -> buffer 1 at [0, nv - k)
      vd[VC + j] = vd[k + j];
      vs[VC + j] = vs[k + j];
      vi[VC + j] = vi[k + j];
    }
    __syncwarp();
    for (int j = lane; j < nv - k; j += 32) {
      vd[j] = vd[VC + j];
      vs[j] = vs[VC + j];
      vi[j] = vi[VC + j];
    }
    if (lane == 0) {
      sh_nv = nv - k;
      sh_room = acc;
    }
  }
  __syncthreads();
  // ranked = not chosen (removed victims included), sorted by (-density, i)
  for (int i = tid; i < n; i += nt) {
    if (chosen[i]) continue;
    atomicAdd(&sh_nr, 1);
    int rank = 0;
    for (int j = 0; j < n; ++j)
      if (j != i && !chosen[j] && ranked_less(dens[j], j, dens[i], i)) ++rank;
    ranked[rank] = i;
  }
  __syncthreads();

  // Bounded greedy (alpha_log_kv.choose_spans) in one warp.  The number of victims a
  // candidate needs comes from an exact integer prefix scan of victim sizes; the float64
  // loss over exactly those victims is the loss prefix summed by lane 0 in the reference's
  // order.  The walk takes candidates 32 at a time: a rejection leaves the victim list as it
  // was, so the warp's lanes test 32 consecutive candidates against the current list at once,
  // and only the first one taken changes it (the walk then goes on right after it).
  if (tid < 32) {
    const int lane = tid;
    const unsigned full = 0xffffffffu;
    int cur = 0, nv = sh_nv, room = sh_room;
    const int nr = sh_nr;
    // Prefixes of the current victim list: inclusive sizes (exact integers, warp scan) and
    // the float64 loss sum(density * size) added left to right from 0.0 (lane 0), so any
    // prefix equals the reference's running `loss` after that many removals.
    auto prefixes = [&]() {
      int carry = 0;
      for (int c0 = 0; c0 < nv; c0 += 32) {
        const int j = c0 + lane;
        int incl = j < nv ? vs[cur * VC + j] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int y = __shfl_up_sync(full, incl, off);
          if (lane >= off) incl += y;
        }
        if (j < nv) psz[j] = carry + incl;
        carry += __shfl_sync(full, incl, 31);
      }
      if (lane == 0) {
        double acc = 0.0;
        for (int j = 0; j < nv; ++j) {
          acc += vd[cur * VC + j] * (double)vs[cur * VC + j];
          pls[j] = acc;
        }
      }
      __syncwarp();
    };
    // Remove the first k victims and insert (di, length, i) at its sorted place.
    auto rebuild = [&](int k, double di, int length, int i) {
      const bool ins = true;
      for (int j = lane; j < k; j += 32) chosen[vi[cur * VC + j]] = 0;
      int at = 0;
      if (ins)
        for (int c0 = k; c0 < nv; c0 += 32) {
          const int j = c0 + lane;
          at += __popc(__ballot_sync(full, j < nv && victim_less(vd[cur * VC + j], vi[cur * VC + j], di, i)));
        }
      const int nn = nv - k + (ins ? 1 : 0), nx = cur ^ 1;
      for (int j = lane; j < nn; j += 32) {
        int src = -1;
        if (!ins) src = k + j;
        else if (j < at) src = k + j;
        else if (j > at) src = k + j - 1;
        if (src >= 0) {
          vd[nx * VC + j] = vd[cur * VC + src];
          vs[nx * VC + j] = vs[cur * VC + src];
          vi[nx * VC + j] = vi[cur * VC + src];
        } else {
          vd[nx * VC + j] = di;
          vs[nx * VC + j] = length;
          vi[nx * VC + j] = i;
        }
      }
      __syncwarp();
      cur = nx;
      nv = nn;
      prefixes();
    };
    prefixes();
    int q = 0;
    while (q < nr) {
      const int j = q + lane;
      int i = 0, length = 0, nrem = 0, avail = room;
      double di = 0.0;
      bool take = false, tested = false;
      if (j < nr) {
        i = ranked[j];
        di = dens[i];
        length = size[i];
        if (room >= length) {
          take = true;
        } else if (nv > 0 && room + psz[nv - 1] >= length) {
          int lo = 0, hi = nv - 1;   // first victim index with room + psz >= length
          while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (room + psz[mid] >= length) hi = mid;
            else lo = mid + 1;
          }
          nrem = lo + 1;
          avail = room + psz[lo];
          take = di * (double)length > pls[lo];
          tested = true;
        }
      }
      const unsigned hit = __ballot_sync(full, take);
      const int f = hit ? __ffs(hit) - 1 : 32;   // first candidate taken in this chunk (32: none)
      if (tested && lane <= f) {   // the candidates decided here; checked for near ties after the walk
        swap_a[i] = di * (double)length;
        swap_b[i] = pls[nrem - 1];
        swap_t[i] = take ? 2 : 1;
      }
      if (!hit) {
        q += 32;
        continue;
      }
      const int ti = __shfl_sync(full, i, f), tlen = __shfl_sync(full, length, f);
      const int trem = __shfl_sync(full, nrem, f), tavail = __shfl_sync(full, avail, f);
      const double tdi = __shfl_sync(full, di, f);
      if (lane == 0) chosen[ti] = 1;
      rebuild(trem, tdi, tlen, ti);
      room = tavail - tlen;
      q += f + 1;
    }
  }
  // Near ties of the walk, logged after it.  Every density comparison of the greedy (the victim
  // and candidate orders, a victim's insertion among the others) is between two closed spans;
  // two near-equal densities are neighbours in the closed spans' (density, index) order.
  for (int i = tid; i < n; i += nt) {
    if (!(flags[i] & 2)) continue;
    int rank = 0;
    for (int j = 0; j < n; ++j)
      if ((flags[j] & 2) && victim_less(dens[j], j, dens[i], i)) ++rank;
    uni[rank] = i;
  }
  __syncthreads();
  int nclosed = 0;
  for (int i = 0; i < n; ++i) nclosed += (flags[i] & 2) ? 1 : 0;
  for (int r = tid; r + 1 < nclosed; r += nt) {
    const int i = uni[r], j = uni[r + 1];
    if (near_tie_d(dens[i], dens[j]))
      log_tie(w, LOGKV_TIE_ALPHA_ORDER, b, -1, -1, r, min(i, j), max(i, j), rel_gap_d(dens[i], dens[j]),
              (float)dens[i]);
  }
  for (int i = tid; i < n; i += nt)
    if (swap_t[i] && near_tie_d(swap_a[i], swap_b[i]))
      log_tie(w, LOGKV_TIE_ALPHA_SWAP, b, -1, -1, i, i, swap_t[i] == 2 ? 1 : 0, rel_gap_d(swap_a[i], swap_b[i]),
              (float)swap_a[i]);
  __syncthreads();
  // Emit keep/archive token lists in candidate order and the new span table.
  int carry_keep = 0, carry_arch = 0, carry_sp = 0;
  __shared__ int tot_k, tot_a, tot_s;
  for (int base = 0; base < n; base += nt) {
    const int i = base + tid;
    const bool in = i < n;
    const int sz = in ? size[i] : 0;
    const bool ch = in && chosen[i];
    const int kincl = block_inclusive_scan(ch ? sz : 0, wsum);
    const int aincl = block_inclusive_scan(in && !ch ? sz : 0, wsum);
    const int sincl = block_inclusive_scan(ch ? 1 : 0, wsum);
    if (in) {
      const size_t c = (size_t)b * NC + i;
      const int s0 = w.cand_s0[c], n0 = w.cand_n0[c], s1 = w.cand_s1[c];
      if (ch) {
        const int at = carry_keep + kincl - sz;
        for (int t = 0; t < sz; ++t) {
          const int src = t < n0 ? s0 + t : s1 + (t - n0);
          if (at + t < P) w.keep_idx[(size_t)b * P + at + t] = src;
        }
        const int sp = carry_sp + sincl - 1;
        if (sp < P) {
          w.span_len[(size_t)b * P + sp] = sz;
          w.span_closed[(size_t)b * P + sp] = (flags[i] & 2) ? 1 : 0;
        }
      } else {
        const int at = carry_arch + aincl - sz;
        for (int t = 0; t < sz; ++t) {
          const int src = t < n0 ? s0 + t : s1 + (t - n0);
          w.arch_idx[(size_t)b * g.NW + at + t] = src;
        }
      }
    }
    if (tid == nt - 1) {
      tot_k = kincl;
      tot_a = aincl;
      tot_s = sincl;
    }
    __syncthreads();
    carry_keep += tot_k;
    carry_arch += tot_a;
    carry_sp += tot_s;
    __syncthreads();
  }
  if (tid == 0) {
    int nkeep = carry_keep;
    if (nkeep > P) {
      set_status(w.status, kStatusListOverflow);
      nkeep = P;
    }
    w.nkeep[b] = nkeep;
    w.narch[b] = carry_arch;
    w.nspans[b] = carry_sp < P ? carry_sp : P;
  }
  __syncthreads();
  // Archive rows in position order (stable).  Usually already sorted.
  const int na = carry_arch;
  int* arch = w.arch_idx + (size_t)b * g.NW;
  __shared__ int unsorted;
  if (tid == 0) unsorted = 0;
  __syncthreads();
  for (int i = tid + 1; i < na; i += nt)
    if (token_position(g, s, w, b, arch[i - 1]) > token_position(g, s, w, b, arch[i])) unsorted = 1;
  __syncthreads();
  if (unsorted) {
    int* tmp = ranked;  // reuse [NC] >= NW scratch in shared memory
    for (int i = tid; i < na; i += nt) tmp[i] = arch[i];
    __syncthreads();
    for (int i = tid; i < na; i += nt) {
      const int64_t pi = token_position(g, s, w, b, tmp[i]);
      int rank = 0;
      for (int j = 0; j < na; ++j) {
        const int64_t pj = token_position(g, s, w, b, tmp[j]);
        if (pj < pi || (pj == pi && j < i)) ++rank;
      }
      arch[rank] = tmp[i];
    }
  }
}

// ---------------------------------------------------------------- K7: pool rewrite
template <typename T>
__global__ void pool_rewrite_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  const int b = blockIdx.z, grp = blockIdx.y;
  const int nkeep = w.nkeep[b];
  T* kdst = static_cast<T*>(s.alpha_k_raw) + ((size_t)b * g.G + grp) * g.P * g.D;
  T* vdst = static_cast<T*>(s.alpha_v) + ((size_t)b * g.G + grp) * g.P * g.D;
  const T* snapk = static_cast<const T*>(w.snap_k);
  const T* snapv = static_cast<const T*>(w.snap_v);
  const T* reck = static_cast<const T*>(s.recent_k_raw);
  const T* recv = static_cast<const T*>(s.recent_v);
  constexpr int VN = Vec<T>::N;
  const int DV = g.D / VN;
  const size_t total = (size_t)g.P * DV;  // 16-byte units
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / DV), d = (int)(i % DV) * VN;
    uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
    if (row < nkeep) {
      const int src = w.keep_idx[(size_t)b * g.P + row];
      kv = *reinterpret_cast<const uint4*>(token_row<T>(g, snapk, reck, b, grp, src) + d);
      vv = *reinterpret_cast<const uint4*>(token_row<T>(g, snapv, recv, b, grp, src) + d);
    }
    reinterpret_cast<uint4*>(kdst)[i] = kv;
    reinterpret_cast<uint4*>(vdst)[i] = vv;
  }
  if (grp == 0 && blockIdx.x == 0) {
    for (int row = threadIdx.x; row < g.P; row += blockDim.x) {
      const bool kept = row < nkeep;
      s.alpha_pos[(size_t)b * g.P + row] = kept ? token_position(g, s, w, b, w.keep_idx[(size_t)b * g.P + row]) : 0;
      s.alpha_valid[(size_t)b * g.P + row] = kept ? 1 : 0;
    }
    // The choice's span table and counts become the pool's (the decision kernels write
    // only the workspace, so that they may run beside readers of the cache).
    const int ns = w.nspans[b];
    for (int i = threadIdx.x; i < ns; i += blockDim.x) {
      s.alpha_span_len[(size_t)b * g.P + i] = w.span_len[(size_t)b * g.P + i];
      s.alpha_span_closed[(size_t)b * g.P + i] = w.span_closed[(size_t)b * g.P + i];
    }
    if (threadIdx.x == 0) {
      s.alpha_nspans[b] = ns;
      s.alpha_rowcount[b] = nkeep;
      if (b == 0) {
        int most = 0;
        for (int j = 0; j < g.B; ++j) most = max(most, w.nkeep[j]);
        *s.alpha_count = most;
      }
    }
  }
}

}  // namespace logkv
