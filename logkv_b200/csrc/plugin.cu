// Operator-level plugin functions (C ABI in include/logkv_plugin.h): the functions
// the reference's fused-kernel modules export, so its own Python orchestration can
// run on sm_100a instead of Triton.  Built with -fmad=false like the flush: every
// feature-axis sum is left to right in one thread and every product and sum is
// rounded as written, i.e. the reference's CPU order, not a tree reduction.
//
//   P1 rows_scatter_kernel   fill(), survivor writes and clears of merge_scatter()
//   P2 pair_merge_kernel     merge_scatter() pairwise merges and survivor staging
//   P3 beta_merge_kernel     merge_scatter() Beta 4->2 groups (select or replay the cut)
//   P4 centroid_kernel       centroid(): ordered run sums, then a separate commit
//   P5 partition_kernel      alpha_partition()
//   P6 attach_assign_kernel  attach_assign()
#include <algorithm>

#include "common.cuh"
#include "../../include/logkv_plugin.h"

namespace logkv {

__device__ __forceinline__ float load_as_float(const void* base, int dtype, size_t i) {
  return dtype == LOGKV_DTYPE_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i])
                                   : static_cast<const float*>(base)[i];
}
__device__ __forceinline__ void store_from_float(void* base, int dtype, size_t i, float v) {
  if (dtype == LOGKV_DTYPE_BF16) static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  else static_cast<float*>(base)[i] = v;
}
// A row read from the pool: stored rows in their dtype; staged rows are cast to the
// storage dtype first (the reference's pool construction casts staging rows).
__device__ __forceinline__ float pool_kv(const void* fbase, const void* sbase, int fdtype, int sdtype, bool stored,
                                         size_t row, int dim, int d) {
  if (stored) return load_as_float(fbase, fdtype, row * dim + d);
  const float x = load_as_float(sbase, sdtype, row * dim + d);
  return fdtype == LOGKV_DTYPE_BF16 ? __bfloat162float(__float2bfloat16_rn(x)) : x;
}

struct Pool {
  logkv_rows_t f, s;
  const int64_t* si;
  const int64_t* gi;
  int64_t ns;
  __device__ __forceinline__ bool stored(int64_t idx) const { return idx < ns; }
  __device__ __forceinline__ size_t row(int64_t idx) const { return (size_t)(idx < ns ? si[idx] : gi[idx - ns]); }
  __device__ __forceinline__ const logkv_rows_t& src(int64_t idx) const { return idx < ns ? f : s; }
};

// ---------------------------------------------------------------- P1: scatter rows / clear
// Rows r < n copy src row (src ? src[r] : offset + r) of `from` to dst[r] of `to`; rows
// n <= r < n + nclear zero every field of `to` at clear[r - n].
__global__ void rows_scatter_kernel(logkv_rows_t to, logkv_rows_t from, const int64_t* src, int64_t offset,
                                    const int64_t* dst, int64_t n, const int64_t* clear, int64_t nclear, int dk,
                                    int dv) {
  const int64_t r = blockIdx.x;
  if (r >= n + nclear) return;
  const bool copy = r < n;
  const size_t s = copy ? (size_t)(src ? src[r] : offset + r) : 0;
  const size_t d = (size_t)(copy ? dst[r] : clear[r - n]);
  for (int e = threadIdx.x; e < dk; e += blockDim.x)
    store_from_float(to.k, to.kv_dtype, d * dk + e, copy ? load_as_float(from.k, from.kv_dtype, s * dk + e) : 0.f);
  for (int e = threadIdx.x; e < dv; e += blockDim.x)
    store_from_float(to.v, to.kv_dtype, d * dv + e, copy ? load_as_float(from.v, from.kv_dtype, s * dv + e) : 0.f);
  if (threadIdx.x == 0) {
    to.w[d] = copy ? from.w[s] : 0.f;
    to.p_lo[d] = copy ? from.p_lo[s] : 0;
    to.p_hi[d] = copy ? from.p_hi[s] : 0;
    to.sum_wp[d] = copy ? from.sum_wp[s] : 0;
    to.order[d] = copy ? from.order[s] : 0;
    to.pad[d] = copy ? from.pad[s] : 0;
  }
}

// ---------------------------------------------------------------- P2: pairwise merges + survivors
// Output rows r < np: merge of pool rows pi[2r], pi[2r+1]; np <= r < np + nv: pool row vi[r - np].
__global__ void pair_merge_kernel(Pool p, logkv_rows_t out, const int64_t* pi, int64_t np, const int64_t* vi,
                                  int64_t nv, int dk, int dv) {
  const int64_t r = blockIdx.x;
  if (r >= np + nv) return;
  const bool pair = r < np;
  const int64_t ai = pair ? pi[2 * r] : vi[r - np];
  const int64_t bi = pair ? pi[2 * r + 1] : 0;
  const size_t ra = p.row(ai), rb = pair ? p.row(bi) : 0;
  const logkv_rows_t& A = p.src(ai);
  const logkv_rows_t& Bq = p.src(pair ? bi : ai);
  const float wa = A.w[ra], wb = pair ? Bq.w[rb] : 0.f;
  const float alpha = fdiv(wa, fmaxf(fadd(wa, wb), 1e-8f));
  const float beta = fsub(1.f, alpha);
  for (int e = threadIdx.x; e < dk; e += blockDim.x) {
    const float a = pool_kv(p.f.k, p.s.k, p.f.kv_dtype, p.s.kv_dtype, p.stored(ai), ra, dk, e);
    float o = a;
    if (pair) o = fadd(fmul(alpha, a), fmul(beta, pool_kv(p.f.k, p.s.k, p.f.kv_dtype, p.s.kv_dtype, p.stored(bi), rb, dk, e)));
    static_cast<float*>(out.k)[(size_t)r * dk + e] = o;
  }
  for (int e = threadIdx.x; e < dv; e += blockDim.x) {
    const float a = pool_kv(p.f.v, p.s.v, p.f.kv_dtype, p.s.kv_dtype, p.stored(ai), ra, dv, e);
    float o = a;
    if (pair) o = fadd(fmul(alpha, a), fmul(beta, pool_kv(p.f.v, p.s.v, p.f.kv_dtype, p.s.kv_dtype, p.stored(bi), rb, dv, e)));
    static_cast<float*>(out.v)[(size_t)r * dv + e] = o;
  }
  if (threadIdx.x == 0) {
    if (!pair) {
      out.w[r] = wa;
      out.p_lo[r] = A.p_lo[ra];
      out.p_hi[r] = A.p_hi[ra];
      out.sum_wp[r] = A.sum_wp[ra];
      out.order[r] = A.order[ra];
      out.pad[r] = A.pad[ra];
    } else {
      const bool ya = wa > 0.f, yb = wb > 0.f;
      const int64_t la = A.p_lo[ra], lb = Bq.p_lo[rb], ha = A.p_hi[ra], hb = Bq.p_hi[rb];
      out.w[r] = fadd(wa, wb);
      out.p_lo[r] = ya && yb ? min(la, lb) : (ya ? la : lb);
      out.p_hi[r] = ya && yb ? max(ha, hb) : (ya ? ha : hb);
      out.sum_wp[r] = A.sum_wp[ra] + Bq.sum_wp[rb];
      out.order[r] = min(A.order[ra], Bq.order[rb]);
      out.pad[r] = A.pad[ra] & Bq.pad[rb];
    }
  }
}

// ---------------------------------------------------------------- P3: Beta groups
// One block per group (start, width, dest) of `layout`, plus trailing blocks that stage
// survivors (8 per block) at np + j.  Cut: 2|2, 1|3 or 3|1 by the least normalised weighted
// SSE of K and V (ties keep the earlier), width 2 always 1; or the recorded cut.
__global__ void beta_merge_kernel(Pool p, logkv_rows_t out, const int64_t* pi, const int64_t* layout, int64_t ng,
                                  uint8_t* cuts, int replay, const int64_t* vi, int64_t np, int64_t nv, int dk,
                                  int dv) {
  const int64_t gidx = blockIdx.x;
  __shared__ float wv[4];
  __shared__ int64_t idx[4];
  __shared__ int cut_s;
  const int tid = threadIdx.x;
  if (gidx >= ng) {
    for (int64_t j = (gidx - ng) * 8; j < min(nv, (gidx - ng + 1) * 8); ++j) {
      const int64_t ai = vi[j];
      const size_t ra = p.row(ai);
      const logkv_rows_t& A = p.src(ai);
      const int64_t r = np + j;
      for (int e = tid; e < dk; e += blockDim.x)
        static_cast<float*>(out.k)[(size_t)r * dk + e] = pool_kv(p.f.k, p.s.k, p.f.kv_dtype, p.s.kv_dtype, p.stored(ai), ra, dk, e);
      for (int e = tid; e < dv; e += blockDim.x)
        static_cast<float*>(out.v)[(size_t)r * dv + e] = pool_kv(p.f.v, p.s.v, p.f.kv_dtype, p.s.kv_dtype, p.stored(ai), ra, dv, e);
      if (tid == 0) {
        out.w[r] = A.w[ra];
        out.p_lo[r] = A.p_lo[ra];
        out.p_hi[r] = A.p_hi[ra];
        out.sum_wp[r] = A.sum_wp[ra];
        out.order[r] = A.order[ra];
        out.pad[r] = A.pad[ra];
      }
    }
    return;
  }
  const int64_t start = layout[3 * gidx], width = layout[3 * gidx + 1], dest = layout[3 * gidx + 2];
  if (tid < 4) {
    idx[tid] = tid < width ? pi[start + tid] : 0;
    wv[tid] = tid < width ? p.src(idx[tid]).w[p.row(idx[tid])] : 0.f;
  }
  __syncthreads();
  auto x_at = [&](int comp, int row, int e) -> float {
    if (row >= width) return 0.f;
    const int64_t ai = idx[row];
    const int dim = comp == 0 ? dk : dv;
    return comp == 0 ? pool_kv(p.f.k, p.s.k, p.f.kv_dtype, p.s.kv_dtype, p.stored(ai), p.row(ai), dim, e)
                     : pool_kv(p.f.v, p.s.v, p.f.kv_dtype, p.s.kv_dtype, p.stored(ai), p.row(ai), dim, e);
  };
  if (replay) {
    if (tid == 0) cut_s = width == 4 ? (int)cuts[gidx] : 1;
  } else if (width != 4) {
    if (tid == 0) {
      cut_s = 1;
      cuts[gidx] = 1;
    }
  } else if (tid == 0) {
    // Canonical order (beta_log_kv.select_cuts): one thread, features left to right.
    float tot = 0.f;
    for (int i = 0; i < 4; ++i) tot = fadd(tot, wv[i]);
    tot = fmaxf(tot, 1e-12f);
    float c3[3] = {0.f, 0.f, 0.f};
    for (int comp = 0; comp < 2; ++comp) {
      const int dim = comp == 0 ? dk : dv;
      float e4[4] = {0.f, 0.f, 0.f, 0.f};
      for (int d = 0; d < dim; ++d)
        for (int i = 0; i < 4; ++i) {
          const float xv = x_at(comp, i, d);
          e4[i] = fadd(e4[i], fmul(xv, xv));
        }
      float acc = 0.f;
      for (int i = 0; i < 4; ++i) acc = fadd(acc, fmul(e4[i], wv[i]));
      const float energy = fmaxf(fdiv(acc, tot), 1e-12f);
      for (int j = 0; j < 3; ++j) {
        const int c = j == 0 ? 2 : (j == 1 ? 1 : 3);
        for (int side = 0; side < 2; ++side) {
          float om[4], ws = 0.f;
          for (int i = 0; i < 4; ++i) {
            om[i] = fmul(wv[i], (side == 0 ? i < c : i >= c) ? 1.f : 0.f);
            ws = fadd(ws, om[i]);
          }
          const float den = fmaxf(ws, 1e-12f);
          float r4[4] = {0.f, 0.f, 0.f, 0.f};
          for (int d = 0; d < dim; ++d) {
            float xv[4], s = 0.f;
            for (int i = 0; i < 4; ++i) {
              xv[i] = x_at(comp, i, d);
              s = fadd(s, fmul(xv[i], om[i]));
            }
            const float mean = fdiv(s, den);
            for (int i = 0; i < 4; ++i) {
              const float df = fsub(xv[i], mean);
              r4[i] = fadd(r4[i], fmul(df, df));
            }
          }
          float loss = 0.f;
          for (int i = 0; i < 4; ++i) loss = fadd(loss, fmul(r4[i], om[i]));
          c3[j] = fadd(c3[j], fdiv(loss, energy));
        }
      }
    }
    int best = 0;
    if (c3[1] < c3[best]) best = 1;
    if (c3[2] < c3[best]) best = 2;
    cut_s = best == 0 ? 2 : (best == 1 ? 1 : 3);
    cuts[gidx] = (uint8_t)cut_s;
  }
  __syncthreads();
  const int cut = cut_s;
  for (int side = 0; side < (width == 4 ? 2 : 1); ++side) {
    float om[4], mass = 0.f;
    for (int i = 0; i < 4; ++i) {
      const bool in = i < width && (width == 2 ? side == 0 : (side == 0 ? i < cut : i >= cut));
      om[i] = fmul(wv[i], in ? 1.f : 0.f);
      mass = fadd(mass, om[i]);
    }
    const float den = fmaxf(mass, 1e-12f);
    const int64_t r = dest + side;
    for (int e = tid; e < dk; e += blockDim.x) {
      float s = 0.f;
      for (int i = 0; i < 4; ++i) s = fadd(s, fmul(x_at(0, i, e), om[i]));
      static_cast<float*>(out.k)[(size_t)r * dk + e] = fdiv(s, den);
    }
    for (int e = tid; e < dv; e += blockDim.x) {
      float s = 0.f;
      for (int i = 0; i < 4; ++i) s = fadd(s, fmul(x_at(1, i, e), om[i]));
      static_cast<float*>(out.v)[(size_t)r * dv + e] = fdiv(s, den);
    }
    if (tid == 0) {
      int64_t lo = INT64_MAX, hi = INT64_MIN, swp = 0, ord = INT64_MAX;
      int pad = 1;
      for (int i = 0; i < 4; ++i) {
        const bool in = i < width && (width == 2 ? side == 0 : (side == 0 ? i < cut : i >= cut));
        if (!in) continue;
        const logkv_rows_t& A = p.src(idx[i]);
        const size_t ra = p.row(idx[i]);
        if (wv[i] > 0.f) {
          lo = min(lo, A.p_lo[ra]);
          hi = max(hi, A.p_hi[ra]);
        }
        swp += A.sum_wp[ra];
        ord = min(ord, A.order[ra]);
        pad &= A.pad[ra] ? 1 : 0;
      }
      out.w[r] = mass;
      out.p_lo[r] = mass > 0.f ? lo : 0;
      out.p_hi[r] = mass > 0.f ? hi : 0;
      out.sum_wp[r] = swp;
      out.order[r] = ord;
      out.pad[r] = (uint8_t)pad;
    }
  }
}

// ---------------------------------------------------------------- P4: centroids
// meta [5, nr]: cluster, (unused), begin, length, forget (float32 bits).  Phase 1 reads the
// state only; phase 2 commits, so no run observes another's update.
__global__ void centroid_kernel(const void* k, int kdtype, int d, const float* mu, const float* ne, const int64_t* meta,
                                int64_t nr, int64_t start, float* out_mu, float* out_ne) {
  const int64_t row = blockIdx.x, r = start + row;
  const int64_t cluster = meta[r], begin = meta[2 * nr + r], length = meta[3 * nr + r];
  const int32_t fbits = (int32_t)meta[4 * nr + r];
  const float forget = __int_as_float(fbits);
  const float pre = fmul(ne[cluster], forget);
  const float n = (float)length;
  const float denom = fadd(pre, n);
  for (int e = threadIdx.x; e < d; e += blockDim.x) {
    float acc = 0.f;
    for (int64_t i = 0; i < length; ++i) acc = fadd(acc, load_as_float(k, kdtype, (size_t)(begin + i) * d + e));
    const float m = mu[cluster * d + e];
    out_mu[row * d + e] = pre > 0.f ? fdiv(fadd(fmul(pre, m), acc), denom) : fdiv(acc, n);
  }
  if (threadIdx.x == 0) out_ne[row] = denom;
}

__global__ void centroid_commit_kernel(float* mu, float* ne, const float* out_mu, const float* out_ne,
                                       const int64_t* meta, int64_t start, int64_t count, int d) {
  const int64_t row = blockIdx.x;
  if (row >= count) return;
  const int64_t cluster = meta[start + row];
  for (int e = threadIdx.x; e < d; e += blockDim.x) mu[cluster * d + e] = out_mu[row * d + e];
  if (threadIdx.x == 0) ne[cluster] = out_ne[row];
}

// ---------------------------------------------------------------- P5: Alpha partition
__global__ void partition_kernel(logkv_partition_t a) {
  const int64_t row = blockIdx.x;
  const int g = blockIdx.y, b = blockIdx.z;
  if (row >= a.exact + a.archive) return;
  const int64_t src = a.indices[(size_t)b * (a.exact + a.archive) + row];
  const bool token = src >= 0;
  const size_t base = ((size_t)b * a.groups + g) * a.tokens + (token ? src : 0);
  const bool keep = row < a.exact;
  const size_t orow = keep ? ((size_t)b * a.groups + g) * a.exact + row
                           : ((size_t)b * a.groups + g) * a.archive + (row - a.exact);
  void* ok = keep ? a.exact_k : a.archive_k;
  void* ov = keep ? a.exact_v : a.archive_v;
  for (int e = threadIdx.x; e < a.dk; e += blockDim.x)
    store_from_float(ok, a.dtype, orow * a.dk + e, token ? load_as_float(a.k, a.dtype, base * a.dk + e) : 0.f);
  for (int e = threadIdx.x; e < a.dv; e += blockDim.x)
    store_from_float(ov, a.dtype, orow * a.dv + e, token ? load_as_float(a.v, a.dtype, base * a.dv + e) : 0.f);
  if (g == 0 && threadIdx.x == 0) {
    const int64_t pos = token ? a.pos[(size_t)b * a.tokens + src] : 0;
    if (keep) {
      a.exact_pos[(size_t)b * a.exact + row] = pos;
      a.exact_valid[(size_t)b * a.exact + row] = token ? 1 : 0;
    } else {
      a.archive_pos[(size_t)b * a.archive + row - a.exact] = pos;
    }
  }
}

// ---------------------------------------------------------------- P6: attach_assign
// One thread per (token slot, lane); clusters and features in canonical order.
__global__ void attach_assign_kernel(logkv_attach_t a) {
  const int64_t slot = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int lane = blockIdx.y, b = lane / a.groups, g = lane % a.groups;
  if (slot >= a.tokens || slot >= a.counts[b]) return;
  const int64_t off = a.order[(size_t)b * a.tokens + slot];
  const int64_t pos = a.positions[(size_t)b * a.pos_stride_b + off];
  const size_t xrow = (size_t)b * a.x_stride_b + (size_t)g * a.x_stride_g + (size_t)off * a.x_stride_t;
  const float* mu = a.centroid + (size_t)lane * a.clusters * a.dim;
  const uint8_t* alive = a.alive + (size_t)lane * a.clusters;
  const int64_t* phi = a.p_hi + (size_t)lane * a.clusters;
  float xx = 0.f;
  for (int d = 0; d < a.dim; ++d) {
    const float x = load_as_float(a.x, a.dtype, xrow + d);
    xx = fadd(xx, fmul(x, x));
  }
  int winner = 0, nearest = 0, nlive = 0;  // argmin over no live cluster is 0, as in the reference
  float best = INFINITY, s_winner = 0.f, best_exact = INFINITY;
  for (int c = 0; c < a.clusters; ++c) {
    float mm = 0.f, dot = 0.f, ex = 0.f;
    for (int d = 0; d < a.dim; ++d) {
      const float x = load_as_float(a.x, a.dtype, xrow + d);
      const float m = mu[(size_t)c * a.dim + d];
      mm = fadd(mm, fmul(m, m));
      dot = fadd(dot, fmul(x, m));
      const float df = fsub(x, m);
      ex = fadd(ex, fmul(df, df));
    }
    const float semantic = fmaxf(fsub(fadd(xx, mm), fmul(2.f, dot)), 0.f);
    const float gap = fmaxf((float)(pos - phi[c]), 0.f);
    const float cost = fadd(semantic, fmul(a.eta, fdiv(gap, fadd(gap, a.g0))));
    if (!alive[c]) continue;
    ++nlive;
    if (cost < best) {
      best = cost;
      winner = c;
      s_winner = semantic;
    }
    if (ex < best_exact) {
      best_exact = ex;
      nearest = c;
    }
  }
  const bool direct = nlive > 0 && s_winner <= fmul(a.lam, a.s_h[lane]);
  a.out[(size_t)lane * a.tokens + slot] = (int8_t)(direct ? winner : nearest);
}

static int launch_ok() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LOGKV_OK : (int)e;
}

static bool rows_ok(const logkv_rows_t* r, bool kv_float_only = false) {
  if (!r || !r->k || !r->v || !r->w || !r->p_lo || !r->p_hi || !r->sum_wp || !r->order || !r->pad) return false;
  if (r->kv_dtype != LOGKV_DTYPE_F32 && r->kv_dtype != LOGKV_DTYPE_BF16) return false;
  return !kv_float_only || r->kv_dtype == LOGKV_DTYPE_F32;
}

}  // namespace logkv

using namespace logkv;

extern "C" {

LOGKV_API int logkv_fill(const logkv_rows_t* fields, const logkv_rows_t* stage, const int64_t* src,
                         const int64_t* dst, int64_t n, int32_t dk, int32_t dv, void* stream) {
  if (n < 0 || dk < 1 || dv < 1) return LOGKV_E_SHAPE;
  if (n == 0) return LOGKV_OK;
  if (!rows_ok(fields) || !rows_ok(stage) || !src || !dst) return LOGKV_E_POINTER;
  rows_scatter_kernel<<<(unsigned)n, 128, 0, static_cast<cudaStream_t>(stream)>>>(*fields, *stage, src, 0, dst, n,
                                                                                   nullptr, 0, dk, dv);
  return launch_ok();
}

LOGKV_API int logkv_merge_scatter(const logkv_rows_t* fields, const logkv_rows_t* stage, const int64_t* si,
                                  int64_t ns, const int64_t* gi, const int64_t* pi, int64_t npi, const int64_t* vi,
                                  int64_t nv, const int64_t* dst, const int64_t* clear, int64_t nclear,
                                  const logkv_rows_t* out, const int64_t* beta_layout, int64_t ngroups,
                                  uint8_t* beta_cuts, int32_t beta_mode, int32_t dk, int32_t dv, void* stream) {
  if (ns < 0 || npi < 0 || (npi & 1) || nv < 0 || nclear < 0 || ngroups < 0 || dk < 1 || dv < 1 || beta_mode < 0 ||
      beta_mode > 2)
    return LOGKV_E_SHAPE;
  if (!rows_ok(fields) || !rows_ok(stage) || !rows_ok(out, true)) return LOGKV_E_POINTER;
  if ((npi && !pi) || (nv && (!vi || !dst)) || (nclear && !clear) || (ns && !si)) return LOGKV_E_POINTER;
  if (beta_mode && ngroups && (!beta_layout || !beta_cuts)) return LOGKV_E_POINTER;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Pool p{*fields, *stage, si, gi, ns};
  const int64_t np = npi / 2;
  if (!beta_mode) {
    if (np + nv) pair_merge_kernel<<<(unsigned)(np + nv), 128, 0, st>>>(p, *out, pi, np, vi, nv, dk, dv);
  } else {
    const int64_t blocks = ngroups + (nv + 7) / 8;
    if (blocks)
      beta_merge_kernel<<<(unsigned)blocks, 128, 0, st>>>(p, *out, pi, beta_layout, ngroups, beta_cuts,
                                                          beta_mode == 2, vi, np, nv, dk, dv);
  }
  if (nv + nclear)
    rows_scatter_kernel<<<(unsigned)(nv + nclear), 128, 0, st>>>(*fields, *out, nullptr, np, dst, nv, clear,
                                                                 nclear, dk, dv);
  return launch_ok();
}

LOGKV_API int logkv_centroid(const void* k, int32_t k_dtype, int32_t dim, float* mu, float* n_eff,
                             const int64_t* metadata, int64_t runs, int64_t start, int64_t count, float* scratch,
                             void* stream) {
  if (dim < 1 || runs < 0 || start < 0 || count < 0 || start + count > runs) return LOGKV_E_SHAPE;
  if (k_dtype != LOGKV_DTYPE_F32 && k_dtype != LOGKV_DTYPE_BF16) return LOGKV_E_DTYPE;
  if (count == 0) return LOGKV_OK;
  if (!k || !mu || !n_eff || !metadata || !scratch) return LOGKV_E_POINTER;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* out_mu = scratch;
  float* out_ne = scratch + (size_t)count * dim;
  centroid_kernel<<<(unsigned)count, 128, 0, st>>>(k, k_dtype, dim, mu, n_eff, metadata, runs, start, out_mu, out_ne);
  centroid_commit_kernel<<<(unsigned)count, 128, 0, st>>>(mu, n_eff, out_mu, out_ne, metadata, start, count, dim);
  return launch_ok();
}

LOGKV_API int logkv_alpha_partition(const logkv_partition_t* args, void* stream) {
  if (!args) return LOGKV_E_POINTER;
  const logkv_partition_t& a = *args;
  if (a.batch < 1 || a.groups < 1 || a.tokens < 0 || a.exact < 0 || a.archive < 0 || a.dk < 1 || a.dv < 1)
    return LOGKV_E_SHAPE;
  if (a.dtype != LOGKV_DTYPE_F32 && a.dtype != LOGKV_DTYPE_BF16) return LOGKV_E_DTYPE;
  if (a.exact + a.archive == 0) return LOGKV_OK;
  if (!a.k || !a.v || !a.pos || !a.indices || !a.exact_k || !a.exact_v || !a.exact_pos || !a.exact_valid ||
      (a.archive && (!a.archive_k || !a.archive_v || !a.archive_pos)))
    return LOGKV_E_POINTER;
  partition_kernel<<<dim3((unsigned)(a.exact + a.archive), a.groups, a.batch), 128, 0,
                     static_cast<cudaStream_t>(stream)>>>(a);
  return launch_ok();
}

LOGKV_API int logkv_attach_assign(const logkv_attach_t* args, void* stream) {
  if (!args) return LOGKV_E_POINTER;
  const logkv_attach_t& a = *args;
  if (a.batch < 1 || a.groups < 1 || a.tokens < 0 || a.clusters < 1 || a.clusters > 127 || a.dim < 1)
    return LOGKV_E_SHAPE;
  if (a.dtype != LOGKV_DTYPE_F32 && a.dtype != LOGKV_DTYPE_BF16) return LOGKV_E_DTYPE;
  if (a.tokens == 0) return LOGKV_OK;
  if (!a.x || !a.positions || !a.order || !a.counts || !a.centroid || !a.alive || !a.p_hi || !a.s_h || !a.out)
    return LOGKV_E_POINTER;
  attach_assign_kernel<<<dim3((unsigned)((a.tokens + 127) / 128), a.batch * a.groups), 128, 0,
                         static_cast<cudaStream_t>(stream)>>>(a);
  return launch_ok();
}

}  // extern "C"
