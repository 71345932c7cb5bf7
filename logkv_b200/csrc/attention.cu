// Read side of the SemanticLogKV cache on sm_100a: mid-anchor attention plan,
// prefix packing and slot attention (C ABI in include/logkv_attention.h).
//
//   K1 attn_plan_kernel     one CTA per (b, g) lane: block scans over the lane's
//                            (cluster, level) counts give every occupied entry its
//                            plan position and every valid entry its compacted one.
//   K2 prefix_pack_kernel   one warp per output row: RoPE at the mid anchor with the
//                            reference's rounding chain, value copy, mass term.
//   K3 pack_mid_kernel      the reference's 136-wide packed layout (same math as K2).
//   K4 slot_attn_kernel     split-K attention for a few query tokens: each warp
//                            streams tiles of slot rows through a private cp.async
//                            ring (every lane reads back only the 16-byte chunks it
//                            copied, so a warp never waits for another), online
//                            softmax in the log2 domain, CTA and cross-CTA combines
//                            in a fixed order (the last CTA of a lane combines).
#include <algorithm>
#include <type_traits>
#include <cstring>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tcgen05.cuh"
#include "../../include/logkv_attention.h"

namespace logkv {

constexpr int32_t kStatusAnchorRange = 1 << 16;

struct PlanGeo {
  int B, G, K, L, Bs, P, D, cap;
};

static PlanGeo make_plan_geo(const logkv_layout_t& l) {
  PlanGeo g;
  g.B = l.batch;
  g.G = l.groups;
  g.K = l.clusters;
  g.L = l.levels;
  g.Bs = l.slots;
  g.P = l.exact;
  g.D = l.dim;
  g.cap = l.clusters * l.levels * l.slots;
  return g;
}

__device__ __forceinline__ int64_t floor_div(int64_t a, int64_t b) {
  int64_t q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) --q;
  return q;
}

// ---------------------------------------------------------------- K1: plan
__global__ void __launch_bounds__(512) attn_plan_kernel(PlanGeo pg, logkv_state_t s, logkv_plan_t p) {
  const int g = blockIdx.x, b = blockIdx.y, lane = b * pg.G + g;
  const int KL = pg.K * pg.L, tid = threadIdx.x, nt = blockDim.x;
  const int warp = tid >> 5, lid = tid & 31, nwarps = nt >> 5;
  __shared__ int off[kMaxClusters * kMaxLevels];
  __shared__ int voff[kMaxClusters * kMaxLevels];
  __shared__ int vcnt[kMaxClusters * kMaxLevels];
  __shared__ int wsum[32];
  __shared__ int tot[2];
  const int16_t* cnt = s.level_count + (size_t)lane * KL;
  const float* w = s.level_w + (size_t)lane * pg.cap;
  const int64_t* swp = s.level_sum_wp + (size_t)lane * pg.cap;
  // Plan order q = c * L + j walks level L - 1 - j: top level first inside a cluster.
  auto group_entry0 = [&](int q) { return (q / pg.L * pg.L + (pg.L - 1 - q % pg.L)) * pg.Bs; };
  auto group_count = [&](int q) { return (int)cnt[q / pg.L * pg.L + (pg.L - 1 - q % pg.L)]; };
  for (int q = warp; q < KL; q += nwarps) {
    const int n = group_count(q), e0 = group_entry0(q);
    int nv = 0;
    for (int i = lid; i - lid < n; i += 32) {
      const bool v = i < n && w[e0 + i] > 0.f;
      nv += __popc(__ballot_sync(0xffffffffu, v));
    }
    if (lid == 0) vcnt[q] = nv;
  }
  __syncthreads();
  const int my = tid < KL ? group_count(tid) : 0;
  const int myv = tid < KL ? vcnt[tid] : 0;
  const int inc = block_inclusive_scan(my, wsum);
  const int vinc = block_inclusive_scan(myv, wsum);
  if (tid < KL) {
    off[tid] = inc - my;
    voff[tid] = vinc - myv;
  }
  if (tid == nt - 1) {
    tot[0] = inc;
    tot[1] = vinc;
  }
  __syncthreads();
  const int width = tot[0], nvalid = tot[1];
  const size_t base = (size_t)lane * pg.cap;
  for (int q = warp; q < KL; q += nwarps) {
    const int n = group_count(q), e0 = group_entry0(q);
    int vrun = voff[q];
    for (int i0 = 0; i0 < n; i0 += 32) {
      const int i = i0 + lid;
      bool v = false;
      int64_t anchor = 0;
      if (i < n) {
        const float wi = w[e0 + i];
        v = wi > 0.f;
        if (v) {
          const int64_t ww = max((int64_t)wi, (int64_t)1);  // weights.long().clamp_min(1)
          anchor = floor_div(2 * swp[e0 + i] + ww, 2 * ww);
        }
        if (p.idx) {
          p.idx[base + off[q] + i] = e0 + i;
          p.anchor[base + off[q] + i] = anchor;
          p.valid[base + off[q] + i] = v ? 1 : 0;
        }
      }
      const unsigned m = __ballot_sync(0xffffffffu, v);
      if (v) {
        const int at = vrun + __popc(m & ((1u << lid) - 1u));
        p.vslot[base + at] = e0 + i;
        p.vanchor[base + at] = anchor;
      }
      vrun += __popc(m);
    }
  }
  if (p.idx) {
    for (int i = width + tid; i < pg.cap; i += nt) {
      p.idx[base + i] = 0;
      p.anchor[base + i] = 0;
      p.valid[base + i] = 0;
    }
  }
  if (tid == 0) {
    if (p.width) p.width[lane] = width;
    if (p.width_max) atomicMax(p.width_max, width);
    p.nvalid[lane] = nvalid;
  }
  // Valid exact-pool rows of batch row b (computed once, by the g == 0 lane).
  if (g == 0) {
    const int ac = min(*s.alpha_count, pg.P);
    int run = 0;
    for (int j0 = 0; j0 < ac; j0 += nt) {
      const int j = j0 + tid;
      const bool v = j < ac && s.alpha_valid[(size_t)b * pg.P + j] != 0;
      const int incl = block_inclusive_scan(v ? 1 : 0, wsum);
      if (v) p.exact_rows[(size_t)b * pg.P + run + incl - 1] = j;
      if (tid == nt - 1) tot[0] = incl;
      __syncthreads();
      run += tot[0];
      __syncthreads();
    }
    if (tid == 0) p.nexact[b] = run;
  }
}

// ---------------------------------------------------------------- RoPE arithmetic
// x * cos + rotate_half(x) * sin (log_kv_position.py:95-99) with torch's promotion:
// float32 arithmetic unless content and tables are both bfloat16, then every op rounds.
template <typename T, typename C>
struct Rope {
  __device__ __forceinline__ static float apply(float x, float rot, float c, float s) {
    return Elem<T>::round(__fadd_rn(__fmul_rn(x, c), __fmul_rn(rot, s)));
  }
};
template <>
struct Rope<__nv_bfloat16, __nv_bfloat16> {
  __device__ __forceinline__ static float apply(float x, float rot, float c, float s) {
    const float a = Elem<__nv_bfloat16>::round(__fmul_rn(x, c));
    const float b = Elem<__nv_bfloat16>::round(__fmul_rn(rot, s));
    return Elem<__nv_bfloat16>::round(__fadd_rn(a, b));
  }
};

template <typename C>
__device__ __forceinline__ float table_load(const C* t, size_t i) {
  return Elem<C>::load(t + i);
}

struct RopeArgs {
  const void* cos;
  const void* sin;
  int rows, rope_n;
};

// One warp writes the rotated key row `dst` from `src` at position `anchor`.
template <typename T, typename C>
__device__ __forceinline__ void rope_row(const RopeArgs& r, int D, const T* src, int64_t anchor, T* dst,
                                         int lid) {
  const C* ct = static_cast<const C*>(r.cos) + (size_t)anchor * r.rope_n;
  const C* st = static_cast<const C*>(r.sin) + (size_t)anchor * r.rope_n;
  const int half = r.rope_n / 2;
  for (int d = lid; d < D; d += 32) {
    const float x = Elem<T>::load(src + d);
    float y = x;
    if (d < r.rope_n) {
      const float rot = d < half ? -Elem<T>::load(src + d + half) : Elem<T>::load(src + d - half);
      y = Rope<T, C>::apply(x, rot, table_load(ct, d), table_load(st, d));
    }
    Elem<T>::store(dst + d, y);
  }
}

__device__ __forceinline__ int64_t checked_anchor(int64_t a, int rows, int32_t* status) {
  if (a < 0 || a >= rows) {
    if (status) atomicOr(status, kStatusAnchorRange);
    return a < 0 ? 0 : rows - 1;
  }
  return a;
}

// ---------------------------------------------------------------- K2: prefix pack
template <typename T, typename C>
__global__ void __launch_bounds__(256) prefix_pack_kernel(PlanGeo pg, logkv_state_t s, logkv_plan_t p, RopeArgs r,
                                                          logkv_prefix_t out, int32_t* status) {
  const int g = blockIdx.y, b = blockIdx.z, lane = b * pg.G + g, D = pg.D;
  const int warp = threadIdx.x >> 5, lid = threadIdx.x & 31;
  const int nv = p.nvalid[lane], ne = p.nexact[b], n = nv + ne;
  if (blockIdx.x == 0 && threadIdx.x == 0) out.length[lane] = n;
  const T* LK = static_cast<const T*>(s.level_k);
  const T* LV = static_cast<const T*>(s.level_v);
  const T* AK = static_cast<const T*>(s.alpha_k_raw);
  const T* AV = static_cast<const T*>(s.alpha_v);
  T* OK = static_cast<T*>(out.k);
  T* OV = static_cast<T*>(out.v);
  const size_t pbase = (size_t)lane * pg.cap, obase = (size_t)lane * out.capacity;
  for (int row = blockIdx.x * 8 + warp; row < n; row += gridDim.x * 8) {
    const T* xk;
    const T* xv;
    int64_t anchor;
    float mass = 0.f;
    if (row < nv) {
      const int e = p.vslot[pbase + row];
      anchor = p.vanchor[pbase + row];
      xk = LK + (pbase + e) * D;
      xv = LV + (pbase + e) * D;
      mass = Elem<T>::round(logf(fmaxf(s.level_w[pbase + e], 1.f)));
    } else {
      const int j = p.exact_rows[(size_t)b * pg.P + row - nv];
      anchor = s.alpha_pos[(size_t)b * pg.P + j];
      xk = AK + ((size_t)lane * pg.P + j) * D;
      xv = AV + ((size_t)lane * pg.P + j) * D;
    }
    anchor = checked_anchor(anchor, r.rows, status);
    rope_row<T, C>(r, D, xk, anchor, OK + (obase + row) * D, lid);
    for (int d = lid; d < D; d += 32) OV[(obase + row) * D + d] = xv[d];
    if (lid == 0) out.mass[obase + row] = mass;
  }
}

// ---------------------------------------------------------------- K3: reference-layout pack
struct PackArgs {
  int width, alpha_count, recent_count, tokens, dim, skip_pooled, recent_start, rcap;
};

template <typename T, typename C>
__global__ void __launch_bounds__(256) pack_mid_kernel(PlanGeo pg, logkv_state_t s, logkv_plan_t p, RopeArgs r,
                                                       PackArgs a, const T* kn, const T* vn, T* ok, T* ov,
                                                       int32_t* status) {
  const int g = blockIdx.y, b = blockIdx.z, lane = b * pg.G + g, D = pg.D;
  const int warp = threadIdx.x >> 5, lid = threadIdx.x & 31;
  const int length = a.width + a.alpha_count + a.recent_count + a.tokens;
  const int first = a.width + a.alpha_count + a.recent_start;
  const T* LK = static_cast<const T*>(s.level_k);
  const T* LV = static_cast<const T*>(s.level_v);
  const T* AK = static_cast<const T*>(s.alpha_k_raw);
  const T* AV = static_cast<const T*>(s.alpha_v);
  const T* RK = static_cast<const T*>(s.recent_k);
  const T* RV = static_cast<const T*>(s.recent_v);
  const size_t pbase = (size_t)lane * pg.cap;
  const float kMask = Elem<T>::round(-10000.f);
  for (int row = blockIdx.x * 8 + warp; row < length; row += gridDim.x * 8) {
    if (row < first && (a.skip_pooled || row >= a.width + a.alpha_count)) continue;
    T* dk = ok + ((size_t)lane * length + row) * a.dim;
    T* dv = ov + ((size_t)lane * length + row) * a.dim;
    const T* xk = nullptr;
    const T* xv = nullptr;
    bool rotate = false, valid = true;
    int64_t anchor = 0;
    float extra = 0.f;
    if (row < a.width) {
      valid = p.valid[pbase + row] != 0;
      const int64_t e = p.idx[pbase + row];
      xk = LK + (pbase + e) * D;
      xv = LV + (pbase + e) * D;
      anchor = p.anchor[pbase + row];
      rotate = true;
      extra = valid ? Elem<T>::round(logf(fmaxf(s.level_w[pbase + e], 1.f))) : kMask;
    } else if (row < a.width + a.alpha_count) {
      const int j = row - a.width;
      valid = s.alpha_valid[(size_t)b * pg.P + j] != 0;
      xk = AK + ((size_t)lane * pg.P + j) * D;
      xv = AV + ((size_t)lane * pg.P + j) * D;
      anchor = s.alpha_pos[(size_t)b * pg.P + j];
      rotate = true;
      extra = valid ? -0.f : kMask;  // (~valid).to(dtype) * -10000
    } else if (row < a.width + a.alpha_count + a.recent_count) {
      const int i = row - a.width - a.alpha_count;
      xk = RK + ((size_t)lane * a.rcap + i) * D;
      xv = RV + ((size_t)lane * a.rcap + i) * D;
    } else {
      const int t = row - a.width - a.alpha_count - a.recent_count;
      xk = kn + ((size_t)lane * a.tokens + t) * D;
      xv = vn + ((size_t)lane * a.tokens + t) * D;
    }
    if (!valid) {
      for (int d = lid; d < a.dim; d += 32) {
        Elem<T>::store(dk + d, d == D ? extra : 0.f);
        Elem<T>::store(dv + d, 0.f);
      }
      continue;
    }
    if (rotate) {
      anchor = checked_anchor(anchor, r.rows, status);
      rope_row<T, C>(r, D, xk, anchor, dk, lid);
    } else {
      for (int d = lid; d < D; d += 32) dk[d] = xk[d];
    }
    for (int d = D + lid; d < a.dim; d += 32) Elem<T>::store(dk + d, d == D ? extra : 0.f);
    for (int d = lid; d < a.dim; d += 32) {
      if (d < D) dv[d] = xv[d];
      else Elem<T>::store(dv + d, 0.f);
    }
  }
}

// ---------------------------------------------------------------- K4: slot attention
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ void unpack16(const uint4& u, float* out, const float*) {
  const float* f = reinterpret_cast<const float*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) out[i] = f[i];
}
__device__ __forceinline__ void unpack16(const uint4& u, float* out, const __nv_bfloat16*) {
  const unsigned* w = reinterpret_cast<const unsigned*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

struct AttnGeo {
  int B, G, H, T, rf;
  int QS;        // token stride of the query and output rows (T unless the caller passes fewer queries)
  int TQ, qoff;  // query tokens of this call and the first one's index among the T new tokens
  int causal;
  int nsplit, pcap, rcap, rcount;
  int nsmin;     // splits a lane of the tensor-core decode kernel uses at least (fills every SM)
  int ups;       // 16-row tiles per split of the tensor-core decode kernel (attn_units_per_split)
  float scale_log2, qx;
};

constexpr int kAttnWarps = 4;
// Tensor-core decode: up to 256 lanes (batch x groups) take three cp.async stages per warp at two
// CTAs per SM and splits of 64 tiles (up to 64 lanes) or 128; more lanes two stages at three CTAs
// per SM (measured on B200 at 8305 slots per lane: 0.69 / 0.79 / 0.84 / 0.90 of HBM at batch 8 /
// 16 / 32 / 64 with 8 groups, against 0.60 / 0.61 / 0.79 / 0.90 with two stages everywhere).
constexpr int kDeepLanes = 256;
static int attn_stages(int lanes) { return lanes <= kDeepLanes ? 3 : 2; }
static int attn_units_per_split(int lanes) { return lanes <= 64 ? 64 : 128; }
constexpr int kAttnStages = 3;
// The tensor-core decode kernel keeps two tiles per warp in flight and fits three CTAs (12 warps)
// per SM, so more warps overlap one tile's math with the next tiles' loads.
constexpr int kMmaStages = 2;

template <typename T, int D, int NQ>
struct AttnShape {
  static constexpr int VN = 16 / (int)sizeof(T);    // elements per 16-byte chunk
  static constexpr int LPR = D / VN;                 // lanes per slot row
  static constexpr int GPW = 32 / LPR;               // row groups per warp
  static constexpr int TS = (32 / NQ) > GPW ? (32 / NQ) : GPW;  // slots per warp tile
  static constexpr int SPL = TS / GPW;               // slots per lane group per tile
  static constexpr int PPL = TS * NQ / 32;           // (slot, query) pairs per lane
  static constexpr size_t warp_elems = (size_t)kAttnStages * 2 * TS * D;
  static constexpr size_t smem = (size_t)kAttnWarps * (warp_elems * sizeof(T) + kAttnStages * TS * sizeof(float));
  static_assert(D % VN == 0 && LPR >= 1 && LPR <= 32 && 32 % LPR == 0, "row must be 16..512 bytes, power of two");
  static_assert(NQ >= 1 && NQ <= 32 && 32 % NQ == 0, "query rows per lane must divide 32");
};

template <typename T, int NQ>
static size_t AttnShapeFor(int D) {
  switch (D) {
    case 16: return AttnShape<T, 16, NQ>::smem;
    case 32: return AttnShape<T, 32, NQ>::smem;
    case 64: return AttnShape<T, 64, NQ>::smem;
    case 128: return AttnShape<T, 128, NQ>::smem;
    default: return 0;
  }
}

// Last-CTA combine of a lane's split partials ([m, l, o[D]] per split and query row): every
// row's maximum over the splits and each split's weight exp2(m_s - max) go to shared memory
// `wsh` ([nsplit][NQ] weights, [nsplit][NQ] sums, [NQ] row sums); then every output column's
// weighted sum over the splits, its loads unrolled.  Same operations in the same split order as
// one pass over the splits per output, so the result is the same.
template <typename T, int D, int NQ>
__device__ void combine_splits(const AttnGeo& a, const float* part, T* out, int ln, int b, int g, float* wsh,
                               int ns) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const size_t pstride = (size_t)D + 2;
  float* wgt = wsh;                 // [ns][NQ]
  float* lsp = wsh + ns * NQ;       // [ns][NQ]
  float* rl = lsp + ns * NQ;        // [NQ] row sums, -1 marks a row without any finite score
  for (int x = tid; x < ns * NQ; x += nt) {
    const float* pp = part + ((size_t)ln * a.nsplit * NQ + x) * pstride;   // split x / NQ, row x % NQ
    wgt[x] = __ldcg(pp);
    lsp[x] = __ldcg(pp + 1);
  }
  __syncthreads();
  if (tid < NQ) {
    const int r = tid;
    float mx = -INFINITY;
    for (int sidx = 0; sidx < ns; ++sidx) mx = fmaxf(mx, wgt[sidx * NQ + r]);
    float l = 0.f;
    if (mx != -INFINITY) {
      for (int sidx = 0; sidx < ns; ++sidx) {
        const float f = exp2f(wgt[sidx * NQ + r] - mx);
        l += lsp[sidx * NQ + r] * f;
        wgt[sidx * NQ + r] = f;
      }
      rl[r] = l;
    } else {
      rl[r] = -1.f;
    }
  }
  __syncthreads();
  for (int x = tid; x < NQ * D; x += nt) {
    const int r = x / D, d = x % D;
    const float l = rl[r];
    float o = 0.f;
    if (l >= 0.f) {
      const float* pp = part + ((size_t)ln * a.nsplit * NQ + r) * pstride + 2 + d;
#pragma unroll 8
      for (int sidx = 0; sidx < ns; ++sidx) o += __ldcg(pp + (size_t)sidx * NQ * pstride) * wgt[sidx * NQ + r];
    }
    const int h = g * a.rf + r / a.TQ, t = a.qoff + r % a.TQ;
    Elem<T>::store(out + (((size_t)b * a.H + h) * a.QS + t) * D + d, l > 0.f ? o / l : 0.f);
  }
}

template <typename T, int D, int NQ>
__global__ void __launch_bounds__(kAttnWarps * 32) slot_attn_kernel(AttnGeo a, logkv_prefix_t pre, const T* rk,
                                                                   const T* rv, const T* kn, const T* vn, const T* q,
                                                                   T* out, float* part, int* ticket) {
  using S = AttnShape<T, D, NQ>;
  constexpr int VN = S::VN, LPR = S::LPR, GPW = S::GPW, TS = S::TS, SPL = S::SPL, PPL = S::PPL;
  extern __shared__ uint4 smem4[];
  __shared__ float sp[kAttnWarps][TS * NQ];
  __shared__ float wm_[kAttnWarps][NQ];
  __shared__ float wl_[kAttnWarps][NQ];
  __shared__ int sh_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int grp = lane / LPR, u = lane % LPR;
  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z, ln = b * a.G + g;
  T* wbuf = reinterpret_cast<T*>(smem4) + (size_t)warp * S::warp_elems;
  float* wmass = reinterpret_cast<float*>(reinterpret_cast<T*>(smem4) + (size_t)kAttnWarps * S::warp_elems) +
                 warp * kAttnStages * TS;
  const T* PK = static_cast<const T*>(pre.k);
  const T* PV = static_cast<const T*>(pre.v);
  const int Lp = min(max(pre.length[ln], 0), pre.capacity), R = a.rcount, Stot = Lp + R + a.T;
  int per = (Stot + a.nsplit - 1) / a.nsplit;
  per = (per + TS - 1) / TS * TS;
  const int s0 = min(Stot, split * per), s1 = min(Stot, s0 + per);
  const int ntile = (s1 - s0 + TS - 1) / TS;
  const int mine = ntile > warp ? (ntile - warp + kAttnWarps - 1) / kAttnWarps : 0;

  float qf[NQ][VN];
#pragma unroll
  for (int r = 0; r < NQ; ++r) {
    const int h = g * a.rf + r / a.TQ, t = a.qoff + r % a.TQ;
    const uint4 raw = *reinterpret_cast<const uint4*>(q + (((size_t)b * a.H + h) * a.QS + t) * D + u * VN);
    unpack16(raw, qf[r], (const T*)nullptr);
  }

  auto issue = [&](int k, int stage) {
    if (k < mine) {
      const int t0 = s0 + (warp + k * kAttnWarps) * TS;
      T* dk = wbuf + (size_t)stage * 2 * TS * D;
      T* dv = dk + TS * D;
#pragma unroll
      for (int i = 0; i < SPL; ++i) {
        const int ts = grp + GPW * i, sl = t0 + ts;
        if (sl < s1) {
          const T* sk;
          const T* sv;
          if (sl < Lp) {
            const size_t row = (size_t)ln * pre.capacity + sl;
            sk = PK + row * D;
            sv = PV + row * D;
            if (u == 0) cp_async4(wmass + stage * TS + ts, pre.mass + row);
          } else {
            if (sl < Lp + R) {
              const size_t row = (size_t)ln * a.rcap + (sl - Lp);
              sk = rk + row * D;
              sv = rv + row * D;
            } else {
              const size_t row = (size_t)ln * a.T + (sl - Lp - R);
              sk = kn + row * D;
              sv = vn + row * D;
            }
            if (u == 0) wmass[stage * TS + ts] = 0.f;
          }
          cp_async16(dk + ts * D + u * VN, sk + u * VN);
          cp_async16(dv + ts * D + u * VN, sv + u * VN);
        } else {
          // Past the split's last slot: zeros, so the masked products (probability 0) stay 0.
          *reinterpret_cast<uint4*>(dk + ts * D + u * VN) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(dv + ts * D + u * VN) = make_uint4(0, 0, 0, 0);
        }
      }
    }
    cp_async_commit();
  };

  float m[NQ], acc[NQ][VN];
#pragma unroll
  for (int r = 0; r < NQ; ++r) {
    m[r] = -INFINITY;
#pragma unroll
    for (int e = 0; e < VN; ++e) acc[r][e] = 0.f;
  }
  float lsum = 0.f;
  const int rown = lane % NQ;

#pragma unroll
  for (int k = 0; k < kAttnStages - 1; ++k) issue(k, k);
  for (int k = 0; k < mine; ++k) {
    issue(k + kAttnStages - 1, (k + kAttnStages - 1) % kAttnStages);
    cp_async_wait<kAttnStages - 1>();
    const int stage = k % kAttnStages;
    const int t0 = s0 + (warp + k * kAttnWarps) * TS;
    const T* ck = wbuf + (size_t)stage * 2 * TS * D;
    const T* cv = ck + TS * D;
    // Scores of this lane group's slots: partial dots over the lane's chunk, then the group sum.
    float z[SPL][NQ];
#pragma unroll
    for (int i = 0; i < SPL; ++i) {
      float kf[VN];
      unpack16(*reinterpret_cast<const uint4*>(ck + (grp + GPW * i) * D + u * VN), kf, (const T*)nullptr);
#pragma unroll
      for (int r = 0; r < NQ; ++r) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < VN; ++e) d = fmaf(qf[r][e], kf[e], d);
        z[i][r] = d;
      }
    }
#pragma unroll
    for (int off = 1; off < LPR; off <<= 1)
#pragma unroll
      for (int i = 0; i < SPL; ++i)
#pragma unroll
        for (int r = 0; r < NQ; ++r) z[i][r] += __shfl_xor_sync(0xffffffffu, z[i][r], off);
    if (u == 0) {
#pragma unroll
      for (int i = 0; i < SPL; ++i) {
        const int ts = grp + GPW * i, sl = t0 + ts;
        const float mass = wmass[stage * TS + ts];
#pragma unroll
        for (int r = 0; r < NQ; ++r) {
          const int c = sl - Lp - R;  // new-token index (>= 0 in the causal tail)
          const bool vis = sl < s1 && (c < 0 || !a.causal || c <= a.qoff + r % a.TQ);
          sp[warp][ts * NQ + r] = vis ? (z[i][r] + a.qx * mass) * a.scale_log2 : -INFINITY;
        }
      }
    }
    __syncwarp();
    // Online softmax: this lane owns pairs j * 32 + lane, all of query row `rown`.
    float zl[PPL], mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < PPL; ++j) {
      zl[j] = sp[warp][j * 32 + lane];
      mt = fmaxf(mt, zl[j]);
    }
#pragma unroll
    for (int off = NQ; off < 32; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
    float alpha[NQ], mown = -INFINITY, aown = 1.f;
#pragma unroll
    for (int r = 0; r < NQ; ++r) {
      const float mn = fmaxf(m[r], __shfl_sync(0xffffffffu, mt, r));
      alpha[r] = mn == -INFINITY ? 1.f : exp2f(m[r] - mn);
      m[r] = mn;
      if (r == rown) {
        mown = mn;
        aown = alpha[r];
      }
    }
    float ps = 0.f;
#pragma unroll
    for (int j = 0; j < PPL; ++j) {
      const float pj = zl[j] == -INFINITY ? 0.f : exp2f(zl[j] - mown);
      sp[warp][j * 32 + lane] = pj;
      ps += pj;
    }
    lsum = lsum * aown + ps;
    __syncwarp();
#pragma unroll
    for (int r = 0; r < NQ; ++r)
#pragma unroll
      for (int e = 0; e < VN; ++e) acc[r][e] *= alpha[r];
#pragma unroll
    for (int i = 0; i < SPL; ++i) {
      const int ts = grp + GPW * i;
      float vf[VN];
      unpack16(*reinterpret_cast<const uint4*>(cv + ts * D + u * VN), vf, (const T*)nullptr);
#pragma unroll
      for (int r = 0; r < NQ; ++r) {
        const float pr = sp[warp][ts * NQ + r];
#pragma unroll
        for (int e = 0; e < VN; ++e) acc[r][e] = fmaf(pr, vf[e], acc[r][e]);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  // Warp totals: row sums over the lanes of each query row, accumulators over the lane groups.
#pragma unroll
  for (int off = NQ; off < 32; off <<= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
#pragma unroll
  for (int r = 0; r < NQ; ++r)
#pragma unroll
    for (int off = LPR; off < 32; off <<= 1)
#pragma unroll
      for (int e = 0; e < VN; ++e) acc[r][e] += __shfl_xor_sync(0xffffffffu, acc[r][e], off);
  float* wacc = reinterpret_cast<float*>(wbuf);  // [NQ][D], reuses this warp's own ring
#pragma unroll
  for (int r = 0; r < NQ; ++r) {
    const float lr = __shfl_sync(0xffffffffu, lsum, r);
    if (lane == 0) {
      wm_[warp][r] = m[r];
      wl_[warp][r] = lr;
    }
    if (grp == 0) {
#pragma unroll
      for (int e = 0; e < VN; ++e) wacc[r * D + u * VN + e] = acc[r][e];
    }
  }
  __syncthreads();
  // CTA combine (fixed warp order), then either the output or this split's partial.
  const size_t pstride = (size_t)D + 2;
  for (int x = tid; x < NQ * D; x += blockDim.x) {
    const int r = x / D, d = x % D;
    float mx = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, wm_[w][r]);
    float l = 0.f, o = 0.f;
    if (mx != -INFINITY) {
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = exp2f(wm_[w][r] - mx);
        l += wl_[w][r] * f;
        o += reinterpret_cast<float*>(reinterpret_cast<T*>(smem4) + (size_t)w * S::warp_elems)[r * D + d] * f;
      }
    }
    if (a.nsplit == 1) {
      const int h = g * a.rf + r / a.TQ, t = a.qoff + r % a.TQ;
      Elem<T>::store(out + (((size_t)b * a.H + h) * a.QS + t) * D + d, l > 0.f ? o / l : 0.f);
    } else {
      float* pp = part + ((size_t)(ln * a.nsplit + split) * NQ + r) * pstride;
      if (d == 0) {
        pp[0] = mx;
        pp[1] = l;
      }
      pp[2 + d] = o;
    }
  }
  if (a.nsplit == 1) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) sh_last = atomicAdd(ticket + ln, 1) == a.nsplit - 1;
  __syncthreads();
  if (!sh_last) return;
  __threadfence();
  combine_splits<T, D, NQ>(a, part, out, ln, b, g, reinterpret_cast<float*>(smem4), a.nsplit);
  if (tid == 0) ticket[ln] = 0;
}

// ---------------------------------------------------------------- K4b: slot attention on tensor cores (bf16)
// The query rows of a lane (heads per group x query tokens <= 16) are the M = 16 rows of
// mma.sync.m16n8k16: per 16-slot tile QK^T is D/16 x 2 MMAs and PV is D/8 MMAs whose A
// operand is the score accumulator itself.  Tiles never straddle the three segments
// (prefix, window, new tokens), so a tile's K and V rows are contiguous blocks; each lane
// copies 16-byte chunks into an XOR-swizzled stage (conflict-free ldmatrix), and a
// __syncwarp after cp.async.wait_group makes every lane's chunks visible to the warp.
__device__ __forceinline__ void ldsm_x4(unsigned addr, unsigned& r0, unsigned& r1, unsigned& r2, unsigned& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(unsigned addr, unsigned& r0, unsigned& r1, unsigned& r2, unsigned& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0,
                                         unsigned b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ unsigned pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const unsigned*>(&v);
}

template <int D, int ST = kMmaStages>
struct MmaShape {
  static constexpr int TS = 16;             // slots per tile (two n8 score tiles, one k16 PV step)
  static constexpr int CPR = D / 8;         // 16-byte chunks per row
  static constexpr int KS = D / 16;         // k16 steps of QK^T
  static constexpr int DT = D / 8;          // n8 output tiles of PV
  static constexpr int STAGE_BYTES = 2 * TS * D * 2 + TS * 4;   // K, V (bf16) and the mass column
  static constexpr size_t smem = (size_t)kAttnWarps * ST * STAGE_BYTES;   // ST stages per warp
  static_assert(D % 16 == 0 && D >= 16 && D <= 256, "head dim must be a multiple of 16 up to 256");
  // Physical 16-byte chunk of logical chunk c in row r: rows of 8 consecutive ldmatrix
  // addresses land in 8 distinct 16-byte bank groups.
  __device__ __forceinline__ static int swz(int r, int c) {
    if (CPR >= 8) return c ^ (r & 7);
    return c ^ ((r * CPR / 8) & (CPR - 1));
  }
};

template <int D, int NQ, int ST>
__global__ void __launch_bounds__(kAttnWarps * 32, ST == 2 ? 3 : 2) slot_attn_mma_kernel(AttnGeo a, logkv_prefix_t pre,
                                                                       const __nv_bfloat16* rk,
                                                                       const __nv_bfloat16* rv,
                                                                       const __nv_bfloat16* kn,
                                                                       const __nv_bfloat16* vn,
                                                                       const __nv_bfloat16* q, __nv_bfloat16* out,
                                                                       float* part, int* ticket) {
  using S = MmaShape<D, ST>;
  constexpr int TS = S::TS, CPR = S::CPR, KS = S::KS, DT = S::DT;
  static_assert(NQ >= 1 && NQ <= 16, "at most 16 query rows per lane");
  extern __shared__ uint4 smem4[];
  __shared__ float wm_[kAttnWarps][NQ];
  __shared__ float wl_[kAttnWarps][NQ];
  __shared__ int sh_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int g8 = lane >> 2, t4 = lane & 3;  // fragment row group and column pair
  const int ln = blockIdx.x, split = blockIdx.y, g = ln % a.G, b = ln / a.G;
  unsigned char* wbase = reinterpret_cast<unsigned char*>(smem4) + (size_t)warp * ST * S::STAGE_BYTES;
  const unsigned wbase_s = (unsigned)__cvta_generic_to_shared(wbase);
  const __nv_bfloat16* PK = static_cast<const __nv_bfloat16*>(pre.k);
  const __nv_bfloat16* PV = static_cast<const __nv_bfloat16*>(pre.v);
  // Work units: tiles of 16 rows inside each segment.
  const int Lp = min(max(pre.length[ln], 0), pre.capacity), R = a.rcount, Tn = a.T;
  const int up = (Lp + TS - 1) / TS, ur = (R + TS - 1) / TS, uc = (Tn + TS - 1) / TS;
  const int U = up + ur + uc;
  // This lane's splits: about a.ups tiles each (long streams per warp), at least
  // a.nsmin (every SM busy at small batch); the grid's further splits return at once.
  const int ns = min(a.nsplit, max(a.nsmin, U / a.ups));
  if (split >= ns) return;
  const int u0 = (int)((long long)U * split / ns), u1 = (int)((long long)U * (split + 1) / ns);
  const int mine = (u1 - u0) > warp ? (u1 - u0 - warp + kAttnWarps - 1) / kAttnWarps : 0;

  // Query A fragments (rows g8 and g8 + 8 of the 16, zero past NQ), loop invariant.
  unsigned qa[KS][4];
  {
    const int r0 = g8, r1 = g8 + 8;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int hrow = 0; hrow < 2; ++hrow) {
        const int r = hrow ? r1 : r0;
        unsigned lo = 0u, hi = 0u;
        if (r < NQ) {
          const int h = g * a.rf + r / a.TQ, t = a.qoff + r % a.TQ;
          const __nv_bfloat16* qp = q + (((size_t)b * a.H + h) * a.QS + t) * D + ks * 16 + 2 * t4;
          lo = *reinterpret_cast<const unsigned*>(qp);
          hi = *reinterpret_cast<const unsigned*>(qp + 8);
        }
        qa[ks][hrow] = lo;       // a0a1 (row g8) / a2a3 (row g8+8)
        qa[ks][2 + hrow] = hi;   // a4a5 / a6a7
      }
    }
  }

  // Unit -> (segment base of K, V, mass; first row; rows in the tile; slot class).
  auto unit_info = [&](int u, const __nv_bfloat16*& kb, const __nv_bfloat16*& vb, const float*& mb, int& rows,
                       int& cls, int& first) {
    if (u < up) {
      first = u * TS;
      rows = min(TS, Lp - first);
      const size_t r = (size_t)ln * pre.capacity + first;
      kb = PK + r * D;
      vb = PV + r * D;
      mb = pre.mass + r;
      cls = 0;
    } else if (u < up + ur) {
      first = (u - up) * TS;
      rows = min(TS, R - first);
      const size_t r = (size_t)ln * a.rcap + first;
      kb = rk + r * D;
      vb = rv + r * D;
      mb = nullptr;
      cls = 1;
    } else {
      first = (u - up - ur) * TS;
      rows = min(TS, Tn - first);
      const size_t r = (size_t)ln * a.T + first;
      kb = kn + r * D;
      vb = vn + r * D;
      mb = nullptr;
      cls = 2;
    }
  };

  auto issue = [&](int k, int stage) {
    if (k < mine) {
      const __nv_bfloat16 *kb, *vb;
      const float* mb;
      int rows, cls, first;
      unit_info(u0 + warp + k * kAttnWarps, kb, vb, mb, rows, cls, first);
      unsigned char* st = wbase + (size_t)stage * S::STAGE_BYTES;
      unsigned char* sk = st;
      unsigned char* sv = st + TS * D * 2;
      float* sm = reinterpret_cast<float*>(st + 2 * TS * D * 2);
#pragma unroll
      for (int i = 0; i < (TS * CPR + 31) / 32; ++i) {
        const int flat = i * 32 + lane;
        if (flat < TS * CPR) {
          const int r = flat / CPR, c = flat % CPR;
          const int off = r * D * 2 + S::swz(r, c) * 16;
          if (r < rows) {
            cp_async16(sk + off, kb + (size_t)flat * 8);
            cp_async16(sv + off, vb + (size_t)flat * 8);
          } else {
            *reinterpret_cast<uint4*>(sk + off) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(sv + off) = make_uint4(0, 0, 0, 0);
          }
        }
      }
      if (lane < TS) {
        if (cls == 0 && lane < rows) cp_async4(sm + lane, mb + lane);
        else sm[lane] = 0.f;
      }
    }
    cp_async_commit();
  };

  float o[DT][4];
#pragma unroll
  for (int j = 0; j < DT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g8 and g8 + 8
  const int rq0 = g8 % a.TQ, rq1 = (g8 + 8) % a.TQ;         // query token of each row

#pragma unroll
  for (int k = 0; k < ST - 1; ++k) issue(k, k);
  for (int k = 0; k < mine; ++k) {
    issue(k + ST - 1, (k + ST - 1) % ST);
    cp_async_wait<ST - 1>();
    __syncwarp();
    const int stage = k % ST;
    const __nv_bfloat16 *kb_, *vb_;
    const float* mb_;
    int rows, cls, first;
    unit_info(u0 + warp + k * kAttnWarps, kb_, vb_, mb_, rows, cls, first);
    const unsigned sk = wbase_s + stage * S::STAGE_BYTES;
    const unsigned sv = sk + TS * D * 2;
    const float* sm = reinterpret_cast<const float*>(wbase + (size_t)stage * S::STAGE_BYTES + 2 * TS * D * 2);
    // S = Q K^T for the 16 slots: two n8 tiles.
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      // matrices: (tile 0, chunk 2ks), (tile 0, chunk 2ks+1), (tile 1, chunk 2ks), (tile 1, chunk 2ks+1)
      const int mi = lane >> 3, rr = (mi >> 1) * 8 + (lane & 7), cc = 2 * ks + (mi & 1);
      unsigned b0, b1, b2, b3;
      ldsm_x4(sk + rr * D * 2 + S::swz(rr, cc) * 16, b0, b1, b2, b3);
      mma_bf16(sc[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
      mma_bf16(sc[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
    }
    // Scores in the log2 domain with the mass term and masks; columns 8 j + 2 t4 + e.
    float mt0 = -INFINITY, mt1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = 8 * j + 2 * t4 + e;
        const float mass = sm[col];
        const bool in = col < rows;
        const bool v0 = in && (cls != 2 || !a.causal || first + col <= a.qoff + rq0);
        const bool v1 = in && (cls != 2 || !a.causal || first + col <= a.qoff + rq1);
        sc[j][e] = v0 ? (sc[j][e] + a.qx * mass) * a.scale_log2 : -INFINITY;
        sc[j][2 + e] = v1 ? (sc[j][2 + e] + a.qx * mass) * a.scale_log2 : -INFINITY;
        mt0 = fmaxf(mt0, sc[j][e]);
        mt1 = fmaxf(mt1, sc[j][2 + e]);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, off));
      mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, off));
    }
    const float mn0 = fmaxf(m0, mt0), mn1 = fmaxf(m1, mt1);
    const float al0 = mn0 == -INFINITY ? 1.f : exp2f(m0 - mn0);
    const float al1 = mn1 == -INFINITY ? 1.f : exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float p[2][4];
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        p[j][e] = sc[j][e] == -INFINITY ? 0.f : exp2f(sc[j][e] - mn0);
        p[j][2 + e] = sc[j][2 + e] == -INFINITY ? 0.f : exp2f(sc[j][2 + e] - mn1);
        s0 += p[j][e];
        s1 += p[j][2 + e];
      }
    }
    l0 = l0 * al0 + s0;
    l1 = l1 * al1 + s1;
    if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
      for (int jd = 0; jd < DT; ++jd) {
        o[jd][0] *= al0;
        o[jd][1] *= al0;
        o[jd][2] *= al1;
        o[jd][3] *= al1;
      }
    }
    // O += P V: P's A fragment is the score accumulator (k = the 16 slots).
    const unsigned pa0 = pack_bf16x2(p[0][0], p[0][1]), pa1 = pack_bf16x2(p[0][2], p[0][3]);
    const unsigned pa2 = pack_bf16x2(p[1][0], p[1][1]), pa3 = pack_bf16x2(p[1][2], p[1][3]);
#pragma unroll
    for (int jd = 0; jd < DT; jd += 2) {
      // matrices: (slots 0-7, chunk jd), (slots 8-15, chunk jd), (slots 0-7, chunk jd+1), (slots 8-15, chunk jd+1)
      const int mi = lane >> 3, rr = (mi & 1) * 8 + (lane & 7), cc = jd + (mi >> 1);
      unsigned b0, b1, b2, b3;
      ldsm_x4_t(sv + rr * D * 2 + S::swz(rr, cc) * 16, b0, b1, b2, b3);
      mma_bf16(o[jd], pa0, pa1, pa2, pa3, b0, b1);
      mma_bf16(o[jd + 1], pa0, pa1, pa2, pa3, b2, b3);
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  __syncwarp();
  // Row sums over the four lanes of each row group.
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  float* wacc = reinterpret_cast<float*>(wbase);  // [NQ][D], this warp's own ring
  if (t4 == 0) {
    if (g8 < NQ) {
      wm_[warp][g8] = m0;
      wl_[warp][g8] = l0;
    }
    if (g8 + 8 < NQ) {
      wm_[warp][g8 + 8] = m1;
      wl_[warp][g8 + 8] = l1;
    }
  }
#pragma unroll
  for (int jd = 0; jd < DT; ++jd) {
    const int c0 = jd * 8 + 2 * t4;
    if (g8 < NQ) {
      wacc[g8 * D + c0] = o[jd][0];
      wacc[g8 * D + c0 + 1] = o[jd][1];
    }
    if (g8 + 8 < NQ) {
      wacc[(g8 + 8) * D + c0] = o[jd][2];
      wacc[(g8 + 8) * D + c0 + 1] = o[jd][3];
    }
  }
  __syncthreads();
  const size_t pstride = (size_t)D + 2;
  for (int x = tid; x < NQ * D; x += blockDim.x) {
    const int r = x / D, d = x % D;
    float mx = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, wm_[w][r]);
    float l = 0.f, ov = 0.f;
    if (mx != -INFINITY) {
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = exp2f(wm_[w][r] - mx);
        l += wl_[w][r] * f;
        ov += reinterpret_cast<const float*>(reinterpret_cast<unsigned char*>(smem4) +
                                             (size_t)w * ST * S::STAGE_BYTES)[r * D + d] * f;
      }
    }
    if (ns == 1) {
      const int h = g * a.rf + r / a.TQ, t = a.qoff + r % a.TQ;
      out[(((size_t)b * a.H + h) * a.QS + t) * D + d] = __float2bfloat16_rn(l > 0.f ? ov / l : 0.f);
    } else {
      float* pp = part + ((size_t)(ln * a.nsplit + split) * NQ + r) * pstride;
      if (d == 0) {
        pp[0] = mx;
        pp[1] = l;
      }
      pp[2 + d] = ov;
    }
  }
  if (ns == 1) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) sh_last = atomicAdd(ticket + ln, 1) == ns - 1;
  __syncthreads();
  if (!sh_last) return;
  __threadfence();
  combine_splits<__nv_bfloat16, D, NQ>(a, part, out, ln, b, g, reinterpret_cast<float*>(smem4), ns);
  if (tid == 0) ticket[ln] = 0;
}

// ---------------------------------------------------------------- K5: chunk (prefill) attention on tensor cores
// One CTA = 128 query rows of a lane (rf heads x 128/rf consecutive tokens); warp w owns rows
// 16w..16w+15 (one head, 16 consecutive tokens).  All warps share 64-slot K/V tiles staged
// by the whole CTA through a cp.async ring; per tile and warp QK^T is 8 n-tiles x D/16
// k-steps and PV is D/8 n-tiles x 4 k-steps of mma.sync.m16n8k16 (bf16 in, f32 accumulate).
// New-token tiles entirely after the CTA's last query token are skipped.
constexpr int kPfWarps = 8;
constexpr int kPfRows = 16 * kPfWarps;  // query rows per CTA
constexpr int kPfTS = 64;               // slots per tile
constexpr int kPfStages = 3;

template <int D>
struct PfShape {
  static constexpr int CPR = D / 8, KS = D / 16, DT = D / 8;
  static constexpr int TILE_BYTES = kPfTS * D * 2;                      // one of K / V
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES + kPfTS * 4;        // K, V, mass
  static constexpr size_t smem = (size_t)kPfStages * STAGE_BYTES;
  __device__ __forceinline__ static int swz(int r, int c) { return MmaShape<D>::swz(r, c); }
};

template <int D>
__global__ void __launch_bounds__(kPfWarps * 32) chunk_attn_mma_kernel(AttnGeo a, logkv_prefix_t pre,
                                                                      const __nv_bfloat16* rk,
                                                                      const __nv_bfloat16* rv,
                                                                      const __nv_bfloat16* kn,
                                                                      const __nv_bfloat16* vn,
                                                                      const __nv_bfloat16* q, __nv_bfloat16* out) {
  using S = PfShape<D>;
  constexpr int CPR = S::CPR, KS = S::KS, DT = S::DT, TS = kPfTS;
  extern __shared__ uint4 smem4[];
  unsigned char* sbase = reinterpret_cast<unsigned char*>(smem4);
  const unsigned sbase_s = (unsigned)__cvta_generic_to_shared(sbase);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int g = blockIdx.y, b = blockIdx.z, ln = b * a.G + g;
  const int QT = kPfRows / a.rf;                       // tokens per CTA
  const int tq0 = a.qoff + blockIdx.x * QT;            // first query token of the CTA
  const int row0 = warp * 16;                          // this warp's first row
  const int hh = row0 / QT, tw = tq0 + row0 % QT;      // head-in-group and first token of the warp
  const int h = g * a.rf + hh;
  const int tlast = min(a.qoff + a.TQ, tq0 + QT) - 1;  // CTA's last query token
  const __nv_bfloat16* PK = static_cast<const __nv_bfloat16*>(pre.k);
  const __nv_bfloat16* PV = static_cast<const __nv_bfloat16*>(pre.v);
  const int Lp = min(max(pre.length[ln], 0), pre.capacity), R = a.rcount;
  const int Tvis = a.causal ? min(a.T, tlast + 1) : a.T;   // new tokens any row of the CTA can see
  const int up = (Lp + TS - 1) / TS, ur = (R + TS - 1) / TS, uc = (Tvis + TS - 1) / TS;
  const int U = up + ur + uc;

  // Query A fragments of the warp's 16 rows (tokens tw .. tw+15 of head h).
  unsigned qa[KS][4];
  {
    const int t0r = tw + g8, t1r = tw + g8 + 8;
    const bool ok0 = t0r < a.qoff + a.TQ, ok1 = t1r < a.qoff + a.TQ;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const __nv_bfloat16* q0 = q + (((size_t)b * a.H + h) * a.QS + t0r) * D + ks * 16 + 2 * t4;
      const __nv_bfloat16* q1 = q + (((size_t)b * a.H + h) * a.QS + t1r) * D + ks * 16 + 2 * t4;
      qa[ks][0] = ok0 ? *reinterpret_cast<const unsigned*>(q0) : 0u;
      qa[ks][1] = ok1 ? *reinterpret_cast<const unsigned*>(q1) : 0u;
      qa[ks][2] = ok0 ? *reinterpret_cast<const unsigned*>(q0 + 8) : 0u;
      qa[ks][3] = ok1 ? *reinterpret_cast<const unsigned*>(q1 + 8) : 0u;
    }
  }

  auto unit_info = [&](int u, const __nv_bfloat16*& kb, const __nv_bfloat16*& vb, const float*& mb, int& rows,
                       int& cls, int& first) {
    if (u < up) {
      first = u * TS;
      rows = min(TS, Lp - first);
      const size_t r = (size_t)ln * pre.capacity + first;
      kb = PK + r * D;
      vb = PV + r * D;
      mb = pre.mass + r;
      cls = 0;
    } else if (u < up + ur) {
      first = (u - up) * TS;
      rows = min(TS, R - first);
      const size_t r = (size_t)ln * a.rcap + first;
      kb = rk + r * D;
      vb = rv + r * D;
      mb = nullptr;
      cls = 1;
    } else {
      first = (u - up - ur) * TS;
      rows = min(TS, Tvis - first);
      const size_t r = (size_t)ln * a.T + first;
      kb = kn + r * D;
      vb = vn + r * D;
      mb = nullptr;
      cls = 2;
    }
  };

  auto issue = [&](int u, int stage) {
    if (u < U) {
      const __nv_bfloat16 *kb, *vb;
      const float* mb;
      int rows, cls, first;
      unit_info(u, kb, vb, mb, rows, cls, first);
      unsigned char* st = sbase + (size_t)stage * S::STAGE_BYTES;
      unsigned char* sk = st;
      unsigned char* sv = st + S::TILE_BYTES;
      float* sm = reinterpret_cast<float*>(st + 2 * S::TILE_BYTES);
      for (int flat = tid; flat < TS * CPR; flat += kPfWarps * 32) {
        const int r = flat / CPR, c = flat % CPR;
        const int off = r * D * 2 + S::swz(r, c) * 16;
        if (r < rows) {
          cp_async16(sk + off, kb + (size_t)flat * 8);
          cp_async16(sv + off, vb + (size_t)flat * 8);
        } else {
          *reinterpret_cast<uint4*>(sk + off) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(sv + off) = make_uint4(0, 0, 0, 0);
        }
      }
      if (tid < TS) {
        if (cls == 0 && tid < rows) cp_async4(sm + tid, mb + tid);
        else sm[tid] = 0.f;
      }
    }
    cp_async_commit();
  };

  float o[DT][4];
#pragma unroll
  for (int j = 0; j < DT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int tr0 = tw + g8, tr1 = tw + g8 + 8;  // query tokens of the lane's two rows

#pragma unroll
  for (int k = 0; k < kPfStages - 1; ++k) issue(k, k);
  for (int u = 0; u < U; ++u) {
    issue(u + kPfStages - 1, (u + kPfStages - 1) % kPfStages);
    cp_async_wait<kPfStages - 1>();
    __syncthreads();
    const int stage = u % kPfStages;
    const __nv_bfloat16 *kb_, *vb_;
    const float* mb_;
    int rows, cls, first;
    unit_info(u, kb_, vb_, mb_, rows, cls, first);
    const unsigned sk = sbase_s + stage * S::STAGE_BYTES;
    const unsigned sv = sk + S::TILE_BYTES;
    const float* sm = reinterpret_cast<const float*>(sbase + (size_t)stage * S::STAGE_BYTES + 2 * S::TILE_BYTES);
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        const int mi = lane >> 3, rr = (2 * jp + (mi >> 1)) * 8 + (lane & 7), cc = 2 * ks + (mi & 1);
        unsigned b0, b1, b2, b3;
        ldsm_x4(sk + rr * D * 2 + S::swz(rr, cc) * 16, b0, b1, b2, b3);
        mma_bf16(sc[2 * jp], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
        mma_bf16(sc[2 * jp + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
      }
    }
    float mt0 = -INFINITY, mt1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = 8 * j + 2 * t4 + e;
        const float mass = sm[col];
        const bool in = col < rows;
        const bool v0 = in && (cls != 2 || !a.causal || first + col <= tr0);
        const bool v1 = in && (cls != 2 || !a.causal || first + col <= tr1);
        sc[j][e] = v0 ? (sc[j][e] + a.qx * mass) * a.scale_log2 : -INFINITY;
        sc[j][2 + e] = v1 ? (sc[j][2 + e] + a.qx * mass) * a.scale_log2 : -INFINITY;
        mt0 = fmaxf(mt0, sc[j][e]);
        mt1 = fmaxf(mt1, sc[j][2 + e]);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, off));
      mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, off));
    }
    const float mn0 = fmaxf(m0, mt0), mn1 = fmaxf(m1, mt1);
    const float al0 = mn0 == -INFINITY ? 1.f : exp2f(m0 - mn0);
    const float al1 = mn1 == -INFINITY ? 1.f : exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sc[j][e] = sc[j][e] == -INFINITY ? 0.f : exp2f(sc[j][e] - mn0);
        sc[j][2 + e] = sc[j][2 + e] == -INFINITY ? 0.f : exp2f(sc[j][2 + e] - mn1);
        s0 += sc[j][e];
        s1 += sc[j][2 + e];
      }
    }
    l0 = l0 * al0 + s0;
    l1 = l1 * al1 + s1;
    if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
      for (int jd = 0; jd < DT; ++jd) {
        o[jd][0] *= al0;
        o[jd][1] *= al0;
        o[jd][2] *= al1;
        o[jd][3] *= al1;
      }
    }
#pragma unroll
    for (int kk = 0; kk < TS / 16; ++kk) {
      const unsigned pa0 = pack_bf16x2(sc[2 * kk][0], sc[2 * kk][1]);
      const unsigned pa1 = pack_bf16x2(sc[2 * kk][2], sc[2 * kk][3]);
      const unsigned pa2 = pack_bf16x2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
      const unsigned pa3 = pack_bf16x2(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
      for (int jd = 0; jd < DT; jd += 2) {
        const int mi = lane >> 3, rr = 16 * kk + (mi & 1) * 8 + (lane & 7), cc = jd + (mi >> 1);
        unsigned b0, b1, b2, b3;
        ldsm_x4_t(sv + rr * D * 2 + S::swz(rr, cc) * 16, b0, b1, b2, b3);
        mma_bf16(o[jd], pa0, pa1, pa2, pa3, b0, b1);
        mma_bf16(o[jd + 1], pa0, pa1, pa2, pa3, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const bool ok0 = tr0 < a.qoff + a.TQ, ok1 = tr1 < a.qoff + a.TQ;
#pragma unroll
  for (int jd = 0; jd < DT; ++jd) {
    const int c0 = jd * 8 + 2 * t4;
    if (ok0)
      *reinterpret_cast<__nv_bfloat162*>(out + (((size_t)b * a.H + h) * a.QS + tr0) * D + c0) =
          __floats2bfloat162_rn(o[jd][0] * inv0, o[jd][1] * inv0);
    if (ok1)
      *reinterpret_cast<__nv_bfloat162*>(out + (((size_t)b * a.H + h) * a.QS + tr1) * D + c0) =
          __floats2bfloat162_rn(o[jd][2] * inv1, o[jd][3] * inv1);
  }
}

// ---------------------------------------------------------------- K6: chunk attention on tcgen05 / TMEM
// One CTA = NQ tiles of 128 query rows of a lane (each rf heads x 128/rf tokens), the M of
// tcgen05.mma.cta_group::1.kind::f16 (bf16 in, f32 accumulate); every K/V tile the loaders
// bring in serves all NQ query tiles.  Warp roles:
//   warps 0..4NQ-1  softmax, one warpgroup per query tile: thread = query row = TMEM lane; read
//                   S(t,u), add the mass term, mask, online softmax (lazy rescaling: the running
//                   max moves only when a tile exceeds it by more than 2^8), write P(t,u) as bf16
//                   over S(t,u)'s first 32 columns;
//   warps 4NQ..5NQ-1  one MMA-issuing thread per query tile t: S(t,u+1) = Q_t K^T while the
//                   softmax of unit u runs, then O_t += P(t,u) V (P from tensor memory, V an
//                   MN-major shared-memory operand).  Each tile's chain waits only on its own
//                   softmax, so a slow step of one tile does not hold back the other's products
//                   (the tensor core takes both issuers' instructions); a K/V stage is free once
//                   both issuers have released it (after their PV, or at once for a unit past a
//                   tile's causal range);
//   next 3 warps    loaders of the 64-slot K/V tiles (TMA for full tiles, cp.async for partial
//                   ones; 128-byte swizzled canonical layouts, chunk ^ (row & 7)).
// Tensor memory: tile t's S in columns [64t, 64t+64), released as soon as the softmax has loaded it
// (so S(t,u+1) is computed while the softmax of tile u runs); its P double-buffered as bf16 in
// [64NQ + 64t + 32b, +32) (b = u & 1); its O at [128NQ + tD, 128NQ + (t+1)D).  Stages and buffers
// are handed over with
// mbarriers; every wait is bounded, and on expiry a role stops, the CTA records kStatusTimeout,
// frees its tensor memory and returns.
constexpr int kTcRows = 128;
constexpr int kTcTS = 64;
constexpr int kTcLoaders = 96;             // three loader warps
constexpr int32_t kStatusTimeout = 1 << 17;
constexpr long long kTcWaitBudget = 4000000000LL;   // clock cycles (about 2 s)

template <int NQ>
struct TcRoles {
  static constexpr int STAGES = NQ == 1 ? 2 : 4;   // K/V stages in shared memory
  static constexpr int SOFTMAX_WARPS = 4 * NQ;
  static constexpr int MMA_WARP0 = 4 * NQ;         // one issuer warp per query tile
  static constexpr int LOADER_WARP0 = 5 * NQ;
  static constexpr int WARPS = 5 * NQ + 3;
  static constexpr uint32_t COLS = NQ == 1 ? 256u : 512u;
};

template <int D, int NQ>
struct TcShape {
  static constexpr int Q1_BYTES = (D / 64) * kTcRows * 128;     // one query tile
  static constexpr int KV_BYTES = (D / 64) * kTcTS * 128;      // one K or V tile
  static constexpr int OFF_Q = 0;
  static constexpr int ST = TcRoles<NQ>::STAGES;
  static constexpr int OFF_K = OFF_Q + NQ * Q1_BYTES;           // ST stages
  static constexpr int OFF_V = OFF_K + ST * KV_BYTES;           // ST stages
  static constexpr int OFF_M = OFF_V + ST * KV_BYTES;           // ST x 64 raw masses
  static constexpr int BYTES = OFF_M + ST * kTcTS * 4;
  static constexpr size_t smem = (size_t)BYTES + 1024;          // + alignment slack
  static_assert(D == 64 || D == 128, "tcgen05 chunk attention handles head dims 64 and 128");
  static_assert(128 * NQ + NQ * D <= (int)TcRoles<NQ>::COLS, "tensor-memory columns");
};

// K/V tile sources as 2-D tensor maps ([rows of every lane, D] bf16, 64 x 64 boxes, 128-byte
// swizzle): prefix, window and new chunk, K then V.  tma_mask bit c set = full tiles of source
// class c come in by TMA; partial tiles (and classes whose map could not be encoded) by cp.async.
struct TcMaps {
  CUtensorMap k[3];
  CUtensorMap v[3];
};

template <int D, int NQ>
__global__ void __launch_bounds__(TcRoles<NQ>::WARPS * 32, 1)
    chunk_attn_tc_kernel(AttnGeo a, logkv_prefix_t pre, const __nv_bfloat16* rk, const __nv_bfloat16* rv,
                         const __nv_bfloat16* kn, const __nv_bfloat16* vn, const __nv_bfloat16* q,
                         __nv_bfloat16* out, int32_t* status, const __grid_constant__ TcMaps maps,
                         int tma_mask, int nsplit, float* part) {
  using S = TcShape<D, NQ>;
  using RL = TcRoles<NQ>;
  constexpr int CPR = D / 8, TS = kTcTS, ST = RL::STAGES;
  extern __shared__ uint4 smem4[];
  __shared__ uint64_t q_full, kv_full[ST], kv_empty[ST], s_full[NQ][2], p_full[NQ][2], pv_done[NQ][2];
  __shared__ uint32_t sh_tmem;
  __shared__ int sh_abort;
  const int tid = threadIdx.x, warp = tid >> 5;
  unsigned char* raw = reinterpret_cast<unsigned char*>(smem4);
  unsigned char* base = raw + ((1024u - (tc::smem_u32(raw) & 1023u)) & 1023u);
  const uint32_t base_s = tc::smem_u32(base);
  const int g = blockIdx.y, b = blockIdx.z, ln = b * a.G + g;
  const int QT = kTcRows / a.rf;
  // CTA x = split * npairs + pair: split `split` of the key range of query tile pair `pair`.
  const int npairs = (int)gridDim.x / nsplit, pair = (int)blockIdx.x % npairs, split = (int)blockIdx.x / npairs;
  // Query tiles of this CTA.  With two tiles and an even tile count, CTA x takes tiles x and
  // ntiles - 1 - x, so every CTA sees the same number of causal chunk units in total (adjacent
  // tiles would leave the last CTA with the two longest); otherwise tiles NQ x .. NQ x + NQ - 1.
  const int ntiles = (a.TQ + QT - 1) / QT;
  const bool mirror = NQ == 2 && (ntiles & 1) == 0;
  auto tq_of = [&](int t) {
    const int tile = mirror ? (t == 0 ? pair : ntiles - 1 - pair) : pair * NQ + t;
    return a.qoff + tile * QT;
  };
  const __nv_bfloat16* PK = static_cast<const __nv_bfloat16*>(pre.k);
  const __nv_bfloat16* PV = static_cast<const __nv_bfloat16*>(pre.v);
  const int Lp = min(max(pre.length[ln], 0), pre.capacity), R = a.rcount;
  const int up = (Lp + TS - 1) / TS, ur = (R + TS - 1) / TS;
  // Units (64-slot K/V tiles) each query tile attends to: prefix, window, then the new tokens up
  // to its last token (causal); the CTA streams the longest tile's units.
  int Ut[NQ];
  int tlast = 0;
#pragma unroll
  for (int t = 0; t < NQ; ++t) {
    const int last = min(a.qoff + a.TQ, tq_of(t) + QT) - 1;
    tlast = t ? max(tlast, last) : last;
    const int tv = a.causal ? min(a.T, last + 1) : a.T;
    Ut[t] = up + ur + (tv + TS - 1) / TS;
  }
  const int Tvis = a.causal ? min(a.T, tlast + 1) : a.T;
  const int uc = (Tvis + TS - 1) / TS;
  // This split's units [ub, U) of the CTA's range; a tile's own units end at min(Ut[t], U).
  const int Uall = up + ur + uc;
  const int ub = (int)((long long)Uall * split / nsplit), U = (int)((long long)Uall * (split + 1) / nsplit);
#pragma unroll
  for (int t = 0; t < NQ; ++t) Ut[t] = max(min(Ut[t], U), ub);

  if (tid == 0) {
    tc::mbar_init(&q_full, 2 * kTcLoaders);
    for (int i = 0; i < ST; ++i) {
      tc::mbar_init(&kv_full[i], 2 * kTcLoaders + 1);   // + the TMA issuer's (expect-tx) arrival
      tc::mbar_init(&kv_empty[i], NQ);   // one release per query tile's issuer
    }
    for (int t = 0; t < NQ; ++t) {
      for (int i = 0; i < 2; ++i) {
        tc::mbar_init(&s_full[t][i], 1);
        tc::mbar_init(&p_full[t][i], kTcRows);
        tc::mbar_init(&pv_done[t][i], 1);
      }
    }
    tc::mbar_fence_init();
    sh_abort = 0;
  }
  if (warp == 0) {
    tc::tmem_alloc(&sh_tmem, RL::COLS);
    tc::tmem_relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = sh_tmem;
  // Per query tile: two 64-column S buffers (unit r's scores in buffer r & 1, then its P as bf16
  // pairs over the buffer's first 32 columns) and O.  QK^T of unit r + 1 overlaps the softmax's
  // read of unit r's scores.
  auto t_s = [&](int t, int buf) { return tmem + 128u * t + 64u * buf; };
  auto t_o = [&](int t) { return tmem + 128u * NQ + (uint32_t)(t * D); };
  auto unit_info = [&](int u, const __nv_bfloat16*& kb, const __nv_bfloat16*& vb, const float*& mb, int& rows,
                       int& cls, int& first) {
    if (u < up) {
      first = u * TS;
      rows = min(TS, Lp - first);
      const size_t r = (size_t)ln * pre.capacity + first;
      kb = PK + r * D;
      vb = PV + r * D;
      mb = pre.mass + r;
      cls = 0;
    } else if (u < up + ur) {
      first = (u - up) * TS;
      rows = min(TS, R - first);
      const size_t r = (size_t)ln * a.rcap + first;
      kb = rk + r * D;
      vb = rv + r * D;
      mb = nullptr;
      cls = 1;
    } else {
      first = (u - up - ur) * TS;
      rows = min(TS, Tvis - first);
      const size_t r = (size_t)ln * a.T + first;
      kb = kn + r * D;
      vb = vn + r * D;
      mb = nullptr;
      cls = 2;
    }
  };
  auto fail = [&]() {
    sh_abort = 1;
    if (status) atomicOr(status, kStatusTimeout);
  };

  if (warp >= RL::LOADER_WARP0) {
    // ------------------------------------------------ loaders
    const int lt = tid - RL::LOADER_WARP0 * 32;
    const float mscale_l = a.qx * a.scale_log2;
    for (int flat = lt; flat < NQ * kTcRows * CPR; flat += kTcLoaders) {
      const int mq = flat / CPR, c = flat % CPR;
      const int t = mq / kTcRows, m = mq % kTcRows;
      const int tok = tq_of(t) + m % QT, h = g * a.rf + m / QT;
      unsigned char* dst = base + S::OFF_Q + t * S::Q1_BYTES + (c >> 3) * (kTcRows * 128) + m * 128 +
                           (((c & 7) ^ (m & 7)) << 4);
      if (tok < a.qoff + a.TQ) cp_async16(dst, q + (((size_t)b * a.H + h) * a.QS + tok) * D + c * 8);
      else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    tc::mbar_arrive_cp_async(&q_full);
    tc::mbar_arrive(&q_full);
    for (int u = ub; u < U; ++u) {
      const int r = u - ub, st = r % ST;
      if (r >= ST && !tc::mbar_wait(&kv_empty[st], ((r - ST) / ST) & 1, kTcWaitBudget)) {
        fail();
        break;
      }
      const __nv_bfloat16 *kb, *vb;
      const float* mb;
      int rows, cls, first;
      unit_info(u, kb, vb, mb, rows, cls, first);
      unsigned char* sk = base + S::OFF_K + st * S::KV_BYTES;
      unsigned char* sv = base + S::OFF_V + st * S::KV_BYTES;
      float* sm = reinterpret_cast<float*>(base + S::OFF_M) + st * TS;
      const bool by_tma = rows == TS && ((tma_mask >> cls) & 1);
      if (by_tma) {
        // One thread: 2 x (D/64) boxes of 64 rows x 128 bytes, already in the swizzled layout.
        if (lt == 0) {
          const int row0 = cls == 0 ? ln * pre.capacity + first : (cls == 1 ? ln * a.rcap + first : ln * a.T + first);
          tc::fence_proxy_async();   // earlier plain zero stores to this stage before the async writes
          tc::mbar_arrive_expect_tx(&kv_full[st], 2 * S::KV_BYTES);
#pragma unroll
          for (int c64 = 0; c64 < D / 64; ++c64) {
            tc::tma_load_2d(tc::smem_u32(sk) + c64 * (TS * 128), &maps.k[cls], c64 * 64, row0, &kv_full[st]);
            tc::tma_load_2d(tc::smem_u32(sv) + c64 * (TS * 128), &maps.v[cls], c64 * 64, row0, &kv_full[st]);
          }
        }
      } else {
        for (int flat = lt; flat < TS * CPR; flat += kTcLoaders) {
          const int r = flat / CPR, c = flat % CPR;
          const int off = (c >> 3) * (TS * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4);
          if (r < rows) {
            cp_async16(sk + off, kb + (size_t)flat * 8);
            cp_async16(sv + off, vb + (size_t)flat * 8);
          } else {
            *reinterpret_cast<uint4*>(sk + off) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(sv + off) = make_uint4(0, 0, 0, 0);
          }
        }
        if (lt == 0) tc::mbar_arrive(&kv_full[st]);   // the issuer's arrival without a TMA
      }
      if (lt < TS) sm[lt] = cls == 0 && lt < rows ? mscale_l * mb[lt] : 0.f;   // log2-scaled mass term
      tc::mbar_arrive_cp_async(&kv_full[st]);   // when this thread's copies land
      tc::mbar_arrive(&kv_full[st]);            // releases its plain zero stores
    }
  } else if (warp >= RL::MMA_WARP0) {
    // ------------------------------------------------ MMA issuer of query tile t
    const int t = warp - RL::MMA_WARP0;
    if ((tid & 31) == 0) {
      constexpr uint32_t idesc_s = tc::f16_idesc(kTcRows, TS, 0, 0);
      constexpr uint32_t idesc_o = tc::f16_idesc(kTcRows, D, 0, 1);
      const int Uq = Ut[t];
      const uint32_t qa = base_s + S::OFF_Q + t * S::Q1_BYTES;
      bool ok = tc::mbar_wait(&q_full, 0, kTcWaitBudget);
      for (int u = ub; ok && u <= U; ++u) {
        const int r = u - ub;
        if (u < U) {
          // Every unit's arrival is awaited (also past this tile's range) so that this issuer's
          // releases of a stage stay in the stage's phase order.
          const int st = r % ST;
          ok = tc::mbar_wait(&kv_full[st], (r / ST) & 1, kTcWaitBudget);
          if (!ok) break;
          if (u < Uq) {
            tc::fence_proxy_async();
            tc::fence_after();
            // S buffer r & 1 is free once PV of unit r - 2 has read its P (the softmax loaded
            // that unit's scores before writing the P).
            if (r >= 2 && !tc::mbar_wait(&pv_done[t][r & 1], ((r - 2) >> 1) & 1, kTcWaitBudget)) {
              ok = false;
              break;
            }
            tc::fence_after();
            const uint32_t kbs = base_s + S::OFF_K + st * S::KV_BYTES;
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
              const uint64_t da = tc::sw128_desc(qa + (ks >> 2) * (kTcRows * 128) + (ks & 3) * 32, 16, 1024);
              const uint64_t db = tc::sw128_desc(kbs + (ks >> 2) * (TS * 128) + (ks & 3) * 32, 16, 1024);
              tc::umma_f16(t_s(t, r & 1), da, db, idesc_s, ks > 0 ? 1u : 0u);
            }
            tc::umma_commit(&s_full[t][r & 1]);
          }
        }
        if (r >= 1) {
          const int v = u - 1, rv_ = r - 1, bp = rv_ & 1, vs = rv_ % ST;
          if (v < Uq) {
            ok = tc::mbar_wait(&p_full[t][bp], (rv_ >> 1) & 1, kTcWaitBudget);
            if (!ok) break;
            tc::fence_after();
            const uint32_t vbs = base_s + S::OFF_V + vs * S::KV_BYTES;
#pragma unroll
            for (int ks = 0; ks < TS / 16; ++ks) {
              const uint64_t db = tc::sw128_desc(vbs + ks * 16 * 128, TS * 128, 1024);
              tc::umma_f16_ts(t_o(t), t_s(t, bp) + ks * 8, db, idesc_o, (rv_ > 0 || ks > 0) ? 1u : 0u);
            }
            tc::umma_commit(&pv_done[t][bp]);
            tc::umma_commit(&kv_empty[vs]);
          } else {
            tc::mbar_arrive(&kv_empty[vs]);   // unit v lies past this tile's causal range
          }
        }
      }
      if (!ok) fail();
    }
  } else {
    // ------------------------------------------------ softmax (query tile qt, row tid % 128)
    const int qt = warp >> 2;
    const int row = tid - qt * kTcRows;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int row_t = tq_of(qt) + (row % QT);
    const int Uq = Ut[qt], nq_ = Uq - ub;   // this tile's units of the split: [ub, Uq)
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int u = ub; u < Uq; ++u) {
      const int r = u - ub, st = r & 1, ks_ = r % ST;
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&kv_full[ks_], (r / ST) & 1, kTcWaitBudget) &&
                                       tc::mbar_wait(&s_full[qt][st], (r >> 1) & 1, kTcWaitBudget));
      if (!ok) break;
      tc::fence_after();
      const __nv_bfloat16 *kb_, *vb_;
      const float* mb_;
      int rows, cls, first;
      unit_info(u, kb_, vb_, mb_, rows, cls, first);
      const float* sm = reinterpret_cast<const float*>(base + S::OFF_M) + ks_ * TS;
      float sv[TS];
      {
        uint32_t r64[64];
        tc::tmem_ld64(t_s(qt, st) + lane_off, r64);
#pragma unroll
        for (int j = 0; j < TS; ++j) sv[j] = __uint_as_float(r64[j]);
      }
      float mt = -INFINITY;
      const bool full = rows == TS && (cls != 2 || !a.causal || first + TS - 1 <= row_t);
      if (full) {
        const uint64_t c2 = tc::f2pack(a.scale_log2, a.scale_log2);
#pragma unroll
        for (int j = 0; j < TS; j += 4) {
          const float4 m4 = *reinterpret_cast<const float4*>(sm + j);   // masses arrive log2-scaled
          tc::f2unpack(tc::ffma2(tc::f2pack(sv[j], sv[j + 1]), c2, tc::f2pack(m4.x, m4.y)), sv[j], sv[j + 1]);
          tc::f2unpack(tc::ffma2(tc::f2pack(sv[j + 2], sv[j + 3]), c2, tc::f2pack(m4.z, m4.w)), sv[j + 2], sv[j + 3]);
          mt = fmaxf(mt, fmaxf(fmaxf(sv[j], sv[j + 1]), fmaxf(sv[j + 2], sv[j + 3])));
        }
      } else {
#pragma unroll
        for (int j = 0; j < TS; ++j) {
          const bool vis = j < rows && (cls != 2 || !a.causal || first + j <= row_t);
          sv[j] = vis ? fmaf(sv[j], a.scale_log2, sm[j]) : -INFINITY;
          mt = fmaxf(mt, sv[j]);
        }
      }
      float alpha = 1.f;
      if (mt > m_used + 8.f || (m_used == -INFINITY && mt != -INFINITY)) {
        alpha = m_used == -INFINITY ? 0.f : tc::ex2(m_used - mt);
        m_used = mt;
      }
      const float msub = m_used == -INFINITY ? 0.f : m_used;
      const uint64_t nm2 = tc::f2pack(-msub, -msub);
      uint64_t ps2 = tc::f2pack(0.f, 0.f);
      uint32_t pk[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float x0, x1;
        tc::f2unpack(tc::fadd2(tc::f2pack(sv[2 * j], sv[2 * j + 1]), nm2), x0, x1);
        const float p0 = tc::ex2(x0), p1 = tc::ex2(x1);
        ps2 = tc::fadd2(ps2, tc::f2pack(p0, p1));
        pk[j] = pack_bf16x2(p0, p1);
      }
      float ps0, ps1;
      tc::f2unpack(ps2, ps0, ps1);
      const float ps = ps0 + ps1;
      l = l * alpha + ps;
      if (r > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // O must hold PV(u-1) before it is rescaled.
        ok = __all_sync(0xffffffffu,
                        tc::mbar_wait(&pv_done[qt][(r - 1) & 1], ((r - 1) >> 1) & 1, kTcWaitBudget));
        if (!ok) break;
        tc::fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t r32[32];
          tc::tmem_ld32(t_o(qt) + lane_off + c0, r32);
#pragma unroll
          for (int j = 0; j < 32; ++j) r32[j] = __float_as_uint(__uint_as_float(r32[j]) * alpha);
          tc::tmem_st32(t_o(qt) + lane_off + c0, r32);
        }
      }
      tc::tmem_st32(t_s(qt, st) + lane_off, pk);   // P over this unit's own (loaded) scores
      tc::fence_before();
      tc::mbar_arrive(&p_full[qt][st]);
    }
    if (ok && nq_ > 0)
      ok = __all_sync(0xffffffffu,
                      tc::mbar_wait(&pv_done[qt][(nq_ - 1) & 1], ((nq_ - 1) >> 1) & 1, kTcWaitBudget));
    if (!ok) {
      if ((tid & 31) == 0) fail();
    } else if (nsplit > 1) {
      // Split partial [m, l, -, -, O[D]] of this row (O unnormalised, relative to 2^m; a tile
      // without units in this split writes m = -inf, l = 0, O = 0) for chunk_combine_kernel.
      // The tensor-memory loads are warp-wide: every lane issues them, rows past the chunk (a
      // partial last tile) only skip the stores.
      tc::fence_after();
      const int hh = row / QT;
      const bool in = row_t < a.qoff + a.TQ;
      const size_t prow = ((size_t)b * a.H + g * a.rf + hh) * a.TQ + (in ? row_t - a.qoff : 0);
      float* pp = part + ((size_t)split * a.B * a.H * a.TQ + prow) * (D + 4);
      if (in) {
        pp[0] = m_used;
        pp[1] = l;
      }
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t r32[32];
        if (nq_ > 0) {   // uniform over the warpgroup (one query tile)
          tc::tmem_ld32(t_o(qt) + lane_off + c0, r32);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r32[j] = 0u;
        }
        if (in) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(pp + 4 + c0 + j) =
                make_float4(__uint_as_float(r32[j]), __uint_as_float(r32[j + 1]), __uint_as_float(r32[j + 2]),
                            __uint_as_float(r32[j + 3]));
        }
      }
    } else if (nq_ > 0) {
      tc::fence_after();
      const int hh = row / QT;
      const bool in = row_t < a.qoff + a.TQ;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = out + (((size_t)b * a.H + g * a.rf + hh) * a.QS + row_t) * D;
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t r32[32];
        tc::tmem_ld32(t_o(qt) + lane_off + c0, r32);
        if (in) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(r32[j]) * inv, __uint_as_float(r32[j + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(r32[j + 2]) * inv, __uint_as_float(r32[j + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(r32[j + 4]) * inv, __uint_as_float(r32[j + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(r32[j + 6]) * inv, __uint_as_float(r32[j + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c0 + j) = w;
          }
        }
      }
    }
  }
  cp_async_wait<0>();
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, RL::COLS);
  }
}

// ---------------------------------------------------------------- host side
static bool dtype_ok(int d) { return d == LOGKV_DTYPE_F32 || d == LOGKV_DTYPE_BF16; }
static size_t esize_of(int d) { return d == LOGKV_DTYPE_F32 ? 4 : 2; }

static int check_layout(const logkv_layout_t* l) {
  if (!l) return LOGKV_E_POINTER;
  if (!dtype_ok(l->dtype)) return LOGKV_E_DTYPE;
  if (l->batch < 1 || l->groups < 1 || l->dim < 1 || l->clusters < 1 || l->clusters > kMaxClusters ||
      l->levels < 1 || l->levels > kMaxLevels || l->slots < 1 || l->exact < 0)
    return LOGKV_E_SHAPE;
  if ((l->dim * esize_of(l->dtype)) % 16 != 0) return LOGKV_E_SHAPE;
  return LOGKV_OK;
}

static int check_rope(const logkv_rope_t* r, int D) {
  if (!r) return LOGKV_E_POINTER;
  if (!dtype_ok(r->dtype)) return LOGKV_E_DTYPE;
  if (r->rope_n < 0 || r->rope_n > D || (r->rope_n & 1)) return LOGKV_E_SHAPE;
  if (r->rope_n > 0 && (!r->cos || !r->sin || r->rows < 1)) return LOGKV_E_POINTER;
  return LOGKV_OK;
}

static int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LOGKV_OK : (int)e;
}

template <typename T>
static void launch_prefix_pack(const PlanGeo& pg, const logkv_state_t& s, const logkv_plan_t& p,
                               const logkv_rope_t& rope, const logkv_prefix_t& pre, int32_t* status,
                               cudaStream_t st) {
  RopeArgs ra{rope.cos, rope.sin, rope.rows, rope.rope_n};
  const int rows = pg.cap + pg.P;
  const int blocks = std::max(1, std::min(64, (rows + 63) / 64));
  const dim3 grid(blocks, pg.G, pg.B);
  if (rope.dtype == LOGKV_DTYPE_BF16)
    prefix_pack_kernel<T, __nv_bfloat16><<<grid, 256, 0, st>>>(pg, s, p, ra, pre, status);
  else
    prefix_pack_kernel<T, float><<<grid, 256, 0, st>>>(pg, s, p, ra, pre, status);
}

template <typename T>
static void launch_pack_mid(const PlanGeo& pg, const logkv_state_t& s, const logkv_plan_t& p,
                            const logkv_rope_t& rope, const PackArgs& a, const void* kn, const void* vn, void* ok,
                            void* ov, int32_t* status, cudaStream_t st) {
  RopeArgs ra{rope.cos, rope.sin, rope.rows, rope.rope_n};
  const int length = a.width + a.alpha_count + a.recent_count + a.tokens;
  const int blocks = std::max(1, std::min(64, (length + 63) / 64));
  const dim3 grid(blocks, pg.G, pg.B);
  if (rope.dtype == LOGKV_DTYPE_BF16)
    pack_mid_kernel<T, __nv_bfloat16><<<grid, 256, 0, st>>>(pg, s, p, ra, a, static_cast<const T*>(kn),
                                                            static_cast<const T*>(vn), static_cast<T*>(ok),
                                                            static_cast<T*>(ov), status);
  else
    pack_mid_kernel<T, float><<<grid, 256, 0, st>>>(pg, s, p, ra, a, static_cast<const T*>(kn),
                                                    static_cast<const T*>(vn), static_cast<T*>(ok),
                                                    static_cast<T*>(ov), status);
}

// Splits per lane of the grid: attn_units_per_split 16-row tiles each at full prefix capacity, and
// at least one CTA per SM over all lanes (attn_min_splits).  The tensor-core kernel sizes each
// lane's splits again from its actual lengths (slot_attn_mma_kernel), at most this many.
static int attn_min_splits(const logkv_layout_t& l) {
  const int lanes = l.batch * l.groups;
  return std::max(1, std::min((148 + lanes - 1) / lanes, 256));
}

static int attn_splits(const logkv_layout_t& l, int prefix_capacity) {
  const int units = (prefix_capacity + l.recent_capacity) / 16 + 1;
  const int ups = attn_units_per_split(l.batch * l.groups);
  return std::max(1, std::min(std::max(units / ups, attn_min_splits(l)), 256));
}

static size_t attn_part_bytes(const logkv_layout_t& l, int nq, int nsplit) {
  return (size_t)l.batch * l.groups * nsplit * nq * (l.dim + 2) * sizeof(float);
}

template <typename T, int D, int NQ>
static int launch_attn_dq(const AttnGeo& ag, const logkv_prefix_t& pre, const logkv_state_t& s,
                          const logkv_attention_args_t& x, float* part, int* ticket, cudaStream_t st) {
  using S = AttnShape<T, D, NQ>;
  if (S::smem > 227 * 1024) return LOGKV_E_SMEM;
  auto kern = slot_attn_kernel<T, D, NQ>;
  if (S::smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::smem);
  kern<<<dim3(ag.nsplit, ag.G, ag.B), kAttnWarps * 32, S::smem, st>>>(
      ag, pre, static_cast<const T*>(s.recent_k), static_cast<const T*>(s.recent_v), static_cast<const T*>(x.k_new),
      static_cast<const T*>(x.v_new), static_cast<const T*>(x.q), static_cast<T*>(x.out), part, ticket);
  return launch_status();
}

template <typename T, int D>
static int launch_attn_d(int nq, const AttnGeo& ag, const logkv_prefix_t& pre, const logkv_state_t& s,
                         const logkv_attention_args_t& x, float* part, int* ticket, cudaStream_t st) {
  switch (nq) {
    case 1: return launch_attn_dq<T, D, 1>(ag, pre, s, x, part, ticket, st);
    case 2: return launch_attn_dq<T, D, 2>(ag, pre, s, x, part, ticket, st);
    case 4: return launch_attn_dq<T, D, 4>(ag, pre, s, x, part, ticket, st);
    case 8: return launch_attn_dq<T, D, 8>(ag, pre, s, x, part, ticket, st);
    default: return LOGKV_E_SHAPE;
  }
}

template <int D, int NQ>
static int launch_mma_dq(const AttnGeo& ag, const logkv_prefix_t& pre, const logkv_state_t& s,
                         const logkv_attention_args_t& x, float* part, int* ticket, cudaStream_t st) {
  auto go = [&](auto stages) {
    constexpr int ST = decltype(stages)::value;
    using S = MmaShape<D, ST>;
    if (S::smem > 227 * 1024) return (int)LOGKV_E_SMEM;
    auto kern = slot_attn_mma_kernel<D, NQ, ST>;
    if (S::smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::smem);
    using B16 = __nv_bfloat16;
    // Lanes along x, splits along y: a lane's unused splits are the last CTAs dispatched.
    kern<<<dim3(ag.G * ag.B, ag.nsplit), kAttnWarps * 32, S::smem, st>>>(
        ag, pre, static_cast<const B16*>(s.recent_k), static_cast<const B16*>(s.recent_v),
        static_cast<const B16*>(x.k_new), static_cast<const B16*>(x.v_new), static_cast<const B16*>(x.q),
        static_cast<B16*>(x.out), part, ticket);
    return launch_status();
  };
  if (attn_stages(ag.G * ag.B) == 3) return go(std::integral_constant<int, 3>{});
  return go(std::integral_constant<int, 2>{});
}

template <int D>
static int launch_mma_d(int nq, const AttnGeo& ag, const logkv_prefix_t& pre, const logkv_state_t& s,
                        const logkv_attention_args_t& x, float* part, int* ticket, cudaStream_t st) {
  switch (nq) {
    case 1: return launch_mma_dq<D, 1>(ag, pre, s, x, part, ticket, st);
    case 2: return launch_mma_dq<D, 2>(ag, pre, s, x, part, ticket, st);
    case 4: return launch_mma_dq<D, 4>(ag, pre, s, x, part, ticket, st);
    case 8: return launch_mma_dq<D, 8>(ag, pre, s, x, part, ticket, st);
    case 16: return launch_mma_dq<D, 16>(ag, pre, s, x, part, ticket, st);
    default: return LOGKV_E_SHAPE;
  }
}

// Chunk kernel: bf16, more than 16 query rows per lane, 16 <= D <= 128, rf a power of two <= 8.
static bool use_chunk_kernel(const logkv_layout_t& l, int heads, int q_tokens) {
  const int rf = heads / l.groups;
  return l.dtype == LOGKV_DTYPE_BF16 && rf * q_tokens > 16 && l.dim % 16 == 0 && l.dim <= 128 &&
         (rf == 1 || rf == 2 || rf == 4 || rf == 8);
}


template <int D>
static int launch_chunk_d(const AttnGeo& ag, const logkv_prefix_t& pre, const logkv_state_t& s,
                          const logkv_attention_args_t& x, cudaStream_t st) {
  using S = PfShape<D>;
  auto kern = chunk_attn_mma_kernel<D>;
  if (S::smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::smem);
  const int QT = kPfRows / ag.rf;
  using B16 = __nv_bfloat16;
  kern<<<dim3((ag.TQ + QT - 1) / QT, ag.G, ag.B), kPfWarps * 32, S::smem, st>>>(
      ag, pre, static_cast<const B16*>(s.recent_k), static_cast<const B16*>(s.recent_v),
      static_cast<const B16*>(x.k_new), static_cast<const B16*>(x.v_new), static_cast<const B16*>(x.q),
      static_cast<B16*>(x.out));
  return launch_status();
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// [rows, D] bf16 rows of D * 2 bytes; 64 x 64-element boxes in the 128-byte swizzle; rows past
// the end read as zeros.  False if the encoder is missing or refuses (e.g. a misaligned base).
static bool encode_rows_map(CUtensorMap* m, const void* base, size_t rows, int D) {
  auto enc = tensor_map_encoder();
  if (!enc || !base || rows == 0 || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kTcTS};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Combine of the chunk kernel's key-range splits: one warp per output row (b, h, token), the
// partials [m, l, -, -, O[D]] weighted by 2^(m_s - max m) in split order.
template <int D>
__global__ void __launch_bounds__(256) chunk_combine_kernel(AttnGeo a, const float* part, int nsplit,
                                                            __nv_bfloat16* out) {
  constexpr int PER = D / 32;
  const int lane = threadIdx.x & 31;
  const size_t rows = (size_t)a.B * a.H * a.TQ;
  const size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const size_t stride = rows * (D + 4);
  const float* p0 = part + row * (D + 4);
  float mx = -INFINITY;
  for (int sp = 0; sp < nsplit; ++sp) mx = fmaxf(mx, p0[sp * stride]);
  float L = 0.f, o[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) o[k] = 0.f;
  for (int sp = 0; sp < nsplit; ++sp) {
    const float* pp = p0 + sp * stride;
    const float m = pp[0];
    const float w = (m == -INFINITY || mx == -INFINITY) ? 0.f : exp2f(m - mx);
    L += pp[1] * w;
#pragma unroll
    for (int k = 0; k < PER; ++k) o[k] += pp[4 + lane + 32 * k] * w;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const size_t bh = row / a.TQ;
  const int t = (int)(row % a.TQ);
  __nv_bfloat16* orow = out + (bh * a.QS + a.qoff + t) * D;
#pragma unroll
  for (int k = 0; k < PER; ++k) orow[lane + 32 * k] = __float2bfloat16_rn(o[k] * inv);
}

// Key-range splits of the chunk kernel: enough CTAs (query tile pairs x splits) to fill the SMs
// when the chunk has few heads (a KV-head-sharded rank's share), at least 16 64-slot units per
// split, at most 8.
static int chunk_tc_nq(int tiles) { return tiles >= 2 ? 2 : 1; }
static int chunk_tc_splits(int B, int G, int tiles, int units) {
  const int ctas = (tiles + chunk_tc_nq(tiles) - 1) / chunk_tc_nq(tiles) * G * B;
  int n = std::max(1, 148 / std::max(1, ctas));
  n = std::min(n, std::max(1, units / 16));
  return std::max(1, std::min(n, 8));
}
static size_t chunk_part_bytes(int B, int H, int TQ, int D, int nsplit) {
  return nsplit > 1 ? (size_t)nsplit * B * H * TQ * (D + 4) * sizeof(float) : 0;
}

template <int D, int NQ>
static int launch_chunk_tc(const AttnGeo& ag, const logkv_prefix_t& pre, const logkv_state_t& s,
                           const logkv_attention_args_t& x, int32_t* status, int nsplit, float* part,
                           cudaStream_t st) {
  using S = TcShape<D, NQ>;
  auto kern = chunk_attn_tc_kernel<D, NQ>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::smem);
  using B16 = __nv_bfloat16;
  const int QT = kTcRows / ag.rf;
  const int tiles = (ag.TQ + QT - 1) / QT;
  const size_t lanes = (size_t)ag.B * ag.G;
  TcMaps maps;
  memset(&maps, 0, sizeof(maps));
  int mask = 0;
  if (encode_rows_map(&maps.k[0], pre.k, lanes * pre.capacity, D) &&
      encode_rows_map(&maps.v[0], pre.v, lanes * pre.capacity, D))
    mask |= 1;
  if (encode_rows_map(&maps.k[1], s.recent_k, lanes * ag.rcap, D) &&
      encode_rows_map(&maps.v[1], s.recent_v, lanes * ag.rcap, D))
    mask |= 2;
  if (encode_rows_map(&maps.k[2], x.k_new, lanes * ag.T, D) && encode_rows_map(&maps.v[2], x.v_new, lanes * ag.T, D))
    mask |= 4;
  kern<<<dim3((tiles + NQ - 1) / NQ * nsplit, ag.G, ag.B), TcRoles<NQ>::WARPS * 32, S::smem, st>>>(
      ag, pre, static_cast<const B16*>(s.recent_k), static_cast<const B16*>(s.recent_v),
      static_cast<const B16*>(x.k_new), static_cast<const B16*>(x.v_new), static_cast<const B16*>(x.q),
      static_cast<B16*>(x.out), status, maps, mask, nsplit, part);
  if (nsplit > 1) {
    const size_t rows = (size_t)ag.B * ag.H * ag.TQ;
    chunk_combine_kernel<D><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(ag, part, nsplit, static_cast<B16*>(x.out));
  }
  return launch_status();
}

// Two query tiles per CTA (a ping-pong pair) whenever there are two; the key range split
// over CTAs when the pairs alone do not fill the SMs (chunk_tc_splits).
template <int D>
static int launch_chunk_tc_auto(const AttnGeo& ag, const logkv_prefix_t& pre, const logkv_state_t& s,
                                const logkv_attention_args_t& x, int32_t* status, int nsplit, float* part,
                                cudaStream_t st) {
  const int QT = kTcRows / ag.rf;
  const int tiles = (ag.TQ + QT - 1) / QT;
  if (chunk_tc_nq(tiles) == 2) return launch_chunk_tc<D, 2>(ag, pre, s, x, status, nsplit, part, st);
  return launch_chunk_tc<D, 1>(ag, pre, s, x, status, nsplit, part, st);
}

// Key-range splits of the tcgen05 chunk kernel for this call shape (1 for the mma.sync one);
// the unit estimate uses the prefix capacity, since the actual length is on the device.
static int chunk_splits_for(const logkv_layout_t& l, int heads, int q_tokens, int prefix_capacity) {
  if (l.dim != 64 && l.dim != 128) return 1;
  const int rf = heads / l.groups, QT = kTcRows / rf;
  const int tiles = (q_tokens + QT - 1) / QT;
  const int units = (prefix_capacity + l.recent_capacity + q_tokens) / kTcTS;
  return chunk_tc_splits(l.batch, l.groups, tiles, units);
}

// Head dims 64 and 128 run on tcgen05 (tensor memory accumulators); 16 and 32 on mma.sync.
static int launch_chunk(int D, const AttnGeo& ag, const logkv_prefix_t& pre, const logkv_state_t& s,
                        const logkv_attention_args_t& x, int32_t* status, int nsplit, float* part,
                        cudaStream_t st) {
  switch (D) {
    case 16: return launch_chunk_d<16>(ag, pre, s, x, st);
    case 32: return launch_chunk_d<32>(ag, pre, s, x, st);
    case 64: return launch_chunk_tc_auto<64>(ag, pre, s, x, status, nsplit, part, st);
    case 128: return launch_chunk_tc_auto<128>(ag, pre, s, x, status, nsplit, part, st);
    default: return LOGKV_E_SHAPE;
  }
}

// bf16: tensor-core kernel; fp32: CUDA-core kernel (keeps float32 products).
static int launch_attn(int dtype, int D, int nq, const AttnGeo& ag, const logkv_prefix_t& pre,
                       const logkv_state_t& s, const logkv_attention_args_t& x, float* part, int* ticket,
                       cudaStream_t st) {
  if (dtype == LOGKV_DTYPE_BF16) {
    switch (D) {
      case 16: return launch_mma_d<16>(nq, ag, pre, s, x, part, ticket, st);
      case 32: return launch_mma_d<32>(nq, ag, pre, s, x, part, ticket, st);
      case 64: return launch_mma_d<64>(nq, ag, pre, s, x, part, ticket, st);
      case 128: return launch_mma_d<128>(nq, ag, pre, s, x, part, ticket, st);
      case 256: return launch_mma_d<256>(nq, ag, pre, s, x, part, ticket, st);
      default: return LOGKV_E_SHAPE;
    }
  }
  switch (D) {
    case 16: return launch_attn_d<float, 16>(nq, ag, pre, s, x, part, ticket, st);
    case 32: return launch_attn_d<float, 32>(nq, ag, pre, s, x, part, ticket, st);
    case 64: return launch_attn_d<float, 64>(nq, ag, pre, s, x, part, ticket, st);
    case 128: return launch_attn_d<float, 128>(nq, ag, pre, s, x, part, ticket, st);
    default: return LOGKV_E_SHAPE;
  }
}

// Dynamic shared memory of the decode kernel launch_attn picks (the last CTA's split combine
// reuses it: 2 * nsplit * nq + nq floats).
static size_t decode_smem(int dtype, int D, int nq, int lanes) {
  auto pick = [&](auto tag) -> size_t {
    using T = decltype(tag);
    switch (nq) {
      case 1: return AttnShapeFor<T, 1>(D);
      case 2: return AttnShapeFor<T, 2>(D);
      case 4: return AttnShapeFor<T, 4>(D);
      case 8: return AttnShapeFor<T, 8>(D);
      default: return 0;
    }
  };
  if (dtype == LOGKV_DTYPE_BF16) {
    const int st = attn_stages(lanes);
    switch (D) {
      case 16: return st == 3 ? MmaShape<16, 3>::smem : MmaShape<16, 2>::smem;
      case 32: return st == 3 ? MmaShape<32, 3>::smem : MmaShape<32, 2>::smem;
      case 64: return st == 3 ? MmaShape<64, 3>::smem : MmaShape<64, 2>::smem;
      case 128: return st == 3 ? MmaShape<128, 3>::smem : MmaShape<128, 2>::smem;
      case 256: return st == 3 ? MmaShape<256, 3>::smem : MmaShape<256, 2>::smem;
      default: return 0;
    }
  }
  return pick(float{});
}

}  // namespace logkv

using namespace logkv;

extern "C" {

LOGKV_API int logkv_attention_plan(const logkv_layout_t* layout, const logkv_state_t* state,
                                   const logkv_plan_t* plan, void* stream) {
  int rc = check_layout(layout);
  if (rc) return rc;
  if (!state || !plan || !plan->vslot || !plan->vanchor || !plan->nvalid || !plan->exact_rows || !plan->nexact)
    return LOGKV_E_POINTER;
  if (plan->idx && (!plan->anchor || !plan->valid)) return LOGKV_E_POINTER;
  const PlanGeo pg = make_plan_geo(*layout);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (plan->width_max) cudaMemsetAsync(plan->width_max, 0, sizeof(int32_t), st);
  attn_plan_kernel<<<dim3(pg.G, pg.B), 512, 0, st>>>(pg, *state, *plan);
  return launch_status();
}

LOGKV_API int logkv_pack_prefix(const logkv_layout_t* layout, const logkv_state_t* state,
                                const logkv_plan_t* plan, const logkv_rope_t* rope,
                                const logkv_prefix_t* prefix, int32_t* status, void* stream) {
  int rc = check_layout(layout);
  if (rc) return rc;
  if (!state || !plan || !prefix || !prefix->k || !prefix->v || !prefix->mass || !prefix->length)
    return LOGKV_E_POINTER;
  if ((rc = check_rope(rope, layout->dim))) return rc;
  const PlanGeo pg = make_plan_geo(*layout);
  if (prefix->capacity < pg.cap + pg.P) return LOGKV_E_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (layout->dtype == LOGKV_DTYPE_BF16)
    launch_prefix_pack<__nv_bfloat16>(pg, *state, *plan, *rope, *prefix, status, st);
  else
    launch_prefix_pack<float>(pg, *state, *plan, *rope, *prefix, status, st);
  return launch_status();
}

LOGKV_API int logkv_pack_mid(const logkv_layout_t* layout, const logkv_state_t* state, const logkv_plan_t* plan,
                             const logkv_rope_t* rope, int32_t width, int32_t alpha_count, int32_t recent_count,
                             const void* k_new, const void* v_new, int32_t tokens, void* out_k, void* out_v,
                             int32_t dim, int32_t skip_pooled, int32_t recent_start, int32_t* status, void* stream) {
  int rc = check_layout(layout);
  if (rc) return rc;
  if (!state || !plan || !plan->idx || !plan->anchor || !plan->valid || !out_k || !out_v) return LOGKV_E_POINTER;
  if (tokens > 0 && (!k_new || !v_new)) return LOGKV_E_POINTER;
  if ((rc = check_rope(rope, layout->dim))) return rc;
  const PlanGeo pg = make_plan_geo(*layout);
  if (dim < layout->dim + 1 || width < 0 || width > pg.cap || alpha_count < 0 || alpha_count > pg.P ||
      recent_count < 0 || recent_count > layout->recent_capacity || tokens < 0 || recent_start < 0 ||
      recent_start > recent_count)
    return LOGKV_E_SHAPE;
  PackArgs a{width, alpha_count, recent_count, tokens, dim, skip_pooled, recent_start, layout->recent_capacity};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (layout->dtype == LOGKV_DTYPE_BF16)
    launch_pack_mid<__nv_bfloat16>(pg, *state, *plan, *rope, a, k_new, v_new, out_k, out_v, status, st);
  else
    launch_pack_mid<float>(pg, *state, *plan, *rope, a, k_new, v_new, out_k, out_v, status, st);
  return launch_status();
}

LOGKV_API size_t logkv_attention_workspace_bytes(const logkv_layout_t* layout, int32_t heads, int32_t q_tokens,
                                                 int32_t prefix_capacity) {
  if (check_layout(layout) || heads < layout->groups || heads % layout->groups || q_tokens < 1) return 0;
  if (use_chunk_kernel(*layout, heads, q_tokens))
    return 256 + chunk_part_bytes(layout->batch, heads, q_tokens, layout->dim,
                                  chunk_splits_for(*layout, heads, q_tokens, prefix_capacity));
  const int nq = heads / layout->groups * q_tokens;
  const int nsplit = attn_splits(*layout, prefix_capacity);
  const size_t lanes = (size_t)layout->batch * layout->groups;
  return 256 + ((lanes * sizeof(int) + 255) / 256) * 256 + attn_part_bytes(*layout, nq, nsplit);
}

LOGKV_API int logkv_attention(const logkv_layout_t* layout, const logkv_state_t* state,
                              const logkv_prefix_t* prefix, const logkv_attention_args_t* args,
                              void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_layout(layout);
  if (rc) return rc;
  if (!state || !prefix || !args || !args->q || !args->out || !prefix->length) return LOGKV_E_POINTER;
  const int G = layout->groups, H = args->heads, T = args->tokens, TQ = args->q_tokens;
  const int QS = args->q_stride ? args->q_stride : T;
  if (H < G || H % G || T < 1 || TQ < 1 || args->q_offset < 0 || args->q_offset + TQ > T ||
      args->q_offset + TQ > QS || QS > T || (QS != T && args->causal) || args->recent_count < 0 ||
      args->recent_count > layout->recent_capacity)
    return LOGKV_E_SHAPE;
  if (!args->k_new || !args->v_new) return LOGKV_E_POINTER;
  const int nq = H / G * TQ;
  const size_t need = logkv_attention_workspace_bytes(layout, H, TQ, prefix->capacity);
  if (!workspace || workspace_bytes < need) return LOGKV_E_WORKSPACE;
  // Splits: attn_splits, at most as many as the last CTA's combine can weigh in shared memory.
  const size_t dsm = decode_smem(layout->dtype, layout->dim, nq, layout->batch * G);
  const int ncap = dsm > (size_t)(4 * nq) ? (int)((dsm - 4 * (size_t)nq) / (8 * (size_t)nq)) : 1;
  const int nsplit = std::max(1, std::min(attn_splits(*layout, prefix->capacity), ncap));
  const size_t lanes = (size_t)layout->batch * G;
  int* ticket = reinterpret_cast<int*>(static_cast<char*>(workspace) + 256);
  float* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256 + ((lanes * sizeof(int) + 255) / 256) * 256);
  AttnGeo ag;
  ag.B = layout->batch;
  ag.G = G;
  ag.H = H;
  ag.T = T;
  ag.QS = QS;
  ag.rf = H / G;
  ag.TQ = TQ;
  ag.qoff = args->q_offset;
  ag.causal = args->causal ? 1 : 0;
  ag.nsplit = nsplit;
  ag.nsmin = std::min(attn_min_splits(*layout), nsplit);
  ag.ups = attn_units_per_split(layout->batch * G);
  ag.pcap = prefix->capacity;
  ag.rcap = layout->recent_capacity;
  ag.rcount = args->recent_count;
  ag.scale_log2 = args->scale * 1.4426950408889634f;
  ag.qx = args->qx;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_chunk_kernel(*layout, H, TQ)) {
    const int ns = chunk_splits_for(*layout, H, TQ, prefix->capacity);
    float* cpart = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
    return launch_chunk(layout->dim, ag, *prefix, *state, *args, static_cast<int32_t*>(workspace), ns, cpart, st);
  }
  return launch_attn(layout->dtype, layout->dim, nq, ag, *prefix, *state, *args, part, ticket, st);
}

}  // extern "C"
