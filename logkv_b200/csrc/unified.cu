// Unified (Ward / radius) route operators: fused pair distances, mirror, and the incremental
// mutual-nearest Ward rounds.
//
// Replaces the plugin functions of litgpt/log_kv_route_triton.py: pair_distances (:585-607),
// mirror (:546-553) and UnifiedReduce (:610-838), whose semantics are those of the reference's
// Torch reducer _UnifiedReduceTorch (litgpt/log_kv_cache.py:448-638): row minima of packed
// (Ward cost bits << 32 | row ^ col) keys, disjoint mutual pairs, exact radius verification when
// limits are given, a per-lane budget of count - target pairs by increasing cost, Lance-Williams
// row updates and rescans of rows whose partner merged.  Every operation is float32, rounded as
// the reference writes it (this file is compiled without fused multiply-adds); the exact squared
// distance of a candidate pair sums the features left to right.
//
// One CTA per lane runs a whole round; its phases are separated by block barriers, and within a
// phase every merge writes only its own row and column, which no other merge of the round reads.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/logkv_unified.h"

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxSize = 4096;      // rows per lane (the sort runs in shared memory)
constexpr long long kInfKey = 0x7F80000000000000LL;

__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// (cost bits << 32) | key, with -0.0 written as +0.0 (_unified_pack, log_kv_cache.py:431-434).
__device__ __forceinline__ long long pack_key(float cost, long long key) {
  if (cost == 0.f) cost = 0.f;
  return ((long long)__float_as_int(cost) << 32) | key;
}

// Ward cost of joining clusters i and j, +inf when the pair is not allowed
// (_unified_pair_cost, log_kv_cache.py:437-445).
__device__ __forceinline__ float pair_cost(float d2, float mi, float mj, float ri, float rj, const float* limit,
                                           bool valid) {
  const float denom = fmaxf(fadd(mi, mj), 1.f);
  valid = valid && mi > 0.f && mj > 0.f;
  if (limit) {
    const float distance = __fsqrt_rn(d2);
    const float b1 = fadd(ri, fmul(fdiv(mj, denom), distance));
    const float b2 = fadd(rj, fmul(fdiv(mi, denom), distance));
    valid = valid && fmaxf(b1, b2) <= *limit;
  }
  return valid ? fmul(d2, fdiv(fmul(mi, mj), denom)) : __int_as_float(0x7F800000);
}

struct Lane {
  float* dist;       // [M, M]
  float* mu;         // [M, D]
  float* mass;       // [M]
  float* radius;     // [M]
  uint8_t* alive;    // [M]
  long long* packed; // [M]
  const float* limit;
};

__device__ Lane lane_of(const logkv_unified_t& u, int lane) {
  const size_t M = u.size;
  Lane l;
  l.dist = u.dist + lane * M * M;
  l.mu = u.mu + lane * M * (size_t)u.dim;
  l.mass = u.mass + lane * M;
  l.radius = u.radius + lane * M;
  l.alive = u.alive + lane * M;
  l.packed = reinterpret_cast<long long*>(u.packed) + lane * M;
  l.limit = u.limits ? u.limits + lane : nullptr;
  return l;
}

// packed[r] = min over columns of the row's packed keys; one warp per row.
__device__ void scan_rows(const Lane& l, int M, const int* rows, int nrows) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int i = warp; i < nrows; i += nwarps) {
    const int r = rows[i];
    const float* drow = l.dist + (size_t)r * M;
    const float mr = l.mass[r], rr = l.radius[r];
    long long best = 0x7FFFFFFFFFFFFFFFLL;
    for (int c = lane; c < M; c += 32) {
      const float cost = pair_cost(drow[c], mr, l.mass[c], rr, l.radius[c], l.limit, c != r);
      best = min(best, pack_key(cost, (long long)(r ^ c)));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, off));
    if (lane == 0) l.packed[r] = best;
  }
}

__global__ void __launch_bounds__(kThreads) pair_distances_kernel(float* gram, const float* norm, int M) {
  const int lane = blockIdx.z;
  const int i = blockIdx.y * 32 + (threadIdx.x >> 5), j = blockIdx.x * 32 + (threadIdx.x & 31);
  if (i >= M || j >= M || i > j) return;
  float* g = gram + (size_t)lane * M * M;
  const float* n = norm + (size_t)lane * M;
  // (n_i + n_j) - 2 G_ij rounds once after the exact doubling, like the reference's epilogue.
  const float d = fmaxf(fsub(fadd(n[i], n[j]), fmul(2.f, g[(size_t)i * M + j])), 0.f);
  g[(size_t)i * M + j] = d;
  if (i != j) g[(size_t)j * M + i] = d;
}

__global__ void __launch_bounds__(kThreads) mirror_kernel(float* dist, int M) {
  const int lane = blockIdx.z;
  const int i = blockIdx.y * 32 + (threadIdx.x >> 5), j = blockIdx.x * 32 + (threadIdx.x & 31);
  if (i >= M || j >= M || i <= j) return;
  float* d = dist + (size_t)lane * M * M;
  d[(size_t)i * M + j] = d[(size_t)j * M + i];
}

__global__ void __launch_bounds__(kThreads) init_kernel(logkv_unified_t u) {
  extern __shared__ int rows[];
  const int lane = blockIdx.x, M = u.size;
  Lane l = lane_of(u, lane);
  const int count = u.status[u.lanes + lane];
  __shared__ int n;
  if (threadIdx.x == 0) {
    n = 0;
    u.status[lane] = 0;
    u.merges[lane] = 0;
    u.stuck[lane] = 0;
  }
  __syncthreads();
  for (int r = threadIdx.x; r < M; r += blockDim.x) {
    const bool live = r < count;
    l.alive[r] = live;
    l.radius[r] = 0.f;
    l.packed[r] = kInfKey;
    if (live) rows[atomicAdd(&n, 1)] = r;
  }
  __syncthreads();
  scan_rows(l, M, rows, n);
}

// Shared memory of one round: sort keys [S] u64 | best [M] i32 | partner [M] i32 | rows [M] i32 |
// bound, pma, pmb, pdab [M] f32 | flags [M] u8 (1 valid, 2 rejected, 4 keep, 8 merged).
__global__ void __launch_bounds__(kThreads) round_kernel(logkv_unified_t u, int S) {
  extern __shared__ unsigned long long sk[];
  const int lane = blockIdx.x, M = u.size, D = u.dim, tid = threadIdx.x, nt = blockDim.x;
  Lane l = lane_of(u, lane);
  int* best = reinterpret_cast<int*>(sk + S);
  int* partner = best + M;
  int* rows = partner + M;
  float* bound = reinterpret_cast<float*>(rows + M);
  float* pma = bound + M;
  float* pmb = pma + M;
  float* pdab = pmb + M;
  uint8_t* flags = reinterpret_cast<uint8_t*>(pdab + M);
  __shared__ int nprop, nfinite, nok, ndirty;
  __shared__ long long rowmin[kMaxSize / 2];
  if (tid == 0) {
    nprop = 0;
    nfinite = 0;
    ndirty = 0;
  }
  const unsigned inf_bits = 0x7F800000u;
  // ---- candidates: each row's best partner; disjoint mutual pairs
  for (int r = tid; r < M; r += nt) {
    const long long p = l.packed[r];
    int b = (int)(((p & 0xFFFFFFFFLL) ^ (long long)r));
    b = b < 0 ? 0 : (b > M - 1 ? M - 1 : b);
    best[r] = b;
    partner[r] = 0;
    pma[r] = 1.f;
    pmb[r] = 0.f;
    pdab[r] = 0.f;
    bound[r] = 0.f;
  }
  __syncthreads();
  for (int r = tid; r < M; r += nt) {
    const long long p = l.packed[r];
    const float cost = __int_as_float((int)(p >> 32));
    const int b = best[r];
    const bool v = l.alive[r] && r < b && best[b] == r && cost < __int_as_float(0x7F800000);
    flags[r] = v ? 1 : 0;
    if (v) atomicAdd(&nprop, 1);
  }
  __syncthreads();
  // ---- exact verification against the radius limits
  if (l.limit) {
    for (int r = tid; r < M; r += nt) {
      if (!(flags[r] & 1)) continue;
      const int o = best[r];
      const float* xa = l.mu + (size_t)r * D;
      const float* xb = l.mu + (size_t)o * D;
      float exact2 = 0.f;
      for (int d = 0; d < D; ++d) {
        const float df = fsub(xa[d], xb[d]);
        exact2 = fadd(exact2, fmul(df, df));
      }
      const float exact = __fsqrt_rn(exact2);
      const float ma = l.mass[r], mb = l.mass[o];
      const float denom = fmaxf(fadd(ma, mb), 1.f);
      const float verified =
          fmaxf(fadd(l.radius[r], fmul(fdiv(mb, denom), exact)), fadd(l.radius[o], fmul(fdiv(ma, denom), exact)));
      if (verified > *l.limit) {
        l.dist[(size_t)r * M + o] = exact2;
        l.dist[(size_t)o * M + r] = exact2;
        flags[r] = 2;          // rejected, no longer valid
        flags[o] |= 2;
      }
      bound[r] = verified;
    }
  }
  __syncthreads();
  // ---- stable order of the pair costs: bitonic sort of (cost bits << 32 | row)
  for (int i = tid; i < S; i += nt) {
    unsigned long long key = ~0ull;
    if (i < M) {
      const unsigned cb = (flags[i] & 1) ? (unsigned)(l.packed[i] >> 32) : inf_bits;
      key = ((unsigned long long)cb << 32) | (unsigned)i;
      if ((flags[i] & 1) && cb < inf_bits) atomicAdd(&nfinite, 1);
    }
    sk[i] = key;
  }
  __syncthreads();
  for (int k = 2; k <= S; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < S; i += nt) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = sk[i], y = sk[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) {
            sk[i] = y;
            sk[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  // ---- budget: the first min(finite, count - target, M / 2) pairs merge
  const int count = u.status[u.lanes + lane];
  if (tid == 0) {
    int n = min(nfinite, M / 2);
    n = min(n, max(count - u.target, 0));
    nok = n;
  }
  __syncthreads();
  const int n_ok = nok;
  const int trace0 = u.merges[lane];
  for (int m = tid; m < n_ok; m += nt) {
    const int a = (int)(sk[m] & 0xFFFFFFFFull), b = best[a];
    flags[a] |= 4 | 8;
    flags[b] |= 8;
    partner[a] = b;
    pma[a] = l.mass[a];
    pmb[a] = l.mass[b];
    pdab[a] = l.dist[(size_t)a * M + b];
    rowmin[m] = 0x7FFFFFFFFFFFFFFFLL;
    u.trace[((size_t)lane * M + trace0 + m) * 2] = a;
    u.trace[((size_t)lane * M + trace0 + m) * 2 + 1] = b;
  }
  __syncthreads();
  // ---- merged clusters: masses, liveness, radii, centres
  for (int m = tid; m < n_ok; m += nt) {
    const int a = (int)(sk[m] & 0xFFFFFFFFull), b = best[a];
    l.mass[a] = fadd(pma[a], pmb[a]);
    l.mass[b] = 0.f;
    l.alive[b] = 0;
    if (l.limit) l.radius[a] = bound[a];
  }
  for (int item = tid; item < n_ok * D; item += nt) {
    const int m = item / D, d = item % D;
    const int a = (int)(sk[m] & 0xFFFFFFFFull), b = best[a];
    const float ma = pma[a], mb = pmb[a];
    const float total = fadd(ma, mb);
    float* ra = l.mu + (size_t)a * D;
    const float* rb = l.mu + (size_t)b * D;
    ra[d] = fdiv(fadd(fmul(ma, ra[d]), fmul(mb, rb[d])), fmaxf(total, 1.f));
  }
  __syncthreads();
  // ---- Lance-Williams rows: one thread per (merge, column)
  for (size_t item = tid; item < (size_t)n_ok * M; item += nt) {
    const int m = (int)(item / M), c = (int)(item % M);
    const int a = (int)(sk[m] & 0xFFFFFFFFull), b = best[a];
    const float ma = pma[a], mb = pmb[a], dab = pdab[a];
    const float total = fadd(ma, mb);
    const float alpha = fdiv(ma, total), beta = fdiv(mb, total);
    const float shift = fmul(fmul(alpha, beta), dab);
    const float x_aa = l.dist[(size_t)a * M + c], x_ba = l.dist[(size_t)b * M + c];
    float nv = fsub(fadd(fmul(alpha, x_aa), fmul(beta, x_ba)), shift);
    const bool keep_c = flags[c] & 4;
    if (keep_c) {
      // Both clusters merged this round: the lower keep index's order, so both owners agree.
      const int q = partner[c];
      const float x_ab = l.dist[(size_t)a * M + q], x_bb = l.dist[(size_t)b * M + q];
      const float qa = pma[c], qb = pmb[c], qd = pdab[c];
      const float qs = fadd(qa, qb);
      const float qal = fdiv(qa, qs), qbe = fdiv(qb, qs);
      const float qsh = fmul(fmul(qal, qbe), qd);
      float v;
      if (a < c) {
        const float inner = fsub(fadd(fmul(alpha, x_ab), fmul(beta, x_bb)), shift);
        v = fsub(fadd(fmul(qal, nv), fmul(qbe, inner)), qsh);
      } else {
        const float t1 = fsub(fadd(fmul(qal, x_aa), fmul(qbe, x_ab)), qsh);
        const float t2 = fsub(fadd(fmul(qal, x_ba), fmul(qbe, x_bb)), qsh);
        v = fsub(fadd(fmul(alpha, t1), fmul(beta, t2)), shift);
      }
      nv = v;
    }
    nv = fmaxf(nv, 0.f);
    if (c == a) nv = 0.f;
    const bool alive_c = l.alive[c];
    if (alive_c && !keep_c) l.dist[(size_t)c * M + a] = nv;
    if (alive_c) l.dist[(size_t)a * M + c] = nv;
    const float cost = pair_cost(nv, total, l.mass[c], l.radius[a], l.radius[c], l.limit, alive_c && c != a);
    const long long key = pack_key(cost, (long long)(a ^ c));
    const bool valid = cost < __int_as_float(0x7F800000);
    if (valid && !keep_c) atomicMin(&l.packed[c], key);
    atomicMin(&rowmin[m], key);
  }
  __syncthreads();
  for (int m = tid; m < n_ok; m += nt) l.packed[(int)(sk[m] & 0xFFFFFFFFull)] = rowmin[m];
  // ---- rows whose best partner merged (or that were rejected) rescan
  for (int r = tid; r < M; r += nt) {
    const uint8_t f = flags[r];
    if (l.alive[r] && !(f & 4) && ((flags[best[r]] & 8) || (f & 2))) rows[atomicAdd(&ndirty, 1)] = r;
  }
  __syncthreads();
  scan_rows(l, M, rows, ndirty);
  __syncthreads();
  if (tid == 0) {
    const int left = count - n_ok;
    u.status[u.lanes + lane] = left;
    u.merges[lane] = trace0 + n_ok;
    const bool remaining = left > u.target;
    if (remaining && nprop == 0) u.stuck[lane] = 1;
    u.status[lane] = remaining && nprop > 0;
  }
}

int next_pow2(int v) {
  int p = 2;
  while (p < v) p <<= 1;
  return p;
}

size_t round_smem(int M, int S) { return (size_t)S * 8 + (size_t)M * (3 * 4 + 4 * 4 + 1) + 16; }

}  // namespace

extern "C" int logkv_pair_distances(float* gram, const float* norm, int32_t lanes, int32_t size, void* stream) {
  if (!gram || !norm) return LOGKV_UNIFIED_E_POINTER;
  if (lanes < 0 || lanes > 65535 || size < 0 || size > (1 << 20)) return LOGKV_UNIFIED_E_SHAPE;
  if (!lanes || !size) return 0;
  const int t = (size + 31) / 32;
  pair_distances_kernel<<<dim3(t, t, lanes), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(gram, norm, size);
  return (int)cudaGetLastError();
}

extern "C" int logkv_mirror(float* dist, int32_t lanes, int32_t size, void* stream) {
  if (!dist) return LOGKV_UNIFIED_E_POINTER;
  if (lanes < 0 || lanes > 65535 || size < 0 || size > (1 << 20)) return LOGKV_UNIFIED_E_SHAPE;
  if (!lanes || size < 2) return 0;
  const int t = (size + 31) / 32;
  mirror_kernel<<<dim3(t, t, lanes), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(dist, size);
  return (int)cudaGetLastError();
}

static int check_unified(const logkv_unified_t* u) {
  if (!u || !u->dist || !u->mu || !u->mass || !u->status || !u->alive || !u->radius || !u->packed || !u->merges ||
      !u->stuck || !u->trace)
    return LOGKV_UNIFIED_E_POINTER;
  if ((reinterpret_cast<uintptr_t>(u->packed) & 7)) return LOGKV_UNIFIED_E_POINTER;
  if (u->lanes < 1 || u->size < 1 || u->size > kMaxSize || u->dim < 1) return LOGKV_UNIFIED_E_SHAPE;
  return 0;
}

extern "C" int logkv_unified_init(const logkv_unified_t* u, void* stream) {
  const int v = check_unified(u);
  if (v) return v;
  init_kernel<<<u->lanes, kThreads, (size_t)u->size * 4, static_cast<cudaStream_t>(stream)>>>(*u);
  return (int)cudaGetLastError();
}

extern "C" int logkv_unified_step(const logkv_unified_t* u, void* stream) {
  const int v = check_unified(u);
  if (v) return v;
  const int S = next_pow2(u->size);
  const size_t smem = round_smem(u->size, S);
  if (smem > 227 * 1024) return LOGKV_UNIFIED_E_SHAPE;
  if (smem > 48 * 1024) cudaFuncSetAttribute(round_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  round_kernel<<<u->lanes, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(*u, S);
  return (int)cudaGetLastError();
}
