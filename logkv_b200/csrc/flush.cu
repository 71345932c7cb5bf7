// Host side of the device-resident flush: workspace carving, launch sequence
// and the C ABI entry points declared in include/logkv_b200.h.
//
// Launch sequence of one flush (all on the caller's stream, no host sync):
//   K0 snapshot   old exact pool -> workspace
//   K1 cut        candidate spans per batch row
//   K2 score      Alpha / Beta span scores
//   K4 attach     frozen-centroid decisions for every pool / window token (runs beside K2)
//   K3 choose     bounded greedy, keep / archive lists, new span table
//   K5 plan       farthest-point seeds (archive rank order), per-cluster grouping and jobs
//   K6a prepare   centroids, scalars, new / delayed cluster staging
//   K6b cascade   ladder append with pairwise or Beta merges
//   K7 pool       exact pool rewrite
//   K8 window     window shift by the flushed tokens
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "flush_alpha.cuh"
#include "flush_cascade.cuh"
#include "flush_ladder.cuh"
#include "flush_route.cuh"
#include "flush_tape.cuh"
#include "flush_unified.cuh"

namespace logkv {

// Greedy span choice: per candidate density, size, rank, flags; victims in two buffers.
static size_t choose_smem_bytes(const Geo& g) {
  return (size_t)g.NC * (8 + 4 + 4 + 2) + 2 * (size_t)(g.P + 1) * (8 + 4 + 4) + (size_t)(g.P + 1) * (8 + 4) + 16 +
         (size_t)g.NC * (8 + 8 + 4 + 1) + 8;  // swap tests, closed-span order, swap flags
}

// Span scores (per warp: means, token energies, centre distances) and attach decisions
// (centres, 8 or 16 token rows, per-pair scores).
static size_t score_smem_bytes(const Geo& g, size_t esize) {
  return 8 * (size_t)score_warp_floats(g.D, g.K, (int)esize) * sizeof(float);  // 8 warps
}
static size_t attach_smem_bytes(const Geo& g) {
  return (size_t)(g.K + kAttachTokens) * (g.D + 4) * sizeof(float);
}
// Delayed re-insert sort keys, token sources and the staged rows of the centroid sum.
static size_t prep_smem_bytes(const Geo& g, size_t esize) {
  return (size_t)g.sort_cap * sizeof(unsigned long long) + (size_t)((g.NW + 3) & ~3) * sizeof(int) +
         (size_t)kPrepRows * g.D * esize;
}

static size_t cascade_smem(const Geo& g, size_t esize) { return walk_smem(g, esize, kTileRows); }

// Every flush kernel is launched with a programmatic dependency on the previous kernel of the
// stream (each kernel begins with pdl_entry()), so launch latency overlaps the previous tail.
template <typename... KArgs, typename... Args>
static void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, args...);
}

template <typename K>
static void smem_limit(K* kern, size_t smem) {
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

// Cascade launches for one (dtype, Beta, head dim) instantiation; DC = 0 is the runtime-D kernel.
// Parallel: merges of every level at once, every level's survivor moves, then the sequential walk
// of the lanes that need it (disjoint from the others).  Otherwise one sequential walk per lane.
// Parallel: merges of every level at once, then every level's survivor moves (the move kernel
// also runs the sequential walk of the lanes that need it).  Otherwise one sequential walk per lane.
template <typename T, bool BETA, int DC>
static void launch_cascade(const Geo& g, const logkv_state_t& s, const Work& w, size_t smem, bool parallel,
                           cudaStream_t st) {
  if (!parallel) {
    smem_limit(cascade_kernel<T, BETA, DC>, smem);
    launch_pdl(cascade_kernel<T, BETA, DC>, dim3(g.K, g.G, g.B), kCascadeThreads, smem, st, g, s, w);
    return;
  }
  const size_t ms = merge_smem(g.D, sizeof(T)), vs = move_smem(g, sizeof(T));
  smem_limit(cascade_merge_kernel<T, BETA, DC>, ms);
  launch_pdl(cascade_merge_kernel<T, BETA, DC>, dim3(kMergeCtas, g.K, g.B * g.G), kMergeWarps * 32, ms, st, g, s, w);
  smem_limit(cascade_move_kernel<T, BETA, DC>, vs);
  launch_pdl(cascade_move_kernel<T, BETA, DC>, dim3(g.L, g.K, g.B * g.G), kMoveThreads, vs, st, g, s, w);
}

// The parallel cascade needs one level's survivors (at most B' rows) in one CTA's shared memory
// and B * G <= 65535; LOGKV_CASCADE=sequential forces the sequential walk (both paths give the
// same bits; tests run both).
static bool parallel_cascade(const Geo& g, size_t esize) {
  const char* env = getenv("LOGKV_CASCADE");
  if (env && strcmp(env, "sequential") == 0) return false;
  return move_smem(g, esize) <= 227 * 1024 && merge_smem(g.D, esize) <= 227 * 1024 && (size_t)g.B * g.G <= 65535;
}

template <typename T>
static void launch_cascade_all(const Geo& g, const logkv_state_t& s, const Work& w, cudaStream_t st) {
  const size_t smem = cascade_smem(g, sizeof(T));
  const bool par = parallel_cascade(g, sizeof(T));
  if (g.beta) {
    if (g.D == 128) launch_cascade<T, true, 128>(g, s, w, smem, par, st);
    else if (g.D == 64) launch_cascade<T, true, 64>(g, s, w, smem, par, st);
    else launch_cascade<T, true, 0>(g, s, w, smem, par, st);
  } else {
    if (g.D == 128) launch_cascade<T, false, 128>(g, s, w, smem, par, st);
    else if (g.D == 64) launch_cascade<T, false, 64>(g, s, w, smem, par, st);
    else launch_cascade<T, false, 0>(g, s, w, smem, par, st);
  }
}

// Span scores: the block's warps stride over the (candidate, group) pairs of batch row
// blockIdx.y, one pair per warp at a time.
template <typename T, int DC>
__global__ void __launch_bounds__(256) score_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int b = blockIdx.y;
  float* ws = sm + warp * score_warp_floats(g.D, g.K, (int)sizeof(T));
  const int npairs = w.n_cand[b] * g.G;
  for (int p = blockIdx.x * nwarps + warp; p < npairs; p += gridDim.x * nwarps) {
    score_pair<T, DC>(g, s, w, b, p / g.G, p % g.G, lane, ws);
    __syncwarp();
  }
}

template <typename T, int DC>
static void launch_score(const Geo& g, const logkv_state_t& s, const Work& w, size_t smem, int blocks,
                         cudaStream_t st) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(score_kernel<T, DC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_pdl(score_kernel<T, DC>, dim3(blocks, g.B), 256, smem, st, g, s, w);
}

template <typename T, int DC>
static void launch_prepare_d(const Geo& g, const logkv_state_t& s, const Work& w, size_t smem, cudaStream_t st) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(prepare_kernel<T, DC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_pdl(prepare_kernel<T, DC>, dim3(g.K, g.G, g.B), 256, smem, st, g, s, w);
}

template <typename T>
static void launch_prepare(const Geo& g, const logkv_state_t& s, const Work& w, cudaStream_t st) {
  const size_t smem = prep_smem_bytes(g, sizeof(T));
  if (g.D == 128) launch_prepare_d<T, 128>(g, s, w, smem, st);
  else if (g.D == 64) launch_prepare_d<T, 64>(g, s, w, smem, st);
  else launch_prepare_d<T, 0>(g, s, w, smem, st);
}

// Attach decisions run beside the span scores.  They read the snapshot (complete before any
// score block passed its entry wait, which is what let this grid launch) and the frozen
// cluster state, so the entry wait is skipped.  Block (0, 0, 0) waits at its end instead:
// this grid then completes only after the score grid, and the next kernel's entry wait
// covers both, while every other block leaves as soon as its tokens are done.
template <typename T, int DC, int CPL>
__global__ void __launch_bounds__(256) attach_kernel(Geo g, logkv_state_t s, Work w) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  attach_body<T, DC, CPL>(g, s, w, blockIdx.x);
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <typename T, int DC, int CPL>
static void launch_attach_cpl(const Geo& g, const logkv_state_t& s, const Work& w, size_t smem, int grid_x,
                              cudaStream_t st) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(attach_kernel<T, DC, CPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_pdl(attach_kernel<T, DC, CPL>, dim3(grid_x, g.G, g.B), 256, smem, st, g, s, w);
}

// Centres per lane: a token's 4 lanes cover K <= 4 * CPL centres.
template <typename T, int DC>
static void launch_attach(const Geo& g, const logkv_state_t& s, const Work& w, size_t smem, int grid_x,
                          cudaStream_t st) {
  if (g.K <= 12) launch_attach_cpl<T, DC, 3>(g, s, w, smem, grid_x, st);
  else if (g.K <= 16) launch_attach_cpl<T, DC, 4>(g, s, w, smem, grid_x, st);
  else launch_attach_cpl<T, DC, 8>(g, s, w, smem, grid_x, st);
}

// ---------------------------------------------------------------- K8: window shift
// The window's K, K_raw and V rows move in 16-byte units (a row is a whole number of them).
template <typename T>
__global__ void window_stage_kernel(Geo g, logkv_state_t s, Work w, int rem) {
  pdl_entry();
  // copy [F, F+rem) -> staging [0, rem) when source and destination overlap
  constexpr int VN = Vec<T>::N;
  const int b = blockIdx.z, grp = blockIdx.y;
  const size_t base = ((size_t)b * g.G + grp) * g.cap2R * g.D / VN;
  const size_t n = (size_t)rem * g.D / VN, off = (size_t)g.F * g.D / VN;
  const uint4* rk = static_cast<const uint4*>(s.recent_k);
  const uint4* rkr = static_cast<const uint4*>(s.recent_k_raw);
  const uint4* rv = static_cast<const uint4*>(s.recent_v);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    static_cast<uint4*>(w.wk)[base + i] = rk[base + off + i];
    static_cast<uint4*>(w.wkr)[base + i] = rkr[base + off + i];
    static_cast<uint4*>(w.wv)[base + i] = rv[base + off + i];
  }
  if (grp == 0 && blockIdx.x == 0)
    for (int i = threadIdx.x; i < rem; i += blockDim.x) {
      w.wpos[(size_t)b * g.cap2R + i] = s.recent_pos[(size_t)b * g.cap2R + g.F + i];
      w.wends[(size_t)b * g.cap2R + i] = s.recent_ends[(size_t)b * g.cap2R + g.F + i];
    }
}

template <typename T>
__global__ void window_shift_kernel(Geo g, logkv_state_t s, Work w, int rem, int staged) {
  pdl_entry();
  constexpr int VN = Vec<T>::N;
  const int b = blockIdx.z, grp = blockIdx.y;
  const size_t base = ((size_t)b * g.G + grp) * g.cap2R * g.D / VN;
  const size_t n = (size_t)g.recent_count * g.D / VN;
  uint4* rk = static_cast<uint4*>(s.recent_k);
  uint4* rkr = static_cast<uint4*>(s.recent_k_raw);
  uint4* rv = static_cast<uint4*>(s.recent_v);
  const uint4* sk = staged ? static_cast<const uint4*>(w.wk) : rk;
  const uint4* skr = staged ? static_cast<const uint4*>(w.wkr) : rkr;
  const uint4* sv = staged ? static_cast<const uint4*>(w.wv) : rv;
  const size_t F = (size_t)g.F * g.D / VN, R = (size_t)rem * g.D / VN;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  // Without staging (rem <= F) unit j of [F, count) is read and then zeroed by
  // the same thread; [rem, F) is never read, and units below rem are only written by the
  // threads of their sources, so the loop starts at rem.  With staging every source is a copy.
  const size_t i0 = staged ? 0 : R;
  for (size_t i = i0 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    if (staged) {
      if (i < R) {
        rk[base + i] = sk[base + i];
        rkr[base + i] = skr[base + i];
        rv[base + i] = sv[base + i];
      } else {
        rk[base + i] = zero;
        rkr[base + i] = zero;
        rv[base + i] = zero;
      }
    } else if (i >= F) {
      const uint4 a = rk[base + i], c = rkr[base + i], e = rv[base + i];
      rk[base + i - F] = a;
      rkr[base + i - F] = c;
      rv[base + i - F] = e;
      rk[base + i] = zero;
      rkr[base + i] = zero;
      rv[base + i] = zero;
    } else if (i >= R) {
      rk[base + i] = zero;
      rkr[base + i] = zero;
      rv[base + i] = zero;
    }
  }
  if (grp == 0 && blockIdx.x == 0) {
    const size_t r = (size_t)b * g.cap2R;
    for (int i = threadIdx.x; i < g.recent_count; i += blockDim.x) {
      if (staged) {
        s.recent_pos[r + i] = i < rem ? w.wpos[r + i] : 0;
        s.recent_ends[r + i] = i < rem ? w.wends[r + i] : 0;
      } else if (i >= g.F) {
        const int64_t p = s.recent_pos[r + i];
        const uint8_t e = s.recent_ends[r + i];
        s.recent_pos[r + i - g.F] = p;
        s.recent_ends[r + i - g.F] = e;
        s.recent_pos[r + i] = 0;
        s.recent_ends[r + i] = 0;
      } else if (i >= rem) {
        s.recent_pos[r + i] = 0;
        s.recent_ends[r + i] = 0;
      }
    }
  }
}

// ---------------------------------------------------------------- window append
// The chunk's post-RoPE K, pre-RoPE K and V rows into window rows [recent_count, recent_count + n)
// (16-byte moves; every source row is contiguous and 16-byte aligned, rows addressed through
// element strides), its positions into recent_pos and its span-end flags into recent_ends.
struct AppendArgs {
  const void* k;
  const void* k_raw;
  const void* v;
  long long ks[3], krs[3], vs[3];   // element strides of the batch, group and token axes
  const int64_t* pos;               // [B, n] positions, or null: positions pos0 + t
  long long ps[2];                  // element strides of positions [B, n]
  long long pos0;
  const uint8_t* ends;              // [B, n] contiguous
  int n, recent_count;
};

// Chunk row t, 16-byte unit v of lane (b, grp) into window row `row` (K, pre-RoPE K, V).
template <typename T>
__device__ __forceinline__ void put_chunk_unit(const Geo& g, const logkv_state_t& s, const AppendArgs& a, int b,
                                               int grp, int t, int v, int row) {
  constexpr int VN = Vec<T>::N;
  const size_t d = (((size_t)b * g.G + grp) * g.cap2R + row) * g.D + (size_t)v * VN;
  const T* sk = static_cast<const T*>(a.k) + b * a.ks[0] + grp * a.ks[1] + t * a.ks[2] + v * VN;
  const T* skr = static_cast<const T*>(a.k_raw) + b * a.krs[0] + grp * a.krs[1] + t * a.krs[2] + v * VN;
  const T* sv = static_cast<const T*>(a.v) + b * a.vs[0] + grp * a.vs[1] + t * a.vs[2] + v * VN;
  *reinterpret_cast<uint4*>(static_cast<T*>(s.recent_k) + d) = *reinterpret_cast<const uint4*>(sk);
  *reinterpret_cast<uint4*>(static_cast<T*>(s.recent_k_raw) + d) = *reinterpret_cast<const uint4*>(skr);
  *reinterpret_cast<uint4*>(static_cast<T*>(s.recent_v) + d) = *reinterpret_cast<const uint4*>(sv);
}

template <typename T>
__global__ void window_append_kernel(Geo g, logkv_state_t s, AppendArgs a) {
  pdl_entry();
  constexpr int VN = Vec<T>::N;
  const int b = blockIdx.z, grp = blockIdx.y, DV = g.D / VN;
  const int units = a.n * DV;   // <= 8192 rows x 256 units
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < units; u += gridDim.x * blockDim.x) {
    const int t = u / DV;
    put_chunk_unit<T>(g, s, a, b, grp, t, u - t * DV, a.recent_count + t);
  }
  if (grp == 0 && blockIdx.x == 0)
    for (int t = threadIdx.x; t < a.n; t += blockDim.x) {
      const size_t r = (size_t)b * g.cap2R + a.recent_count + t;
      s.recent_pos[r] = a.pos ? a.pos[b * a.ps[0] + t * a.ps[1]] : a.pos0 + t;
      s.recent_ends[r] = a.ends[(size_t)b * a.n + t];
    }
}

// The window write of a flush whose chunk was not appended (logkv_flush_chunk): with c0 =
// a.recent_count old rows, F = g.F flushed, rem0 = c0 - F <= F kept, the window becomes
// [old rows F .. c0) ++ [chunk rows 0 .. n) ++ zeros.  Row r of [rem0, max(c0, rem0 + n)) is one
// thread's: it reads old row r (r in [F, c0)) and writes it to r - F (below rem0, a row no
// thread reads), then writes chunk row r - rem0 to r, or zeros (an old row left over).  Rows
// at c0 and above are zero already (every shift zeroes what it vacates) unless a chunk row
// lands there.
template <typename T>
__global__ void window_commit_kernel(Geo g, logkv_state_t s, AppendArgs a) {
  pdl_entry();
  constexpr int VN = Vec<T>::N;
  const int b = blockIdx.z, grp = blockIdx.y, DV = g.D / VN;
  const int c0 = a.recent_count, F = g.F, rem0 = c0 - F, hi = max(c0, rem0 + a.n);
  uint4* rk = static_cast<uint4*>(s.recent_k);
  uint4* rkr = static_cast<uint4*>(s.recent_k_raw);
  uint4* rv = static_cast<uint4*>(s.recent_v);
  const size_t base = ((size_t)b * g.G + grp) * g.cap2R * DV;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  for (int u = rem0 * DV + blockIdx.x * blockDim.x + threadIdx.x; u < hi * DV; u += gridDim.x * blockDim.x) {
    const int r = u / DV, v = u - r * DV;
    if (r >= F && r < c0) {
      const uint4 x0 = rk[base + u], x1 = rkr[base + u], x2 = rv[base + u];
      rk[base + u - (size_t)F * DV] = x0;
      rkr[base + u - (size_t)F * DV] = x1;
      rv[base + u - (size_t)F * DV] = x2;
    }
    if (r - rem0 < a.n) {
      put_chunk_unit<T>(g, s, a, b, grp, r - rem0, v, r);
    } else {
      rk[base + u] = zero;
      rkr[base + u] = zero;
      rv[base + u] = zero;
    }
  }
  if (grp == 0 && blockIdx.x == 0) {
    const size_t w0 = (size_t)b * g.cap2R;
    for (int r = rem0 + threadIdx.x; r < hi; r += blockDim.x) {
      if (r >= F && r < c0) {
        const int64_t p = s.recent_pos[w0 + r];
        const uint8_t e = s.recent_ends[w0 + r];
        s.recent_pos[w0 + r - F] = p;
        s.recent_ends[w0 + r - F] = e;
      }
      const int t = r - rem0;
      if (t < a.n) {
        s.recent_pos[w0 + r] = a.pos ? a.pos[b * a.ps[0] + t * a.ps[1]] : a.pos0 + t;
        s.recent_ends[w0 + r] = a.ends[(size_t)b * a.n + t];
      } else {
        s.recent_pos[w0 + r] = 0;
        s.recent_ends[w0 + r] = 0;
      }
    }
  }
}

// ---------------------------------------------------------------- workspace
struct Carver {
  char* base;
  size_t off = 0;
  template <typename P>
  P* take(size_t count, size_t elem) {
    off = (off + 255) & ~size_t(255);
    P* p = reinterpret_cast<P*>(base ? base + off : nullptr);
    off += count * elem;
    return p;
  }
};

static int next_pow2(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

static Geo make_geo(const logkv_layout_t& L, int F, int recent_count) {
  Geo g{};
  g.B = L.batch;
  g.G = L.groups;
  g.D = L.dim;
  g.K = L.clusters;
  g.L = L.levels;
  g.Bs = L.slots;
  g.cap2R = L.recent_capacity;
  g.P = L.exact;
  g.span_cap = L.span_cap;
  g.beta = L.beta;
  g.F = F;
  g.NW = g.P + F;
  g.NC = g.P + F;
  g.recent_count = recent_count;
  g.S = g.NW + g.K * g.L * g.Bs + g.K * (g.L + 2);
  g.sort_cap = next_pow2(g.L * g.Bs + g.NW);
  g.eta = L.eta;
  g.g0 = L.g0;
  g.lam = L.lam;
  g.shard_ranks = 1;
  g.route = L.route;
  g.passes = L.merge_passes < 1 ? 1 : L.merge_passes;
  g.Mg = g.NW + g.K;
  return g;
}

static size_t carve(const Geo& g, size_t esize, char* base, Work* w) {
  Carver c{base};
  const size_t B = g.B, G = g.G, D = g.D, K = g.K, P = g.P, NC = g.NC, NW = g.NW, S = g.S;
  w->tape_cut_lane = -1;
  w->status = c.take<int32_t>(1, 4);
  w->counters = c.take<unsigned long long>(kNumCounters, 8);
  w->ties = c.take<TieEntry>(kTieCap, sizeof(TieEntry));  // lands at kTieOffset (checked below)
  w->snap_k = c.take<char>(B * G * P * D, esize);
  w->snap_v = c.take<char>(B * G * P * D, esize);
  w->snap_pos = c.take<int64_t>(B * P, 8);
  w->snap_rowcount = c.take<int32_t>(B, 4);
  w->cand_s0 = c.take<int32_t>(B * NC, 4);
  w->cand_n0 = c.take<int32_t>(B * NC, 4);
  w->cand_s1 = c.take<int32_t>(B * NC, 4);
  w->cand_n1 = c.take<int32_t>(B * NC, 4);
  w->cand_flags = c.take<uint8_t>(B * NC, 1);
  w->n_cand = c.take<int32_t>(B, 4);
  w->scores = c.take<float>(B * NC, 4);
  w->gpart = c.take<float>(B * NC * G * 2, 4);
  w->keep_idx = c.take<int32_t>(B * P, 4);
  w->nkeep = c.take<int32_t>(B, 4);
  w->arch_idx = c.take<int32_t>(B * NW, 4);
  w->narch = c.take<int32_t>(B, 4);
  w->span_len = c.take<int32_t>(B * P, 4);
  w->span_closed = c.take<uint8_t>(B * P, 1);
  w->nspans = c.take<int32_t>(B, 4);
  w->assign = c.take<int8_t>(B * G * NW, 1);
  w->assign_tok = c.take<int8_t>(B * G * NW, 1);
  w->orphan = c.take<uint8_t>(B * G * NW, 1);
  w->s_winner = c.take<float>(B * G * NW, 4);
  w->cnorm = c.take<float>(B * G * K, 4);
  w->tok_pos = c.take<int64_t>(B * NW, 8);
  w->tok_list = c.take<int32_t>(B * G * NW, 4);
  w->plan_off = c.take<int32_t>(B * G * K, 4);
  w->plan_n = c.take<int32_t>(B * G * K, 4);
  w->plan_type = c.take<int32_t>(B * G * K, 4);
  w->plan_m0 = c.take<int32_t>(B * G * K, 4);
  w->plan_scr = c.take<int32_t>(B * G * K, 4);
  w->plan_base = c.take<int64_t>(B * G * K, 8);
  w->lane_mode = c.take<int32_t>(B * G * K, 4);
  w->lane_plan = c.take<LevelPlan>(B * G * K * (size_t)g.L, sizeof(LevelPlan));
  w->sk = c.take<char>(B * G * 2 * S * D, esize);
  w->sv = c.take<char>(B * G * 2 * S * D, esize);
  w->sw = c.take<float>(B * G * 2 * S, 4);
  w->slo = c.take<int64_t>(B * G * 2 * S, 8);
  w->shi = c.take<int64_t>(B * G * 2 * S, 8);
  w->sswp = c.take<int64_t>(B * G * 2 * S, 8);
  w->sord = c.take<int64_t>(B * G * 2 * S, 8);
  w->spad = c.take<uint8_t>(B * G * 2 * S, 1);
  const size_t R = g.cap2R;
  w->wk = c.take<char>(B * G * R * D, esize);
  w->wkr = c.take<char>(B * G * R * D, esize);
  w->wv = c.take<char>(B * G * R * D, esize);
  w->wpos = c.take<int64_t>(B * R, 8);
  w->wends = c.take<uint8_t>(B * R, 1);
  if (g.route == LOGKV_ROUTE_UNIFIED) {
    const size_t lanes = B * G, Mg = g.Mg;
    UWork& u = w->u;
    u.dist = c.take<float>(lanes * Mg * Mg, 4);
    u.mu_c = c.take<float>(lanes * NW * D, 4);
    u.mu_g = c.take<float>(lanes * Mg * D, 4);
    u.mass = c.take<float>(lanes * Mg, 4);
    u.radius = c.take<float>(lanes * Mg, 4);
    u.packed = c.take<long long>(lanes * Mg, 8);
    u.restr = c.take<long long>(lanes * Mg, 8);
    u.trace_c = c.take<int32_t>(lanes * NW * 2, 4);
    u.trace_g = c.take<int32_t>(lanes * Mg * 2, 4);
    u.label = c.take<int32_t>(lanes * NW, 4);
    u.words = c.take<int32_t>(lanes * kULaneWords, 4);
    u.limit = c.take<float>(lanes, 4);
    u.old = c.take<int32_t>(lanes * K, 4);
    u.ward = c.take<int32_t>(lanes * K * 2, 4);
    u.alive = c.take<uint8_t>(lanes * Mg, 1);
    u.stuck = c.take<uint8_t>(lanes * 2, 1);
  }
  return (c.off + 255) & ~size_t(255);
}

static int validate(const logkv_layout_t* L, int F) {
  if (!L) return LOGKV_E_POINTER;
  if (L->dtype != LOGKV_DTYPE_F32 && L->dtype != LOGKV_DTYPE_BF16) return LOGKV_E_DTYPE;
  if (L->batch < 1 || L->groups < 1 || L->dim < 4 || L->dim > 1024) return LOGKV_E_SHAPE;
  if (L->dim % (L->dtype == LOGKV_DTYPE_BF16 ? 8 : 4)) return LOGKV_E_SHAPE;  // 16-byte rows
  if (L->clusters < 2 || L->clusters > kMaxClusters || L->levels < 2 || L->levels > kMaxLevels) return LOGKV_E_SHAPE;
  if (L->slots < 2 || L->exact < 1 || L->span_cap < 1 || L->span_cap > L->exact) return LOGKV_E_SHAPE;
  if (F < 1 || F > L->recent_capacity || L->exact + F > 8192) return LOGKV_E_SHAPE;
  if (L->levels * L->slots + L->exact + F > (1 << 14)) return LOGKV_E_SHAPE;
  if (L->route != LOGKV_ROUTE_ATTACH && L->route != LOGKV_ROUTE_UNIFIED) return LOGKV_E_SHAPE;
  if (L->route == LOGKV_ROUTE_UNIFIED &&
      (L->merge_passes < 1 || L->exact + F + L->clusters > LOGKV_UNIFIED_MAX_ROWS || L->dim % 4))
    return LOGKV_E_SHAPE;
  return LOGKV_OK;
}

// The decision arrays of a flush: workspace and state <-> tape (to_tape selects the direction).
static TapeSegs tape_segments(const Geo& g, const logkv_state_t& s, const Work& w, const TapeView& t, bool to_tape) {
  TapeSegs segs{};
  const size_t B = g.B, G = g.G, K = g.K, P = g.P, NW = g.NW;
  auto add = [&](void* live, void* rec, size_t bytes) {
    segs.src[segs.n] = to_tape ? live : rec;
    segs.dst[segs.n] = to_tape ? rec : live;
    segs.bytes[segs.n] = bytes;
    ++segs.n;
  };
  add(w.keep_idx, t.keep_idx, B * P * 4);
  add(w.nkeep, t.nkeep, B * 4);
  add(w.arch_idx, t.arch_idx, B * NW * 4);
  add(w.narch, t.narch, B * 4);
  add(w.span_len, t.span_len, B * P * 4);
  add(w.span_closed, t.span_closed, B * P);
  add(w.nspans, t.nspans, B * 4);
  add(w.tok_list, t.tok_list, B * G * NW * 4);
  add(w.plan_off, t.plan_off, B * G * K * 4);
  add(w.plan_n, t.plan_n, B * G * K * 4);
  add(w.plan_type, t.plan_type, B * G * K * 4);
  add(w.plan_m0, t.plan_m0, B * G * K * 4);
  add(w.plan_scr, t.plan_scr, B * G * K * 4);
  add(w.plan_base, t.plan_base, B * G * K * 8);
  if (g.route == LOGKV_ROUTE_UNIFIED) {
    add(w.u.words, t.uwords, B * G * kULaneWords * 4);
    add(w.u.ward, t.ward, B * G * K * 2 * 4);
  }
  return segs;
}

// ---------------------------------------------------------------- unified route launches
// The Gram tile's output staging (its panels are static shared memory).
static size_t unified_gram_smem(const Geo&) { return (size_t)kGramTile * (kGramTile + 1) * 4; }
// Every CTA of a reduction cluster holds the round's tables; sized for the smallest cluster (2).
static size_t unified_round_smem(const Geo& g) {
  return logkv_ward::round_smem_bytes(g.Mg, logkv_ward::sort_width(g.Mg), 2);
}
// CTAs per lane of the reductions: one lane per cluster and one CTA per SM (the round's shared
// memory), so larger clusters shorten a lane's rounds while smaller ones fit more lanes at once:
// 8 while the lanes fit on the SMs in one wave of 8-CTA clusters (15 lanes), else 4 (measured at
// 32 lanes and D = 128: 10.5 ms per pass pair with 8, 7.0 with 4, 9.0 with 2).
static int unified_cluster(const Geo& g) {
  const int lanes = g.B * g.G;
  const char* env = getenv("LOGKV_UNIFIED_CLUSTER");
  if (env) {
    const int v = atoi(env);
    if (v == 2 || v == 4 || v == 8) return v;
  }
  return lanes <= 15 ? 8 : 4;
}
// A cluster launch that also carries the programmatic dependency on the previous kernel.
template <typename... KArgs, typename... Args>
static void launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               int cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, kern, args...);
}
static int unified_sort_cap(const Geo& g) {
  int p = 2;
  while (p < 2 * g.L * g.Bs) p <<= 1;
  return p;
}
static size_t unified_walk_bytes(const Geo& g, size_t esize) { return (walk_smem(g, esize, kTileRows) + 15) & ~size_t(15); }
static size_t unified_ward_smem(const Geo& g, size_t esize) {
  return unified_walk_bytes(g, esize) + 2 * (size_t)unified_sort_cap(g) * 8;
}
static bool unified_fits(const Geo& g, size_t esize) {
  const size_t lim = 227 * 1024;
  return unified_gram_smem(g) <= lim && unified_round_smem(g) <= lim && unified_ward_smem(g, esize) <= lim &&
         3 * (size_t)g.NW * 4 <= lim && 3 * (size_t)g.Mg * 4 <= lim && (size_t)g.B * 4 <= lim &&
         (size_t)g.B * g.G <= 65535;
}

template <typename T, bool BETA, int DC>
static void launch_ward(const Geo& g, const logkv_state_t& s, const Work& w, cudaStream_t st, uint8_t* ward_cuts) {
  const size_t smem = unified_ward_smem(g, sizeof(T));
  smem_limit(unified_ward_kernel<T, BETA, DC>, smem);
  launch_pdl(unified_ward_kernel<T, BETA, DC>, dim3(g.G, g.B), kCascadeThreads, smem, st, g, s, w,
             unified_sort_cap(g), unified_walk_bytes(g, sizeof(T)), ward_cuts);
}

// The Ward merges of a flush (recorded jobs when replaying an update tape).
template <typename T>
static void launch_ward_all(const Geo& g, const logkv_state_t& s, const Work& w, cudaStream_t st, uint8_t* ward_cuts) {
  if (g.beta) {
    if (g.D == 128) launch_ward<T, true, 128>(g, s, w, st, ward_cuts);
    else if (g.D == 64) launch_ward<T, true, 64>(g, s, w, st, ward_cuts);
    else launch_ward<T, true, 0>(g, s, w, st, ward_cuts);
  } else {
    if (g.D == 128) launch_ward<T, false, 128>(g, s, w, st, ward_cuts);
    else if (g.D == 64) launch_ward<T, false, 64>(g, s, w, st, ward_cuts);
    else launch_ward<T, false, 0>(g, s, w, st, ward_cuts);
  }
}

// The unified route between the span choice and the per-cluster plan: candidate pass, labels,
// global pass, route, Ward merges (11 launches, no host synchronisation).
template <typename T>
static void launch_unified(const Geo& g, const logkv_state_t& s, const Work& w, cudaStream_t st, uint8_t* ward_cuts) {
  const int lanes = g.B * g.G, tiles = (g.Mg + kGramTile - 1) / kGramTile;
  const int S = logkv_ward::sort_width(g.Mg), CL = unified_cluster(g);
  const size_t gram = unified_gram_smem(g), round = unified_round_smem(g);
  const size_t lab = 3 * (size_t)g.NW * 4, rte = 3 * (size_t)g.Mg * 4, tile = (size_t)g.B * 4;
  smem_limit(unified_dist_kernel, gram);
  smem_limit(unified_reduce_kernel, round);
  smem_limit(unified_labels_kernel, lab);
  smem_limit(unified_route_kernel, rte);
  smem_limit(unified_tile_kernel, tile);
  const int per = std::max(1, std::min(64, (g.NW * g.D + 255) / 256));
  for (int pass = 0; pass < 2; ++pass) {
    // The load kernel clears the lane words, so the candidate pass's tile flags follow it.
    if (pass == 0) launch_pdl(unified_load_kernel<T>, dim3(per, g.G, g.B), 256, 0, st, g, s, w);
    launch_pdl(unified_tile_kernel, dim3(1), 1024, tile, st, g, w, pass);
    launch_pdl(unified_dist_kernel, dim3(tiles, tiles, lanes), 256, gram, st, g, w, pass);
    launch_pdl_cluster(unified_reduce_kernel, dim3(lanes * CL), logkv_ward::kUThreads, round, st, CL, g, w, pass, S);
    if (pass == 0) launch_pdl(unified_labels_kernel, dim3(g.G, g.B), 1024, lab, st, g, s, w);
  }
  launch_pdl(unified_route_kernel, dim3(g.G, g.B), 1024, rte, st, g, s, w);
  launch_ward_all<T>(g, s, w, st, ward_cuts);
}

// Phases: kPhaseScores = snapshot, span cut, span scores (the group parts of this rank) and
// attach decisions; kPhaseRoute = the bounded greedy, seeding and the per-cluster plan;
// kPhaseApply = the ladder (prepare, cascade), the pool rewrite and the window shift.  Scores
// and route write only the workspace.  A KV-head-sharded flush all-gathers the group parts
// between scores and route; an overlapped flush runs scores + route on a side stream.
constexpr int kPhaseScores = 1, kPhaseRoute = 2, kPhaseApply = 4, kPhaseDecide = 3, kPhaseCommit = 6, kPhaseAll = 7;

template <typename T>
static int launch_flush(const Geo& g, const logkv_state_t& s, const Work& w, cudaStream_t st, cudaEvent_t* ev,
                        int phases = kPhaseAll, const TapeView* tape = nullptr, const AppendArgs* chunk = nullptr) {
  int stage = 0;
  auto mark = [&]() {
    if (ev) cudaEventRecord(ev[stage], st);
    ++stage;
  };
  const int sm_count = 148;
  const int per_bg = std::max(1, std::min(64, (g.P * g.D / (int)(16 / sizeof(T)) + 255) / 256));
  const int per_pay = std::max(1, std::min(64, (g.F * g.D / (int)(16 / sizeof(T)) + 255) / 256));
  // Recording: the flushed window rows as this flush sees them, before anything moves.
  if (tape) launch_pdl(tape_payload_kernel<T>, dim3(per_pay, g.G, g.B), 256, 0, st, g, s, *tape, 1);
  if (phases & kPhaseScores) {
  mark();
  launch_pdl(snapshot_kernel<T>, dim3(per_bg, g.G, g.B), 256, 0, st, g, s, w);
  mark();
  const size_t cut_smem = 2 * (size_t)g.F * sizeof(int);
  if (cut_smem > 48 * 1024) cudaFuncSetAttribute(alpha_cut_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cut_smem);
  launch_pdl(alpha_cut_kernel, g.B, 1024, cut_smem, st, g, s, w);
  mark();
  const size_t score_smem = score_smem_bytes(g, sizeof(T));
  const int score_blocks = std::max(1, std::min((g.NC * g.G + 7) / 8, 2 * sm_count / g.B + 1));
  if (g.D == 128) launch_score<T, 128>(g, s, w, score_smem, score_blocks, st);
  else if (g.D == 64) launch_score<T, 64>(g, s, w, score_smem, score_blocks, st);
  else launch_score<T, 0>(g, s, w, score_smem, score_blocks, st);
  if (g.route != LOGKV_ROUTE_UNIFIED) {
    const size_t attach_smem = attach_smem_bytes(g);
    const int attach_x = (g.NW + kAttachTokens - 1) / kAttachTokens;
    if (g.D == 128) launch_attach<T, 128>(g, s, w, attach_smem, attach_x, st);
    else if (g.D == 64) launch_attach<T, 64>(g, s, w, attach_smem, attach_x, st);
    else launch_attach<T, 0>(g, s, w, attach_smem, attach_x, st);
  }
  }
  if (phases & kPhaseRoute) {
  mark();
  const size_t choose_smem = choose_smem_bytes(g);
  if (choose_smem > 48 * 1024)
    cudaFuncSetAttribute(alpha_choose_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)choose_smem);
  launch_pdl(alpha_choose_kernel, g.B, 1024, choose_smem, st, g, s, w);
  mark();
  if (g.route == LOGKV_ROUTE_UNIFIED) {
    launch_unified<T>(g, s, w, st, tape ? tape->ward_cuts : nullptr);
  } else {
    // Seeding: one 8-CTA cluster per lane; rows staged in shared memory when they fit.
    Geo gs = g;
    const size_t chunk = (size_t)(g.NW + kSeedCluster - 1) / kSeedCluster;
    const size_t base = ((size_t)g.D + (size_t)g.K * (g.D + 1) + chunk + chunk * g.K) * sizeof(float);
    const size_t rows = chunk * (size_t)(g.D + 4 / sizeof(T)) * sizeof(T);
    gs.seed_staged = base + rows <= 200 * 1024 ? 1 : 0;
    const size_t seed_smem = base + (gs.seed_staged ? rows : 0);
    if (seed_smem > 48 * 1024)
      cudaFuncSetAttribute(seed_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)seed_smem);
    launch_pdl(seed_kernel<T>, dim3(kSeedCluster * g.G, g.B), 512, seed_smem, st, gs, s, w);
  }
  launch_pdl(plan_kernel<T>, dim3(g.G, g.B), 1024, 0, st, g, s, w);
  }
  if (!(phases & kPhaseApply)) return (int)cudaGetLastError();
  mark();
  launch_prepare<T>(g, s, w, st);
  mark();
  launch_cascade_all<T>(g, s, w, st);
  mark();
  launch_pdl(pool_rewrite_kernel<T>, dim3(per_bg, g.G, g.B), 256, 0, st, g, s, w);
  mark();
  if (chunk) {
    const int rem0 = chunk->recent_count - g.F, rows = std::max(chunk->recent_count, rem0 + chunk->n) - rem0;
    const int per = std::max(1, std::min(128, (rows * g.D / (int)(16 / sizeof(T)) + 255) / 256));
    launch_pdl(window_commit_kernel<T>, dim3(per, g.G, g.B), 256, 0, st, g, s, *chunk);
  } else {
    const int rem = g.recent_count - g.F;
    const int per_win = std::max(1, std::min(128, (g.recent_count * g.D / (int)(16 / sizeof(T)) + 255) / 256));
    const int staged = rem > g.F ? 1 : 0;
    if (staged) launch_pdl(window_stage_kernel<T>, dim3(per_win, g.G, g.B), 256, 0, st, g, s, w, rem);
    launch_pdl(window_shift_kernel<T>, dim3(per_win, g.G, g.B), 256, 0, st, g, s, w, rem, staged);
  }
  mark();
  // Recording: the decisions (workspace) and the new span table (state) into the tape.
  if (tape) launch_pdl(tape_copy_kernel, dim3(2 * sm_count), 256, 0, st, tape_segments(g, s, w, *tape, true));
  return (int)cudaGetLastError();
}

// Replay of a recorded flush: the recorded payload replaces the window's flushed rows, the
// recorded decisions replace the span cut / scores / choice / attach / seeding / plan kernels,
// and the cascade takes the recorded Beta cuts; the state transition is the recorded one.
template <typename T>
static int launch_replay(const Geo& g, const logkv_state_t& s, const Work& w, const TapeView& tape, cudaStream_t st) {
  const int sm_count = 148;
  const int per_bg = std::max(1, std::min(64, (g.P * g.D / (int)(16 / sizeof(T)) + 255) / 256));
  const int per_pay = std::max(1, std::min(64, (g.F * g.D / (int)(16 / sizeof(T)) + 255) / 256));
  launch_pdl(snapshot_kernel<T>, dim3(per_bg, g.G, g.B), 256, 0, st, g, s, w);
  launch_pdl(tape_payload_kernel<T>, dim3(per_pay, g.G, g.B), 256, 0, st, g, s, tape, 0);
  launch_pdl(tape_copy_kernel, dim3(2 * sm_count), 256, 0, st, tape_segments(g, s, w, tape, false));
  if (g.route == LOGKV_ROUTE_UNIFIED) {
    // The recorded Ward merges (with their recorded cuts) before the per-cluster plan; they use the
    // plan fields of the lanes they rebuild, so the recorded plan is copied back after them.
    launch_ward_all<T>(g, s, w, st, tape.ward_cuts);
    launch_pdl(tape_copy_kernel, dim3(2 * sm_count), 256, 0, st, tape_segments(g, s, w, tape, false));
  }
  launch_pdl(lane_plan_kernel, dim3(g.G, g.B), 32 * ((g.K + 31) / 32), 0, st, g, s, w);
  launch_prepare<T>(g, s, w, st);
  launch_cascade_all<T>(g, s, w, st);
  launch_pdl(pool_rewrite_kernel<T>, dim3(per_bg, g.G, g.B), 256, 0, st, g, s, w);
  const int rem = g.recent_count - g.F;
  const int per_win = std::max(1, std::min(128, (g.recent_count * g.D / (int)(16 / sizeof(T)) + 255) / 256));
  const int staged = rem > g.F ? 1 : 0;
  if (staged) launch_pdl(window_stage_kernel<T>, dim3(per_win, g.G, g.B), 256, 0, st, g, s, w, rem);
  launch_pdl(window_shift_kernel<T>, dim3(per_win, g.G, g.B), 256, 0, st, g, s, w, rem, staged);
  return (int)cudaGetLastError();
}

static int run_flush(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                     int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream, cudaEvent_t* ev,
                     int phases = kPhaseAll, const float* gpart_all = nullptr, int ranks = 1,
                     int tape_mode = kTapeNone, void* tape = nullptr, size_t tape_bytes = 0,
                     long long rank_stride = 0, const AppendArgs* chunk = nullptr) {
  const int v = validate(layout, flush_tokens);
  if (v != LOGKV_OK) return v;
  if (!state || !workspace) return LOGKV_E_POINTER;
  // Rows move in 16-byte units: every K/V buffer, the centres and the workspace start on a
  // 16-byte boundary; the other buffers at least on their element size.
  auto a16 = [](const void* p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  auto a8 = [](const void* p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 7) == 0; };
  auto a4 = [](const void* p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 3) == 0; };
  const logkv_state_t& S = *state;
  if (!a16(workspace) || !a16(S.level_k) || !a16(S.level_v) || !a16(S.centroid) || !a16(S.recent_k) ||
      !a16(S.recent_k_raw) || !a16(S.recent_v) || !a16(S.alpha_k_raw) || !a16(S.alpha_v) || !a4(S.level_w) ||
      !a8(S.level_p_lo) || !a8(S.level_p_hi) || !a8(S.level_sum_wp) || !a8(S.level_order) || !S.pad_mask ||
      !S.level_count || !a4(S.n_eff) || !a4(S.n_total) || !a8(S.p_hi_c) || !a4(S.level0_phase) || !S.alive ||
      !a4(S.s_h) || !a8(S.recent_pos) || !S.recent_ends || !a8(S.alpha_pos) || !S.alpha_valid ||
      !a4(S.alpha_span_len) || !S.alpha_span_closed || !a4(S.alpha_nspans) || !a4(S.alpha_rowcount) ||
      !a4(S.alpha_count))
    return LOGKV_E_POINTER;
  if (recent_count < flush_tokens || recent_count > layout->recent_capacity) return LOGKV_E_SHAPE;
  const size_t esize = layout->dtype == LOGKV_DTYPE_BF16 ? 2 : 4;
  if (ranks < 1 || (ranks > 1 && !gpart_all)) return LOGKV_E_POINTER;
  Geo g = make_geo(*layout, flush_tokens, recent_count);
  g.shard_ranks = ranks;
  g.gpart_stride = rank_stride > 0 ? rank_stride : (long long)g.B * g.NC * g.G * 2;
  if (rank_stride > 0 && rank_stride < (long long)g.B * g.NC * g.G * 2) return LOGKV_E_SHAPE;
  Work w{};
  const size_t need = carve(g, esize, static_cast<char*>(workspace), &w);
  if (workspace_bytes < need) return LOGKV_E_WORKSPACE;
  if (reinterpret_cast<char*>(w.ties) != static_cast<char*>(workspace) + kTieOffset) return LOGKV_E_WORKSPACE;
  if (cascade_smem(g, esize) > 227 * 1024 || prep_smem_bytes(g, esize) > 227 * 1024 ||
      choose_smem_bytes(g) > 227 * 1024 || score_smem_bytes(g, esize) > 227 * 1024 || attach_smem_bytes(g) > 227 * 1024)
    return LOGKV_E_SMEM;
  if (g.route == LOGKV_ROUTE_UNIFIED && !unified_fits(g, esize)) return LOGKV_E_SMEM;
  w.gpart_all = gpart_all;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (chunk && (tape_mode != kTapeNone || phases != kPhaseAll)) return LOGKV_E_SHAPE;
  // The unified route's Ward merges rewrite ladders before the per-cluster plan, so its route
  // phase runs only together with the apply phase, and only whole flushes keep update tapes.
  if (layout->route == LOGKV_ROUTE_UNIFIED &&
      (((phases & kPhaseRoute) && !(phases & kPhaseApply)) ||
       (tape_mode != kTapeNone && (phases != kPhaseAll || ranks != 1))))
    return LOGKV_E_SHAPE;
  if (tape_mode != kTapeNone) {
    TapeView t{};
    // A whole unsharded flush, or the commit half of a sharded one when recording (the record
    // holds the span choice, so its replay needs no exchange).
    const bool whole = phases == kPhaseAll && ranks == 1;
    const bool commit_record = phases == kPhaseCommit && tape_mode == kTapeRecord;
    if (!tape || (reinterpret_cast<uintptr_t>(tape) & 15) != 0 || !(whole || commit_record)) return LOGKV_E_POINTER;
    if (tape_bytes < tape_carve(g, esize, static_cast<char*>(tape), &t)) return LOGKV_E_WORKSPACE;
    g.tape = tape_mode;
    w.tape_cuts = t.cuts;
    if (tape_mode == kTapeReplay) {
      if (layout->dtype == LOGKV_DTYPE_BF16) return launch_replay<__nv_bfloat16>(g, *state, w, t, st);
      return launch_replay<float>(g, *state, w, t, st);
    }
    if (layout->dtype == LOGKV_DTYPE_BF16) return launch_flush<__nv_bfloat16>(g, *state, w, st, ev, phases, &t);
    return launch_flush<float>(g, *state, w, st, ev, phases, &t);
  }
  if (layout->dtype == LOGKV_DTYPE_BF16) return launch_flush<__nv_bfloat16>(g, *state, w, st, ev, phases, nullptr, chunk);
  return launch_flush<float>(g, *state, w, st, ev, phases, nullptr, chunk);
}

}  // namespace logkv

using namespace logkv;

extern "C" size_t logkv_flush_workspace_bytes(const logkv_layout_t* layout, int32_t flush_tokens) {
  if (validate(layout, flush_tokens) != LOGKV_OK) return 0;
  const Geo g = make_geo(*layout, flush_tokens, layout->recent_capacity);
  Work w{};
  return carve(g, layout->dtype == LOGKV_DTYPE_BF16 ? 2 : 4, nullptr, &w);
}

extern "C" int logkv_flush(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                           int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream) {
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream, nullptr);
}

extern "C" int logkv_flush_decide(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                  int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream) {
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream, nullptr,
                   kPhaseDecide);
}

extern "C" int logkv_flush_apply(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                 int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream) {
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream, nullptr,
                   kPhaseApply);
}

extern "C" size_t logkv_tape_bytes(const logkv_layout_t* layout, int32_t flush_tokens) {
  if (validate(layout, flush_tokens) != LOGKV_OK) return 0;
  const Geo g = make_geo(*layout, flush_tokens, layout->recent_capacity);
  TapeView t{};
  return tape_carve(g, layout->dtype == LOGKV_DTYPE_BF16 ? 2 : 4, nullptr, &t);
}

extern "C" int logkv_flush_record(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                  int32_t recent_count, void* workspace, size_t workspace_bytes, void* tape,
                                  size_t tape_bytes, void* stream) {
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream, nullptr,
                   kPhaseAll, nullptr, 1, kTapeRecord, tape, tape_bytes);
}

extern "C" int logkv_flush_commit_record(const logkv_layout_t* layout, const logkv_state_t* state,
                                         int32_t flush_tokens, int32_t recent_count, void* workspace,
                                         size_t workspace_bytes, const float* partials_all, int32_t ranks,
                                         int64_t rank_stride, void* tape, size_t tape_bytes, void* stream) {
  if (rank_stride < 0) return LOGKV_E_SHAPE;
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream, nullptr,
                   kPhaseCommit, partials_all, ranks, kTapeRecord, tape, tape_bytes, rank_stride);
}

extern "C" int logkv_flush_replay(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                  int32_t recent_count, void* workspace, size_t workspace_bytes, const void* tape,
                                  size_t tape_bytes, void* stream) {
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream, nullptr,
                   kPhaseAll, nullptr, 1, kTapeReplay, const_cast<void*>(tape), tape_bytes);
}

// Chunk arguments: checks (LOGKV_E_POINTER for a missing or misaligned row, LOGKV_E_SHAPE for
// rows past the window) and the kernel's view.
static int make_append(const logkv_layout_t* layout, const logkv_state_t* state, const void* k,
                       const int64_t* k_strides, const void* k_raw, const int64_t* k_raw_strides, const void* v,
                       const int64_t* v_strides, const int64_t* positions, const int64_t* pos_strides, int64_t pos0,
                       const uint8_t* ends, int32_t n, int32_t recent_count, AppendArgs* out) {
  if (!state || !k || !k_raw || !v || !ends || !k_strides || !k_raw_strides || !v_strides ||
      (positions && !pos_strides))
    return LOGKV_E_POINTER;
  if (n < 1 || recent_count < 0 || recent_count + n > layout->recent_capacity) return LOGKV_E_SHAPE;
  const size_t esize = layout->dtype == LOGKV_DTYPE_BF16 ? 2 : 4;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  AppendArgs a{};
  a.k = k;
  a.k_raw = k_raw;
  a.v = v;
  for (int i = 0; i < 3; ++i) {
    a.ks[i] = k_strides[i];
    a.krs[i] = k_raw_strides[i];
    a.vs[i] = v_strides[i];
    // Every row must start on a 16-byte boundary (rows are contiguous along the head dim).
    if ((a.ks[i] * (long long)esize) % 16 || (a.krs[i] * (long long)esize) % 16 || (a.vs[i] * (long long)esize) % 16)
      return LOGKV_E_POINTER;
  }
  a.ps[0] = positions ? pos_strides[0] : 0;
  a.ps[1] = positions ? pos_strides[1] : 0;
  a.pos = positions;
  a.pos0 = pos0;
  a.ends = ends;
  a.n = n;
  a.recent_count = recent_count;
  if (!a16(k) || !a16(k_raw) || !a16(v) || !a16(state->recent_k) || !a16(state->recent_k_raw) ||
      !a16(state->recent_v) || !state->recent_pos || !state->recent_ends)
    return LOGKV_E_POINTER;
  *out = a;
  return LOGKV_OK;
}

extern "C" int logkv_window_append(const logkv_layout_t* layout, const logkv_state_t* state, const void* k,
                                   const int64_t* k_strides, const void* k_raw, const int64_t* k_raw_strides,
                                   const void* v, const int64_t* v_strides, const int64_t* positions,
                                   const int64_t* pos_strides, int64_t pos0, const uint8_t* ends, int32_t n,
                                   int32_t recent_count, void* stream) {
  const int val = validate(layout, 1);
  if (val != LOGKV_OK) return val;
  AppendArgs a{};
  const int rc = make_append(layout, state, k, k_strides, k_raw, k_raw_strides, v, v_strides, positions, pos_strides,
                             pos0, ends, n, recent_count, &a);
  if (rc != LOGKV_OK) return rc;
  const size_t esize = layout->dtype == LOGKV_DTYPE_BF16 ? 2 : 4;
  const Geo g = make_geo(*layout, 1, recent_count);
  const int per = std::max(1, std::min(64, (int)(((size_t)n * g.D / (16 / esize) + 255) / 256)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (layout->dtype == LOGKV_DTYPE_BF16)
    launch_pdl(window_append_kernel<__nv_bfloat16>, dim3(per, g.G, g.B), 256, 0, st, g, *state, a);
  else
    launch_pdl(window_append_kernel<float>, dim3(per, g.G, g.B), 256, 0, st, g, *state, a);
  return (int)cudaGetLastError();
}

static int flush_chunk(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                       int32_t recent_count, const logkv_chunk_t* c, void* workspace, size_t workspace_bytes,
                       void* stream, cudaEvent_t* ev) {
  const int val = validate(layout, flush_tokens);
  if (val != LOGKV_OK) return val;
  if (!c) return LOGKV_E_POINTER;
  if (recent_count < flush_tokens || recent_count > 2 * flush_tokens) return LOGKV_E_SHAPE;
  AppendArgs a{};
  const int rc = make_append(layout, state, c->k, c->k_strides, c->k_raw, c->k_raw_strides, c->v, c->v_strides,
                             c->positions, c->pos_strides, c->pos0, c->ends, c->n, recent_count, &a);
  if (rc != LOGKV_OK) return rc;
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream, ev, kPhaseAll,
                   nullptr, 1, kTapeNone, nullptr, 0, 0, &a);
}

extern "C" int logkv_flush_chunk(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                 int32_t recent_count, const logkv_chunk_t* chunk, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  return flush_chunk(layout, state, flush_tokens, recent_count, chunk, workspace, workspace_bytes, stream, nullptr);
}

extern "C" int logkv_flush_chunk_profiled(const logkv_layout_t* layout, const logkv_state_t* state,
                                          int32_t flush_tokens, int32_t recent_count, const logkv_chunk_t* chunk,
                                          void* workspace, size_t workspace_bytes, void* stream, void** events,
                                          int32_t n_events) {
  if (!events || n_events < LOGKV_FLUSH_STAGES + 1) return LOGKV_E_POINTER;
  return flush_chunk(layout, state, flush_tokens, recent_count, chunk, workspace, workspace_bytes, stream,
                     reinterpret_cast<cudaEvent_t*>(events));
}

extern "C" int logkv_flush_oplog_append(const logkv_layout_t* layout, int32_t flush_tokens, void* workspace,
                                        int32_t* op_log, int32_t* op_log_len, int32_t capacity, void* stream) {
  const int v = validate(layout, flush_tokens);
  if (v != LOGKV_OK) return v;
  if (!workspace || !op_log || !op_log_len || capacity < 1) return LOGKV_E_POINTER;
  if ((reinterpret_cast<uintptr_t>(op_log) & 15) || (reinterpret_cast<uintptr_t>(op_log_len) & 3)) return LOGKV_E_POINTER;
  const Geo g = make_geo(*layout, flush_tokens, layout->recent_capacity);
  Work w{};
  carve(g, layout->dtype == LOGKV_DTYPE_BF16 ? 2 : 4, static_cast<char*>(workspace), &w);
  oplog_append_kernel<<<dim3(g.G, g.B), 256, 0, static_cast<cudaStream_t>(stream)>>>(g, w, op_log, op_log_len,
                                                                                   capacity);
  return (int)cudaGetLastError();
}

extern "C" int logkv_flush_scores(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                  int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream) {
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream, nullptr,
                   kPhaseScores);
}

extern "C" int logkv_flush_commit(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                  int32_t recent_count, void* workspace, size_t workspace_bytes,
                                  const float* partials_all, int32_t ranks, void* stream) {
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream, nullptr,
                   kPhaseCommit, partials_all, ranks);
}

extern "C" int logkv_flush_commit_strided(const logkv_layout_t* layout, const logkv_state_t* state,
                                          int32_t flush_tokens, int32_t recent_count, void* workspace,
                                          size_t workspace_bytes, const float* partials_all, int32_t ranks,
                                          int64_t rank_stride, void* stream) {
  if (rank_stride < 1) return LOGKV_E_SHAPE;
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream, nullptr,
                   kPhaseCommit, partials_all, ranks, kTapeNone, nullptr, 0, rank_stride);
}

extern "C" int logkv_flush_partials(const logkv_layout_t* layout, int32_t flush_tokens, void* workspace,
                                    float** partials, size_t* count) {
  const int v = validate(layout, flush_tokens);
  if (v != LOGKV_OK) return v;
  if (!workspace || !partials || !count) return LOGKV_E_POINTER;
  const Geo g = make_geo(*layout, flush_tokens, layout->recent_capacity);
  Work w{};
  carve(g, layout->dtype == LOGKV_DTYPE_BF16 ? 2 : 4, static_cast<char*>(workspace), &w);
  *partials = w.gpart;
  *count = (size_t)g.B * g.NC * g.G * 2;
  return LOGKV_OK;
}

extern "C" int logkv_flush_profiled(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                    int32_t recent_count, void* workspace, size_t workspace_bytes, void* stream,
                                    void** events, int32_t n_events) {
  if (!events || n_events < LOGKV_FLUSH_STAGES + 1) return LOGKV_E_POINTER;
  return run_flush(layout, state, flush_tokens, recent_count, workspace, workspace_bytes, stream,
                   reinterpret_cast<cudaEvent_t*>(events));
}

extern "C" int logkv_stream_capture_id(void* stream, unsigned long long* id) {
  if (!id) return LOGKV_E_POINTER;
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  unsigned long long cid = 0;
  const cudaError_t e = cudaStreamGetCaptureInfo(static_cast<cudaStream_t>(stream), &status, &cid);
  if (e != cudaSuccess) return (int)e;
  *id = status == cudaStreamCaptureStatusActive ? cid : 0ull;
  return LOGKV_OK;
}

// ---------------------------------------------------------------- allocation-free flush
// Callers that may not allocate device memory (a host whose allocator is
// locked after start-up, or a binding that cannot hand a device buffer over
// the C boundary) flush through one fixed scratch region compiled into this
// library instead of a caller-provided workspace.
namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;  // 32 MiB per GPU, held until process exit
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// The symbol name is only a host-side stand-in; its device address belongs to the CUDA context
// the library's module was loaded into.  Addresses are cached per context, keyed by the
// driver's context id (unique for the life of the process), so a context torn down and
// created again (cudaDeviceReset) gets a fresh lookup instead of a dangling address.
typedef int (*CtxGetCurrentFn)(void**);
typedef int (*CtxGetIdFn)(void*, unsigned long long*);
struct StaticSlot {
  unsigned long long ctx_id;
  void* ptr;
};
constexpr int kMaxContexts = 64;
std::mutex g_static_mutex;
StaticSlot g_static_slots[kMaxContexts] = {};
int g_static_next = 0;
CtxGetCurrentFn g_ctx_current = nullptr;
CtxGetIdFn g_ctx_id = nullptr;

// Id of the current context (called with g_static_mutex held).
int current_context_id(unsigned long long* id) {
  if (!g_ctx_current || !g_ctx_id) {
    void* f_cur = nullptr;
    void* f_id = nullptr;
    cudaDriverEntryPointQueryResult q_cur = cudaDriverEntryPointSymbolNotFound, q_id = q_cur;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f_cur, 12000, cudaEnableDefault, &q_cur);
    if (e != cudaSuccess) return (int)e;
    e = cudaGetDriverEntryPointByVersion("cuCtxGetId", &f_id, 12000, cudaEnableDefault, &q_id);
    if (e != cudaSuccess) return (int)e;
    if (q_cur != cudaDriverEntryPointSuccess || q_id != cudaDriverEntryPointSuccess || !f_cur || !f_id)
      return (int)cudaErrorSymbolNotFound;
    g_ctx_current = reinterpret_cast<CtxGetCurrentFn>(f_cur);
    g_ctx_id = reinterpret_cast<CtxGetIdFn>(f_id);
  }
  void* ctx = nullptr;
  if (g_ctx_current(&ctx) != 0 || !ctx) return (int)cudaErrorDeviceUninitialized;
  if (g_ctx_id(ctx, id) != 0) return (int)cudaErrorDeviceUninitialized;
  return LOGKV_OK;
}

// Device address of g_static_scratch on the current device.  When `owner` is given it must be
// device memory of that device (the cache state the flush works on): a state on another device
// is refused with LOGKV_E_DEVICE instead of flushing through the wrong GPU's scratch.
int static_scratch(const void* owner, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (owner) {
    cudaPointerAttributes attr{};
    e = cudaPointerGetAttributes(&attr, owner);
    if (e != cudaSuccess) return (int)e;
    if ((attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) || attr.device != dev)
      return LOGKV_E_DEVICE;
  }
  e = cudaSetDevice(dev);  // makes the device's primary context current (creating nothing else)
  if (e != cudaSuccess) return (int)e;
  std::lock_guard<std::mutex> lock(g_static_mutex);
  unsigned long long cid = 0;
  const int c = current_context_id(&cid);
  if (c != LOGKV_OK) return c;
  for (int i = 0; i < kMaxContexts; ++i)
    if (g_static_slots[i].ptr && g_static_slots[i].ctx_id == cid) {
      *out = g_static_slots[i].ptr;
      return LOGKV_OK;
    }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess) return (int)e;
  g_static_slots[g_static_next] = StaticSlot{cid, p};
  g_static_next = (g_static_next + 1) % kMaxContexts;
  *out = p;
  return LOGKV_OK;
}

}  // namespace

extern "C" int logkv_flush_static(const logkv_layout_t* layout, const logkv_state_t* state, int32_t flush_tokens,
                                  int32_t recent_count, void* stream) {
  const int v = validate(layout, flush_tokens);
  if (v != LOGKV_OK) return v;
  if (!state || !state->level_k) return LOGKV_E_POINTER;
  const size_t need = logkv_flush_workspace_bytes(layout, flush_tokens);
  if (need == 0 || need > kStaticScratchBytes) return LOGKV_E_WORKSPACE;
  void* scratch = nullptr;
  const int r = static_scratch(state->level_k, &scratch);
  if (r != LOGKV_OK) return r;
  // The status word and the row counters (first 512 bytes) must start at zero;
  // everything else in the scratch is written before it is read within a flush.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = cudaMemsetAsync(scratch, 0, 512, st);
  if (e != cudaSuccess) return (int)e;
  return run_flush(layout, state, flush_tokens, recent_count, scratch, kStaticScratchBytes, stream, nullptr);
}

extern "C" int logkv_read_status(const void* workspace, int32_t* out, void* stream) {
  if (!out) return LOGKV_E_POINTER;
  if (!workspace) {
    void* scratch = nullptr;
    const int r = static_scratch(nullptr, &scratch);
    if (r != LOGKV_OK) return r;
    workspace = scratch;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(out, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return (int)e;
}

extern "C" int logkv_read_ties(void* workspace, logkv_tie_t* out, int32_t cap, int64_t* total, int32_t clear,
                               void* stream) {
  if (!total || cap < 0 || (cap > 0 && !out)) return LOGKV_E_POINTER;
  if (!workspace) {
    void* scratch = nullptr;
    const int r = static_scratch(nullptr, &scratch);
    if (r != LOGKV_OK) return r;
    workspace = scratch;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* base = static_cast<char*>(workspace);
  unsigned long long* count = reinterpret_cast<unsigned long long*>(base + 256) + kCntTies;
  unsigned long long n = 0;
  cudaError_t e = cudaMemcpyAsync(&n, count, sizeof(n), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return (int)e;
  *total = (int64_t)n;
  const size_t keep = std::min<size_t>(std::min<size_t>((size_t)n, (size_t)kTieCap), (size_t)cap);
  if (keep) e = cudaMemcpyAsync(out, base + kTieOffset, keep * sizeof(TieEntry), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(count, 0, sizeof(unsigned long long), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return (int)e;
}

extern "C" int logkv_read_unified(const logkv_layout_t* layout, int32_t flush_tokens, const void* workspace,
                                  int32_t* out, int32_t n, void* stream) {
  const int v = validate(layout, flush_tokens);
  if (v != LOGKV_OK) return v;
  if (!workspace || !out || n < 1) return LOGKV_E_POINTER;
  if (layout->route != LOGKV_ROUTE_UNIFIED) return LOGKV_E_SHAPE;
  const Geo g = make_geo(*layout, flush_tokens, layout->recent_capacity);
  Work w{};
  carve(g, layout->dtype == LOGKV_DTYPE_BF16 ? 2 : 4, static_cast<char*>(const_cast<void*>(workspace)), &w);
  const size_t words = (size_t)g.B * g.G * kULaneWords;
  const size_t m = (size_t)n < words ? (size_t)n : words;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(out, w.u.words, m * sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return (int)e;
}

extern "C" int logkv_read_counters(const void* workspace, uint64_t* out, int32_t n, void* stream) {
  if (!out || n < 1) return LOGKV_E_POINTER;
  if (!workspace) {
    void* scratch = nullptr;
    const int r = static_scratch(nullptr, &scratch);
    if (r != LOGKV_OK) return r;
    workspace = scratch;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int m = n < kNumCounters ? n : kNumCounters;
  cudaError_t e = cudaMemcpyAsync(out, static_cast<const char*>(workspace) + 256, m * sizeof(uint64_t),
                                  cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return (int)e;
}
