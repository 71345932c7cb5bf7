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
// The round itself (one thread-block cluster of kUCluster CTAs per lane) is unified_core.cuh's,
// shared with the flush-level route; here each launch runs one round of every lane.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/logkv_unified.h"
#include "unified_core.cuh"

namespace {

using namespace logkv_ward;
constexpr int kThreads = kUThreads;
constexpr int kCluster = kUCluster;
constexpr int kMaxSize = kUMaxSize;

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

// One lane of the operator-level state.
__device__ RunLane lane_of(const logkv_unified_t& u, int lane) {
  const size_t M = u.size;
  RunLane l;
  l.dist = u.dist + lane * M * M;
  l.mu = u.mu + lane * M * (size_t)u.dim;
  l.mass = u.mass + lane * M;
  l.radius = u.radius + lane * M;
  l.alive = u.alive + lane * M;
  l.packed = reinterpret_cast<long long*>(u.packed) + lane * M;
  l.restricted = nullptr;
  l.limit = u.limits ? u.limits + lane : nullptr;
  l.count = u.status + u.lanes + lane;
  l.active = u.status + lane;
  l.merges = u.merges + lane;
  l.stuck = u.stuck + lane;
  l.trace = u.trace + (size_t)lane * M * 2;
  l.M = (int)M;
  l.D = u.dim;
  l.target = u.target;
  l.passes = 1;
  l.cost_order = 1;
  l.pass = 0;
  l.ties = TieSink{nullptr, nullptr, nullptr, 0, 0, 0};
  return l;
}

// Every live row's minimum; the lane's rows are split over kCluster CTAs (row r goes to r % kCluster).
__global__ void __launch_bounds__(kThreads) init_kernel(logkv_unified_t u) {
  extern __shared__ int rows[];
  __shared__ int n;
  const int lane = blockIdx.x / kCluster, part = blockIdx.x % kCluster;
  const RunLane l = lane_of(u, lane);
  if (part == 0 && threadIdx.x == 0) {
    *l.active = 0;
    *l.merges = 0;
    *l.stuck = 0;
  }
  init_lane(l, part, kCluster, rows, &n);
}

// One round of one lane on a cluster of kCluster CTAs.
__global__ void __launch_bounds__(kThreads) round_kernel(logkv_unified_t u, int S) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ int act[2];
  cg::cluster_group cluster = cg::this_cluster();
  const RunLane l = lane_of(u, blockIdx.x / kCluster);
  run_round(cluster, l, smem_raw, S, act, 0);
}

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
  if (u->lanes < 1 || u->lanes > (1 << 24) || u->size < 1 || u->size > kMaxSize || u->dim < 1)
    return LOGKV_UNIFIED_E_SHAPE;
  return 0;
}

extern "C" int logkv_unified_init(const logkv_unified_t* u, void* stream) {
  const int v = check_unified(u);
  if (v) return v;
  init_kernel<<<u->lanes * kCluster, kThreads, (size_t)u->size * 4, static_cast<cudaStream_t>(stream)>>>(*u);
  return (int)cudaGetLastError();
}

extern "C" int logkv_unified_step(const logkv_unified_t* u, void* stream) {
  const int v = check_unified(u);
  if (v) return v;
  const int S = sort_width(u->size);   // at most size / 2 disjoint pairs are sorted
  const size_t smem = round_smem_bytes(u->size, S, kCluster);
  if (smem > 227 * 1024) return LOGKV_UNIFIED_E_SHAPE;
  if (smem > 48 * 1024) cudaFuncSetAttribute(round_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(u->lanes * kCluster);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, round_kernel, *u, S);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}
