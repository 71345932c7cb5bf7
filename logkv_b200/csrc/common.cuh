// Shared device helpers for the SemanticLogKV flush kernels (sm_100a).
//
// Numerics contract: every floating-point expression of the flush path is
// written with explicitly rounded intrinsics (__fmul_rn/__fadd_rn/__fsub_rn/
// __fdiv_rn) and the flush translation unit is built with -fmad=false, so no
// multiply-add is contracted.  Feature-axis reductions are left-to-right
// sums done by one thread, which is the canonical order the CPU oracle uses.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/logkv_b200.h"

namespace logkv {

constexpr int kMaxClusters = 32;
constexpr int kMaxLevels = 16;

// Status bits written by kernels into the workspace status word.
enum StatusBits : int32_t {
  kStatusCarryOverflow = 1,
  kStatusListOverflow = 2,
  kStatusCandidateOverflow = 4,
  kStatusBadCluster = 8,
  kStatusCopyTimeout = 16,   // a bounded wait for the kernel's own bulk copies gave up
};

__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

template <typename T> struct Elem;
template <> struct Elem<float> {
  __device__ __forceinline__ static float load(const float* p) { return *p; }
  __device__ __forceinline__ static void store(float* p, float v) { *p = v; }
  __device__ __forceinline__ static float round(float v) { return v; }
  __device__ __forceinline__ static float zero() { return 0.f; }
};
template <> struct Elem<__nv_bfloat16> {
  __device__ __forceinline__ static float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
  __device__ __forceinline__ static float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
  __device__ __forceinline__ static __nv_bfloat16 zero() { return __float2bfloat16_rn(0.f); }
};

// Programmatic dependent launch: wait until the preceding kernel of the stream has completed
// and its writes are visible (a no-op when the launch carries no programmatic dependency),
// then let the next kernel start launching while this one runs.
__device__ __forceinline__ void pdl_entry() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

__device__ __forceinline__ void set_status(int32_t* status, int32_t bit) {
  if (status) atomicOr(status, bit);
}

// Block-wide inclusive prefix sum of one int per thread (blockDim.x <= 1024, multiple of 32).
__device__ __forceinline__ int block_inclusive_scan(int v, int* warp_sums) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += y;
  }
  if (lane == 31) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int s = lane < nwarps ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= off) s += y;
    }
    if (lane < nwarps) warp_sums[lane] = s;
  }
  __syncthreads();
  int add = warp > 0 ? warp_sums[warp - 1] : 0;
  __syncthreads();
  return v + add;
}

}  // namespace logkv
