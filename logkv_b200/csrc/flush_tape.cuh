// Update tape of one flush: what a replay needs to repeat the flush's state transition
// without routing.
//
// Follows the reference's update recording (_SemanticReplayUpdates and the record / replay
// branches of route_and_flush_batch, litgpt/log_kv_cache.py:111-137, :4946-5031): a replayed
// flush appends the recorded payload with the recorded decisions and Beta cuts and leaves the
// cache exactly as the recorded flush did; it never re-routes.  Here the record is a device
// buffer written by the flush itself:
//   payload   the flushed window rows (pre-RoPE K and V, [B,G,F,D]) as the recorded flush saw them
//   choice    kept and archived token indices and counts, the new span table (lengths, closed
//             flags, span count); the row counts and alpha_count follow from the kept counts
//   plan      per-cluster jobs (token lists, offsets, counts, kinds, scratch ranges, base orders)
//   cuts      the Beta cut of every 4-row group the cascade merged, per (lane, level, group)
//   unified route: the Ward merge jobs and counts, and the Beta cuts of their ladder rebuilds
#pragma once

#include "flush_common.cuh"

namespace logkv {

struct TapeView {
  void* pay_k;             // [B,G,F,D] T
  void* pay_v;
  int32_t* keep_idx;       // [B,P]
  int32_t* nkeep;          // [B]
  int32_t* arch_idx;       // [B,NW]
  int32_t* narch;          // [B]
  int32_t* span_len;       // [B,P]
  uint8_t* span_closed;    // [B,P]
  int32_t* nspans;         // [B]
  int32_t* tok_list;       // [B,G,NW]
  int32_t* plan_off;       // [B,G,K] each
  int32_t* plan_n;
  int32_t* plan_type;
  int32_t* plan_m0;
  int32_t* plan_scr;
  int64_t* plan_base;      // [B,G,K]
  uint8_t* cuts;           // [B,G,K,L,cut_stride]
  // Unified route only: the lane words (Ward merge counts), the Ward merge jobs and the Beta cuts
  // of the Ward merges' ladder rebuilds, per (b, g, merge).
  int32_t* uwords;         // [B,G,kULaneWords]
  int32_t* ward;           // [B,G,K,2]
  uint8_t* ward_cuts;      // [B,G,K,L,cut_stride]
};

// Beta groups a level can merge: its pool holds at most Bs stored rows plus its incoming rows,
// at most L * Bs re-inserted entries and NW tokens (a delayed lane re-appends everything).
__host__ __device__ inline int tape_cut_stride(const Geo& g) { return ((g.L + 1) * g.Bs + g.NW + 3) / 4; }

// Carves the tape (base may be null to size it); returns its size in bytes.
inline size_t tape_carve(const Geo& g, size_t esize, char* base, TapeView* t) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> void* {
    off = (off + 255) & ~size_t(255);
    void* p = base ? base + off : nullptr;
    off += bytes;
    return p;
  };
  const size_t B = g.B, G = g.G, K = g.K, P = g.P, NW = g.NW;
  t->pay_k = take(B * G * g.F * g.D * esize);
  t->pay_v = take(B * G * g.F * g.D * esize);
  t->keep_idx = static_cast<int32_t*>(take(B * P * 4));
  t->nkeep = static_cast<int32_t*>(take(B * 4));
  t->arch_idx = static_cast<int32_t*>(take(B * NW * 4));
  t->narch = static_cast<int32_t*>(take(B * 4));
  t->span_len = static_cast<int32_t*>(take(B * P * 4));
  t->span_closed = static_cast<uint8_t*>(take(B * P));
  t->nspans = static_cast<int32_t*>(take(B * 4));
  t->tok_list = static_cast<int32_t*>(take(B * G * NW * 4));
  t->plan_off = static_cast<int32_t*>(take(B * G * K * 4));
  t->plan_n = static_cast<int32_t*>(take(B * G * K * 4));
  t->plan_type = static_cast<int32_t*>(take(B * G * K * 4));
  t->plan_m0 = static_cast<int32_t*>(take(B * G * K * 4));
  t->plan_scr = static_cast<int32_t*>(take(B * G * K * 4));
  t->plan_base = static_cast<int64_t*>(take(B * G * K * 8));
  t->cuts = static_cast<uint8_t*>(take(B * G * K * (size_t)g.L * tape_cut_stride(g)));
  t->uwords = nullptr;
  t->ward = nullptr;
  t->ward_cuts = nullptr;
  if (g.route == LOGKV_ROUTE_UNIFIED) {
    t->uwords = static_cast<int32_t*>(take(B * G * kULaneWords * 4));
    t->ward = static_cast<int32_t*>(take(B * G * K * 2 * 4));
    t->ward_cuts = static_cast<uint8_t*>(take(B * G * K * (size_t)g.L * tape_cut_stride(g)));
  }
  return (off + 255) & ~size_t(255);
}

// Copies of up to kTapeSegs byte ranges in one launch (16-byte units when both ends and the
// length allow it).  Blocks stride over the segments' units.
constexpr int kTapeSegs = 20;
struct TapeSegs {
  const void* src[kTapeSegs];
  void* dst[kTapeSegs];
  size_t bytes[kTapeSegs];
  int n;
};

__global__ void tape_copy_kernel(TapeSegs segs) {
  pdl_entry();
  for (int i = 0; i < segs.n; ++i) {
    const char* src = static_cast<const char*>(segs.src[i]);
    char* dst = static_cast<char*>(segs.dst[i]);
    const size_t n = segs.bytes[i];
    const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | n) & 15) == 0;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    if (vec) {
      for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < n / 16; u += stride)
        reinterpret_cast<uint4*>(dst)[u] = reinterpret_cast<const uint4*>(src)[u];
    } else {
      for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < n; u += stride) dst[u] = src[u];
    }
  }
}

// The flushed window rows [0, F) of every (b, g) lane <-> the tape payload (16-byte units).
// to_tape = 1 saves the window's rows; 0 writes the recorded rows back into the window.
template <typename T>
__global__ void tape_payload_kernel(Geo g, logkv_state_t s, TapeView t, int to_tape) {
  pdl_entry();
  const int b = blockIdx.z, grp = blockIdx.y;
  const size_t lane = (size_t)b * g.G + grp;
  const size_t n = (size_t)g.F * g.D / Vec<T>::N;   // units per lane
  uint4* wk = reinterpret_cast<uint4*>(static_cast<T*>(s.recent_k_raw) + lane * g.cap2R * g.D);
  uint4* wv = reinterpret_cast<uint4*>(static_cast<T*>(s.recent_v) + lane * g.cap2R * g.D);
  uint4* tk = reinterpret_cast<uint4*>(static_cast<T*>(t.pay_k) + lane * g.F * g.D);
  uint4* tv = reinterpret_cast<uint4*>(static_cast<T*>(t.pay_v) + lane * g.F * g.D);
  for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < n; u += (size_t)gridDim.x * blockDim.x) {
    if (to_tape) {
      tk[u] = wk[u];
      tv[u] = wv[u];
    } else {
      wk[u] = tk[u];
      wv[u] = tv[u];
    }
  }
}

}  // namespace logkv
