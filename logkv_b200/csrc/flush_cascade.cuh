// Ladder cascade (K6b): one CTA per (batch, group, cluster) lane walks the
// levels; each overflowing level streams its pool through shared memory in
// tiles of kTileRows rows.  Tiles are double-buffered: while tile t is merged,
// tile t+1's K/V rows are already in flight (cp.async, 16 bytes per copy) and
// its metadata is loading into registers.
//
// Hazard-free in place: a tile is fully staged before any of its outputs are
// written, survivors land in slots below the tile's last row (all staged
// already), the prefetched tile lies above every slot written so far, and
// merged rows go to the other scratch buffer.
#pragma once

#include "flush_ladder.cuh"
#include "flush_tape.cuh"

namespace logkv {

constexpr int kTileRows = 64;                 // multiple of 4 (Beta groups never straddle tiles)
constexpr int kTileGroups = kTileRows / 4;


// Sum 16 per-lane values over the warp; every lane gets all 16 sums.  Transposed
// butterfly: each exchange halves the values a lane carries (16 shuffles), then one
// shuffle per value gathers the sums (lane 2k holds sum k).
__device__ __forceinline__ void warp_allreduce16(float* v, int lane) {
  const unsigned full = 0xffffffffu;
  float h8[8], h4[4], h2[2], h1;
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    h8[k] = (b4 ? v[k + 8] : v[k]) + __shfl_xor_sync(full, b4 ? v[k] : v[k + 8], 16);
#pragma unroll
  for (int k = 0; k < 4; ++k)
    h4[k] = (b3 ? h8[k + 4] : h8[k]) + __shfl_xor_sync(full, b3 ? h8[k] : h8[k + 4], 8);
#pragma unroll
  for (int k = 0; k < 2; ++k)
    h2[k] = (b2 ? h4[k + 2] : h4[k]) + __shfl_xor_sync(full, b2 ? h4[k] : h4[k + 2], 4);
  h1 = (b1 ? h2[1] : h2[0]) + __shfl_xor_sync(full, b1 ? h2[0] : h2[1], 2);
  h1 += __shfl_xor_sync(full, h1, 1);  // lane l now holds sum number l >> 1
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = __shfl_sync(full, h1, 2 * k);
}

// N consecutive elements of a staged row as floats (one vector load when N * sizeof(T) is
// 4, 8 or 16 bytes; the caller keeps the address aligned to that size).
template <typename T, int N>
__device__ __forceinline__ void load_run(const T* p, float* out) {
  constexpr int BYTES = N * (int)sizeof(T);
  if constexpr (BYTES == 16) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    unpack(u, out, (const T*)nullptr);
  } else if constexpr (BYTES == 8) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < N; ++j) out[j] = Elem<T>::load(e + j);
  } else if constexpr (BYTES == 4) {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < N; ++j) out[j] = Elem<T>::load(e + j);
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) out[j] = Elem<T>::load(p + j);
  }
}

// Beta cut of one group of four rows by one warp, certified against the canonical cost.
//
// The canonical cost (beta_log_kv.select_cuts, beta_log_kv.py:29-46) of cut c for one
// component: energy = max(sum_i w_i E_i / max(sum w, 1e-12), 1e-12) with E_i = sum_d x_id^2;
// per side, mean_d = (sum_i om_i x_id) / max(sum om, 1e-12) (om = w on the side, else 0),
// loss = sum_i om_i sum_d (x_id - mean_d)^2; cost_c += loss / energy over sides and
// components, argmin over cuts (2, 1, 3) with ties to the earlier.
//
// This warp uses the identity  sum_i w_i |x_i - m|^2 = (sum_{i<j} w_i w_j |x_i - x_j|^2) / W
// (m the weighted mean, W the side's mass): a side's loss from the pairwise squared
// distances D_ab of its rows (pairs 01, 02, 12, 13, 23 cover every side of the three cuts;
// single-row sides lose nothing).  Every term is non-negative, so the result is within a
// relative (D / 16 + 39) u of the exact cost (u = 2^-24: (D / 32 + 7) u for a distance or a
// row energy summed per lane and across lanes, 10 u for a side's products, sums and division,
// 11 u more for the energy and its reciprocal, 4 u for the cost's sum; the three divisions on
// a term's path are __fdividef, within 2 ulp = 4 u each, for denominators in [1e-12, 1e30]).
// The canonical evaluation is within (2 D + 25) u relative of the exact cost
// at its rounded means, and a mean rounded by delta changes a side's loss by only
// W |delta|^2 <= 36 u^2 W sum_i E_i (the mean minimises the loss).  So the returned cut is the
// canonical one whenever runner-up minus best exceeds 2 rel * runner-up with
// rel = (4 D + 128) u >= (2.0625 D + 64) u, the sum of both relative bounds, plus twice
// B = sum over components of 40 u^2 (sum w)(sum_i E_i) / energy, plus a floor for subnormal
// rounding.  Otherwise (a near tie), when a side's mass lies in (0, 1e-12) (the canonical
// clamp), or when a row energy exceeds 1e30 (no overflow anywhere below that), -1 asks for
// the canonical evaluation.
template <typename T, int DC>
__device__ int beta_cut_warp(const T* tk, const T* tv, const Meta* tm, int start, int Drt, int lane) {
  const int D = DC ? DC : Drt;
  constexpr int NPL = (DC >= 32 && DC % 32 == 0) ? DC / 32 : 0;  // consecutive features per lane
  float wv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) wv[i] = tm[start + i].w;
  // v[0..8]: K's E_0..E_3, D_01, D_02, D_12, D_13, D_23; v[9..15] + x[0..1]: the same for V.
  float v[16], x2[2];
#pragma unroll
  for (int comp = 0; comp < 2; ++comp) {
    const T* base = (comp == 0 ? tk : tv) + start * D;
    float e0 = 0.f, e1 = 0.f, e2 = 0.f, e3 = 0.f, p01 = 0.f, p02 = 0.f, p12 = 0.f, p13 = 0.f, p23 = 0.f;
    auto feature = [&](float a, float b, float c, float d) {
      e0 = __fmaf_rn(a, a, e0);
      e1 = __fmaf_rn(b, b, e1);
      e2 = __fmaf_rn(c, c, e2);
      e3 = __fmaf_rn(d, d, e3);
      float t;
      t = __fsub_rn(a, b); p01 = __fmaf_rn(t, t, p01);
      t = __fsub_rn(a, c); p02 = __fmaf_rn(t, t, p02);
      t = __fsub_rn(b, c); p12 = __fmaf_rn(t, t, p12);
      t = __fsub_rn(b, d); p13 = __fmaf_rn(t, t, p13);
      t = __fsub_rn(c, d); p23 = __fmaf_rn(t, t, p23);
    };
    if constexpr (NPL > 0) {
      float r0[NPL], r1[NPL], r2[NPL], r3[NPL];
      load_run<T, NPL>(base + NPL * lane, r0);
      load_run<T, NPL>(base + D + NPL * lane, r1);
      load_run<T, NPL>(base + 2 * D + NPL * lane, r2);
      load_run<T, NPL>(base + 3 * D + NPL * lane, r3);
#pragma unroll
      for (int j = 0; j < NPL; ++j) feature(r0[j], r1[j], r2[j], r3[j]);
    } else {
#pragma unroll 1
      for (int d = lane; d < D; d += 32)
        feature(Elem<T>::load(base + d), Elem<T>::load(base + D + d), Elem<T>::load(base + 2 * D + d),
                Elem<T>::load(base + 3 * D + d));
    }
    const float vals[9] = {e0, e1, e2, e3, p01, p02, p12, p13, p23};
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      const int idx = comp * 9 + k;
      if (idx < 16) v[idx] = vals[k];
      else x2[idx - 16] = vals[k];
    }
  }
  warp_allreduce16(v, lane);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    x2[0] += __shfl_xor_sync(0xffffffffu, x2[0], off);
    x2[1] += __shfl_xor_sync(0xffffffffu, x2[1], off);
  }
  const float w0 = wv[0], w1 = wv[1], w2 = wv[2], w3 = wv[3];
  const float wsum = fadd(fadd(fadd(w0, w1), w2), w3);
  const float tot = fmaxf(wsum, 1e-12f);
  const float m01 = fadd(w0, w1), m23 = fadd(w2, w3), m123 = fadd(fadd(w1, w2), w3), m012 = fadd(m01, w2);
  auto mass_ok = [](float m) { return m == 0.f || m >= 1e-12f; };
  bool ok = mass_ok(w0) && mass_ok(w3) && mass_ok(m01) && mass_ok(m23) && mass_ok(m123) && mass_ok(m012);
  const float w01 = fmul(w0, w1), w02 = fmul(w0, w2), w12 = fmul(w1, w2), w13 = fmul(w1, w3), w23 = fmul(w2, w3);
  float costs[3] = {0.f, 0.f, 0.f};
  float bound = 0.f;
#pragma unroll
  for (int comp = 0; comp < 2; ++comp) {
    const float E0 = v[comp * 9], E1 = v[comp * 9 + 1], E2 = v[comp * 9 + 2], E3 = v[comp * 9 + 3];
    const float P01 = v[comp * 9 + 4], P02 = v[comp * 9 + 5], P12 = v[comp * 9 + 6];
    const float P13 = comp == 0 ? v[7] : x2[0], P23 = comp == 0 ? v[8] : x2[1];
    const float esum = E0 + E1 + E2 + E3;
    ok = ok && esum <= 1e30f;  // also false for NaN
    // Denominators: tot, the side masses >= 1e-12 and energy in [1e-12, 1e30] (ok below).
    const float energy = fmaxf(__fdividef(fadd(fadd(fadd(fmul(E0, w0), fmul(E1, w1)), fmul(E2, w2)), fmul(E3, w3)),
                                          tot),
                               1e-12f);
    const float inv_e = __fdividef(1.f, energy);
    const float l2 = __fdividef(fmul(w01, P01), fmaxf(m01, 1e-12f));
    const float r2 = __fdividef(fmul(w23, P23), fmaxf(m23, 1e-12f));
    const float r1 = __fdividef(fadd(fadd(fmul(w12, P12), fmul(w13, P13)), fmul(w23, P23)), fmaxf(m123, 1e-12f));
    const float l3 = __fdividef(fadd(fadd(fmul(w01, P01), fmul(w02, P02)), fmul(w12, P12)), fmaxf(m012, 1e-12f));
    costs[0] = fadd(costs[0], fmul(fadd(l2, r2), inv_e));  // cut 2: rows 0,1 | 2,3
    costs[1] = fadd(costs[1], fmul(r1, inv_e));            // cut 1: row 0 | 1,2,3
    costs[2] = fadd(costs[2], fmul(l3, inv_e));            // cut 3: rows 0,1,2 | 3
    bound += 40.f * 3.5527137e-15f * wsum * esum * inv_e;  // 40 u^2 (sum w)(sum E) / energy
  }
  if (!ok) return -1;
  int best = 0;
  float bc = costs[0];
  if (costs[1] < bc) {
    best = 1;
    bc = costs[1];
  }
  if (costs[2] < bc) {
    best = 2;
    bc = costs[2];
  }
  const float second = best == 0 ? fminf(costs[1], costs[2]) : (best == 1 ? fminf(costs[0], costs[2])
                                                                          : fminf(costs[0], costs[1]));
  const float rel = (4.f * D + 128.f) * 5.9604645e-8f;
  const float margin = 2.f * rel * second + 2.f * bound + 1e-25f * (1.f + wsum);
  if (!(second - bc > margin)) return -1;  // near tie (or NaN): canonical evaluation
  return best == 0 ? 2 : (best == 1 ? 1 : 3);
}

// Merges of pool rows [t0, mend) of level `ell` (staged in shared memory as rows 0.. of tk / tv /
// tm) into merged rows t0 / 2 + j of scratch buffer `out_buf`, counted from row `out_off` of the
// lane's range: pairwise count-weighted merges, or Beta 4->2 cuts (certified warp cut, canonical
// order on near ties, recorded / replayed cuts under an update tape).  Called by the whole block.
template <typename T, bool BETA, int DC>
__device__ void merge_tile(const LaneCtx<T>& x, const Geo& g, const Work& w, const T* tk, const T* tv,
                           const Meta* tm, int t0, int mend, int npair, int ell, int out_buf, int out_off,
                           float (*bloss)[12], float (*bener)[2], int* bcut, int* sh_exact) {
  constexpr int VN = Vec<T>::N;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int D = DC ? DC : g.D, DV = D / VN;
  T* SK = static_cast<T*>(w.sk);
  T* SV = static_cast<T*>(w.sv);
    if (!BETA) {
      const int j0 = t0 / 2, jn = (mend - t0) / 2;
      for (int item = tid; item < jn * DV * 2; item += nt) {
        const int j = item / (2 * DV), f = (item / DV) & 1, v = item % DV;
        const int ra = 2 * j, rb = 2 * j + 1;
        const float wa = tm[ra].w, wb = tm[rb].w;
        const float alpha = fdiv(wa, fmaxf(fadd(wa, wb), 1e-8f));
        const float beta = fsub(1.f, alpha);
        const T* base = f ? tv : tk;
        float a[VN], b[VN], o[VN];
        unpack(*reinterpret_cast<const uint4*>(base + ra * D + v * VN), a, (const T*)nullptr);
        unpack(*reinterpret_cast<const uint4*>(base + rb * D + v * VN), b, (const T*)nullptr);
#pragma unroll
        for (int e = 0; e < VN; ++e) o[e] = fadd(fmul(alpha, a[e]), fmul(beta, b[e]));
        *reinterpret_cast<uint4*>((f ? SV : SK) + x.scr_row(out_buf, out_off + j0 + j) * D + v * VN) = pack(o, (const T*)nullptr);
      }
      for (int j = tid; j < jn; j += nt) x.put_scratch(out_buf, out_off + j0 + j, merge_meta(tm[2 * j], tm[2 * j + 1]));
    } else {
      const int qn = (mend - t0 + 3) / 4;  // groups of this tile (tile rows 4q..4q+3)
      // Recorded cuts of this (lane, level, tile): written when recording, read when replaying.
      uint8_t* tcut = g.tape != kTapeNone
                          ? w.tape_cuts + ((size_t)(w.tape_cut_lane >= 0 ? w.tape_cut_lane : (long long)x.lane) * g.L + ell) * tape_cut_stride(g) + t0 / 4
                          : nullptr;
      if (g.tape == kTapeReplay) {
        for (int q = tid; q < qn; q += nt) bcut[q] = tcut[q];
        __syncthreads();
      } else {
      // Certified warp-parallel cut per group; near ties fall back to the canonical order below.
      const int warp = tid >> 5, lane = tid & 31, nwarps = nt >> 5;
      for (int q = warp; q < qn; q += nwarps) {
        const int width = min(4, npair - (t0 + 4 * q));
        const int cut = width == 4 ? beta_cut_warp<T, DC>(tk, tv, tm, 4 * q, D, lane) : 1;
        if (lane == 0) {
          bcut[q] = cut;
          if (cut < 0) atomicAdd(sh_exact, 1);
        }
      }
      __syncthreads();
      if (*sh_exact) {
      for (int item = tid; item < qn * 14; item += nt) {
        const int q = item / 14, k = item % 14;
        const int start = 4 * q;
        const int width = min(4, npair - (t0 + start));
        if (width != 4 || bcut[q] >= 0) continue;
        float wv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) wv[i] = tm[start + i].w;
        const int comp = k < 12 ? k / 6 : k - 12;
        const T* base = comp == 0 ? tk : tv;
        if (k >= 12) {
          float e[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
          for (int d = 0; d < D; ++d)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float xv = Elem<T>::load(base + (start + i) * D + d);
              e[i] = fadd(e[i], fmul(xv, xv));
            }
          float tot = 0.f, acc = 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) tot = fadd(tot, wv[i]);
          tot = fmaxf(tot, 1e-12f);
#pragma unroll
          for (int i = 0; i < 4; ++i) acc = fadd(acc, fmul(e[i], wv[i]));
          bener[q][comp] = fmaxf(fdiv(acc, tot), 1e-12f);
        } else {
          const int j = (k % 6) / 2, side = k % 2;
          const int cut = j == 0 ? 2 : (j == 1 ? 1 : 3);
          float om[4];
          float ws = 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const bool in = side == 0 ? (i < cut) : (i >= cut);
            om[i] = fmul(wv[i], in ? 1.f : 0.f);
            ws = fadd(ws, om[i]);
          }
          const float den = fmaxf(ws, 1e-12f);
          float r[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
          for (int d = 0; d < D; ++d) {
            float xv[4];
            float sacc = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              xv[i] = Elem<T>::load(base + (start + i) * D + d);
              sacc = fadd(sacc, fmul(xv[i], om[i]));
            }
            const float mean = fdiv(sacc, den);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float df = fsub(xv[i], mean);
              r[i] = fadd(r[i], fmul(df, df));
            }
          }
          float loss = 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) loss = fadd(loss, fmul(r[i], om[i]));
          bloss[q][k] = loss;
        }
      }
      __syncthreads();
      for (int q = tid; q < qn; q += nt) {
        if (bcut[q] >= 0) continue;
        float costs[3] = {0.f, 0.f, 0.f};
        for (int comp = 0; comp < 2; ++comp)
          for (int j = 0; j < 3; ++j)
            for (int side = 0; side < 2; ++side)
              costs[j] = fadd(costs[j], fdiv(bloss[q][comp * 6 + j * 2 + side], bener[q][comp]));
        int best = 0;
        if (costs[1] < costs[best]) best = 1;
        if (costs[2] < costs[best]) best = 2;
        bcut[q] = best == 0 ? 2 : (best == 1 ? 1 : 3);
        // Runner-up (earlier cut on equal costs) for the near-tie log.
        const int r = best == 0 ? (costs[2] < costs[1] ? 2 : 1) : (best == 1 ? (costs[2] < costs[0] ? 2 : 0)
                                                                              : (costs[1] < costs[0] ? 1 : 0));
        if (near_tie(costs[best], costs[r]))
          log_tie(w, LOGKV_TIE_BETA_CUT, x.b, x.grp, x.c, ell * 65536 + (t0 + 4 * q) / 4, bcut[q],
                  r == 0 ? 2 : (r == 1 ? 1 : 3), rel_gap(costs[best], costs[r]), costs[best]);
      }
      __syncthreads();
      if (tid == 0) {
        atomicAdd(&w.counters[kCntExactCuts], (unsigned long long)*sh_exact);
        *sh_exact = 0;
      }
      }
      if (g.tape == kTapeRecord)
        for (int q = tid; q < qn; q += nt) tcut[q] = (uint8_t)bcut[q];
      }
      // Apply: per output side, sum over member rows (row order) of w*x / max(mass, 1e-12).
      // One item computes both sides of a (group, component, 16-byte column) from one load
      // of each member row; each side keeps its own products (x * 0 for rows of the other
      // side) and sums in row order.  Groups are 4 rows wide, or 2 (the tail: one side).
      for (int item = tid; item < qn * 2 * DV; item += nt) {
        const int q = item / (2 * DV), f = (item / DV) & 1, v = item % DV;
        const int start = 4 * q;
        const int width = min(4, npair - (t0 + start));
        const bool two = width == 4;
        const int cut = bcut[q];
        const T* base = f ? tv : tk;
        float acc0[VN], acc1[VN], mass0 = 0.f, mass1 = 0.f;
#pragma unroll
        for (int e = 0; e < VN; ++e) acc0[e] = acc1[e] = 0.f;
        for (int i = 0; i < 4; ++i) {
          const bool valid = i < width;
          const bool in0 = valid && (!two || i < cut), in1 = valid && two && i >= cut;
          const float wi = valid ? tm[start + i].w : 0.f;
          const float om0 = fmul(wi, in0 ? 1.f : 0.f), om1 = fmul(wi, in1 ? 1.f : 0.f);
          float xr[VN];
          if (valid) {
            unpack(*reinterpret_cast<const uint4*>(base + (start + i) * D + v * VN), xr, (const T*)nullptr);
          } else {
#pragma unroll
            for (int e = 0; e < VN; ++e) xr[e] = 0.f;
          }
          mass0 = fadd(mass0, om0);
          mass1 = fadd(mass1, om1);
#pragma unroll
          for (int e = 0; e < VN; ++e) {
            acc0[e] = fadd(acc0[e], fmul(xr[e], om0));
            acc1[e] = fadd(acc1[e], fmul(xr[e], om1));
          }
        }
        const float den0 = fmaxf(mass0, 1e-12f);
#pragma unroll
        for (int e = 0; e < VN; ++e) acc0[e] = fdiv(acc0[e], den0);
        const int outrow = (t0 + start) / 2;
        *reinterpret_cast<uint4*>((f ? SV : SK) + x.scr_row(out_buf, out_off + outrow) * D + v * VN) = pack(acc0, (const T*)nullptr);
        if (two) {
          const float den1 = fmaxf(mass1, 1e-12f);
#pragma unroll
          for (int e = 0; e < VN; ++e) acc1[e] = fdiv(acc1[e], den1);
          *reinterpret_cast<uint4*>((f ? SV : SK) + x.scr_row(out_buf, out_off + outrow + 1) * D + v * VN) =
              pack(acc1, (const T*)nullptr);
        }
      }
      for (int item = tid; item < qn * 2; item += nt) {
        const int q = item / 2, side = item % 2;
        const int start = 4 * q;
        const int width = min(4, npair - (t0 + start));
        if (side == 1 && width != 4) continue;
        const int cut = bcut[q];
        float mass = 0.f;
        int64_t lo = INT64_MAX, hi = INT64_MIN, swp = 0, ord = INT64_MAX;
        uint8_t pad = 1;
        for (int i = 0; i < width; ++i) {
          const bool in = width == 2 ? side == 0 : (side == 0 ? i < cut : i >= cut);
          const Meta& r = tm[start + i];
          mass = fadd(mass, fmul(r.w, in ? 1.f : 0.f));
          if (!in) continue;
          if (r.w > 0.f) {
            lo = min(lo, r.lo);
            hi = max(hi, r.hi);
          }
          swp += r.swp;
          ord = min(ord, r.ord);
          pad &= r.pad;
        }
        x.put_scratch(out_buf, out_off + (t0 + start) / 2 + side,
                      Meta{mass, mass > 0.f ? lo : 0, mass > 0.f ? hi : 0, swp, ord, pad});
      }
    }
}

constexpr int kCascadeThreads = 256;  // two CTAs per SM (registers and shared memory)

// Sequential level walk of one lane by the whole block: every level in order, each overflowing
// level's pool streamed through double-buffered tiles of TILE rows (dynamic shared memory of
// walk_smem(g, esize, TILE) bytes).
template <typename T, bool BETA, int DC, int TILE>
__device__ void cascade_walk(const LaneCtx<T>& x, const Geo& g, const logkv_state_t& s, const Work& w) {
  static_assert(TILE % 4 == 0, "Beta groups never straddle tiles");
  const int type = w.plan_type[x.lane];
  constexpr int VN = Vec<T>::N;
  const int tid = threadIdx.x, nt = blockDim.x, Bs = g.Bs;
  // Compile-time head dim when DC != 0: every row/vector index map becomes shifts.
  const int D = DC ? DC : g.D, DV = D / VN;
  extern __shared__ uint4 smem4[];
  T* tkb = reinterpret_cast<T*>(smem4);                                 // [2][TILE][D]
  T* tvb = tkb + 2 * (size_t)TILE * D;                             // [2][TILE][D]
  Meta* tmb = reinterpret_cast<Meta*>(tvb + 2 * (size_t)TILE * D);  // [2][TILE]
  int64_t* tpos = reinterpret_cast<int64_t*>(tmb + 2 * TILE);      // [NW] token positions
  int* srcs = reinterpret_cast<int*>(tpos + g.NW);                      // [NW] token sources
  __shared__ float bloss[(TILE / 4)][12];
  __shared__ float bener[(TILE / 4)][2];
  __shared__ int bcut[(TILE / 4)];
  __shared__ int sh_exact;  // groups of the current tile needing the canonical cost order
  __shared__ const T* rowp[2][2][TILE];  // [tile buffer][K, V][row] source rows of staged tiles
  if (threadIdx.x == 0) sh_exact = 0;
  T* LK = static_cast<T*>(s.level_k);
  T* LV = static_cast<T*>(s.level_v);
  T* SK = static_cast<T*>(w.sk);
  T* SV = static_cast<T*>(w.sv);
  const int ntok = type == kJobLate ? 0 : w.plan_n[x.lane];
  for (int i = tid; i < ntok; i += nt) {
    const int src = x.arch[x.toks[x.toff + i]];
    srcs[i] = src;
    tpos[i] = token_position(g, s, w, x.b, src);
  }
  __syncthreads();
  Stage st;
  st.kind = type == kJobLate ? 1 : 0;
  st.buf = 0;
  st.m = w.plan_m0[x.lane];
  int nb = 1;
  // Incoming rows: tokens through the source table, else scratch rows.
  auto stage_k = [&](int i) -> const T* {
    if (st.kind == 0) return token_row<T>(g, x.snapk, x.reck, x.b, x.grp, srcs[i]);
    return SK + x.scr_row(st.buf, i) * D;
  };
  auto stage_v = [&](int i) -> const T* {
    if (st.kind == 0) return token_row<T>(g, x.snapv, x.recv, x.b, x.grp, srcs[i]);
    return SV + x.scr_row(st.buf, i) * D;
  };
  auto stage_meta = [&](int i) -> Meta {
    if (st.kind == 0) {
      const int64_t p = tpos[i];
      return Meta{1.f, p, p, p, x.base_order + i, 0};
    }
    const size_t r = x.scr_row(st.buf, i);
    return Meta{w.sw[r], w.slo[r], w.shi[r], w.sswp[r], w.sord[r], w.spad[r]};
  };
  for (int ell = 0; ell < g.L; ++ell) {
    const int m = st.m;
    if (m == 0) break;
    const int cnt = s.level_count[x.lane * g.L + ell];
    const size_t lrow0 = x.level_row(ell, 0);
    auto pool_k = [&](int p) -> const T* { return p < cnt ? LK + (lrow0 + p) * D : stage_k(p - cnt); };
    auto pool_v = [&](int p) -> const T* { return p < cnt ? LV + (lrow0 + p) * D : stage_v(p - cnt); };
    auto pool_m = [&](int p) -> Meta {
      if (p < cnt) {
        const size_t r = lrow0 + p;
        return Meta{s.level_w[r], s.level_p_lo[r], s.level_p_hi[r], s.level_sum_wp[r], s.level_order[r],
                    s.pad_mask[r]};
      }
      return stage_meta(p - cnt);
    };
    if (cnt + m <= Bs) {
      // Fill: incoming rows become slots cnt.. (already in the storage dtype).
      for (int item = tid; item < m * DV * 2; item += nt) {
        const int i = item / (2 * DV), f = (item / DV) & 1, v = item % DV;
        const T* src = (f ? stage_v(i) : stage_k(i)) + v * VN;
        T* dst = (f ? LV : LK) + (lrow0 + cnt + i) * D + v * VN;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
      }
      for (int i = tid; i < m; i += nt) x.put_level_meta(lrow0 + cnt + i, stage_meta(i));
      if (tid == 0) {
        s.level_count[x.lane * g.L + ell] = (int16_t)(cnt + m);
        atomicAdd(&w.counters[kCntStageRead], (unsigned long long)m);
        atomicAdd(&w.counters[kCntFill], (unsigned long long)m);
      }
      break;
    }
    const int rem = cnt + m - Bs;
    if (ell == g.L - 1) {
      // Saturated top level (rare): slot 0 = left fold of pool[0..rem], rounded each step;
      // slots 1.. = pool[rem+1..].  Staged through tile buffer 0 (row 0 holds the fold).
      T* tk = tkb;
      T* tv = tvb;
      Meta* tm = tmb;
      for (int d = tid; d < D; d += nt) {
        float ak = Elem<T>::load(pool_k(0) + d), av = Elem<T>::load(pool_v(0) + d);
        float aw = pool_m(0).w;
        for (int t = 1; t <= rem; ++t) {
          const float bw = pool_m(t).w;
          const float alpha = fdiv(aw, fmaxf(fadd(aw, bw), 1e-8f));
          const float beta = fsub(1.f, alpha);
          ak = Elem<T>::round(fadd(fmul(alpha, ak), fmul(beta, Elem<T>::load(pool_k(t) + d))));
          av = Elem<T>::round(fadd(fmul(alpha, av), fmul(beta, Elem<T>::load(pool_v(t) + d))));
          aw = fadd(aw, bw);
        }
        Elem<T>::store(tk + d, ak);
        Elem<T>::store(tv + d, av);
      }
      if (tid == 0) {
        Meta acc = pool_m(0);
        for (int t = 1; t <= rem; ++t) acc = merge_meta(acc, pool_m(t));
        tm[0] = acc;
      }
      __syncthreads();
      // Shift: slot j (1 <= j < Bs) <- pool[rem + j]; sources lie above the written slots.
      for (int j0 = 1; j0 < Bs; j0 += TILE - 1) {
        const int jn = min(TILE - 1, Bs - j0);
        for (int item = tid; item < jn * D; item += nt) {
          const int r = item / D, d = item % D;
          tk[(1 + r) * D + d] = pool_k(rem + j0 + r)[d];
          tv[(1 + r) * D + d] = pool_v(rem + j0 + r)[d];
        }
        for (int r = tid; r < jn; r += nt) tm[1 + r] = pool_m(rem + j0 + r);
        __syncthreads();
        for (int item = tid; item < jn * D; item += nt) {
          const int r = item / D, d = item % D;
          LK[(lrow0 + j0 + r) * D + d] = tk[(1 + r) * D + d];
          LV[(lrow0 + j0 + r) * D + d] = tv[(1 + r) * D + d];
        }
        for (int r = tid; r < jn; r += nt) x.put_level_meta(lrow0 + j0 + r, tm[1 + r]);
        __syncthreads();
      }
      for (int d = tid; d < D; d += nt) {
        LK[lrow0 * D + d] = tk[d];
        LV[lrow0 * D + d] = tv[d];
      }
      if (tid == 0) {
        x.put_level_meta(lrow0, tm[0]);
        s.level_count[x.lane * g.L + ell] = (int16_t)Bs;
        atomicAdd(&w.counters[kCntStorageRead], (unsigned long long)cnt);
        atomicAdd(&w.counters[kCntStageRead], (unsigned long long)m);
        atomicAdd(&w.counters[kCntSurvivor], (unsigned long long)Bs);
      }
      break;
    }
    const int npair = 2 * ((rem + 1) / 2);
    const int ncarry = npair / 2;
    const int nsurv = cnt + m - npair;
    const int total = cnt + m;
    // Issue the asynchronous K/V copies of the tile starting at pool row t0 into buffer `buf`;
    // the calling thread's metadata row (if any) is returned through `pend`.
    Meta pend{};
    // Every row's source pointers are resolved once (one thread per row) into rowp[buf] before
    // a barrier that precedes the tile's issue, so a 16-byte copy costs an offset, not the
    // pool / token / scratch address arithmetic.  Tile t0 uses buffer (t0 / TILE) & 1.
    auto resolve = [&](int t0, int buf) {
      const int tn = min(TILE, total - t0);
      if (tid < tn) {
        rowp[buf][0][tid] = pool_k(t0 + tid);
        rowp[buf][1][tid] = pool_v(t0 + tid);
      }
    };
    auto issue = [&](int t0, int buf) {
      const int tn = min(TILE, total - t0);
      T* tk = tkb + (size_t)buf * TILE * D;
      T* tv = tvb + (size_t)buf * TILE * D;
      for (int item = tid; item < tn * DV * 2; item += nt) {
        const int r = item / (2 * DV), f = (item / DV) & 1, v = item % DV;
        cp_async16((f ? tv : tk) + r * D + v * VN, rowp[buf][f][r] + v * VN);
      }
      cp_async_commit();
      if (tid < tn) pend = pool_m(t0 + tid);
    };
    resolve(0, 0);
    if (TILE < total) resolve(TILE, 1);
    __syncthreads();
    issue(0, 0);
    int cur = 0;
    for (int t0 = 0; t0 < total; t0 += TILE) {
      const int tn = min(TILE, total - t0);
      T* tk = tkb + (size_t)cur * TILE * D;
      T* tv = tvb + (size_t)cur * TILE * D;
      Meta* tm = tmb + cur * TILE;
      cp_async_wait_all();
      if (tid < tn) tm[tid] = pend;
      __syncthreads();
      if (t0 + TILE < total) issue(t0 + TILE, cur ^ 1);
      // Buffer `cur` was last read by this tile's issue, before the barrier above; the next
      // reader (tile t0 + 2 tiles) issues after the next iteration's barrier.
      if (t0 + 2 * TILE < total) resolve(t0 + 2 * TILE, cur);
      const int mend = min(t0 + tn, npair);  // merge rows of this tile: [t0, mend)
      if (mend > t0)
        merge_tile<T, BETA, DC>(x, g, w, tk, tv, tm, t0, mend, npair, ell, nb, 0, bloss, bener, bcut, &sh_exact);
      // Survivors of this tile: pool row p >= npair -> slot p - npair.
      const int sbeg = max(t0, npair);
      const int sn = t0 + tn - sbeg;
      if (sn > 0) {
        for (int item = tid; item < sn * DV * 2; item += nt) {
          const int r = item / (2 * DV), f = (item / DV) & 1, v = item % DV;
          const int p = sbeg + r;
          *reinterpret_cast<uint4*>((f ? LV : LK) + (lrow0 + p - npair) * D + v * VN) =
              *reinterpret_cast<const uint4*>((f ? tv : tk) + (p - t0) * D + v * VN);
        }
        for (int r = tid; r < sn; r += nt) x.put_level_meta(lrow0 + sbeg + r - npair, tm[sbeg + r - t0]);
      }
      __syncthreads();
      cur ^= 1;
    }
    // Tail slots are zeroed.
    const int nclr = Bs - nsurv;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    for (int item = tid; item < nclr * DV * 2; item += nt) {
      const int r = item / (2 * DV), f = (item / DV) & 1, v = item % DV;
      *reinterpret_cast<uint4*>((f ? LV : LK) + (lrow0 + nsurv + r) * D + v * VN) = zero;
    }
    for (int r = tid; r < nclr; r += nt) x.put_level_meta(lrow0 + nsurv + r, Meta{0.f, 0, 0, 0, 0, 0});
    if (tid == 0) {
      s.level_count[x.lane * g.L + ell] = (int16_t)nsurv;
      atomicAdd(&w.counters[kCntStorageRead], (unsigned long long)cnt);
      atomicAdd(&w.counters[kCntStageRead], (unsigned long long)m);
      atomicAdd(&w.counters[kCntSurvivor], (unsigned long long)nsurv);
      atomicAdd(&w.counters[kCntClear], (unsigned long long)nclr);
      atomicAdd(&w.counters[kCntCarry], (unsigned long long)ncarry);
    }
    __syncthreads();
    st.kind = 1;
    st.buf = nb;
    st.m = ncarry;
    nb = 1 - nb;
  }
}

inline size_t walk_smem(const Geo& g, size_t esize, int tile) {
  // two K/V tile buffers, two metadata tiles, token positions and sources
  return 4 * (size_t)tile * g.D * esize + 2 * (size_t)tile * sizeof(Meta) + (size_t)g.NW * (sizeof(int64_t) + sizeof(int)) +
         16;
}

// The sequential walk as its own kernel, one CTA per lane (used when the parallel cascade is off).
template <typename T, bool BETA, int DC>
__global__ void __launch_bounds__(kCascadeThreads, 2) cascade_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  const LaneCtx<T> x = make_ctx<T>(g, s, w);
  if (w.plan_type[x.lane] == kJobNone) return;
  cascade_walk<T, BETA, DC, kTileRows>(x, g, s, w);
}

// ---------------------------------------------------------------- parallel cascade
// What every level of one lane does in this flush, from its counts and the lane's incoming row
// count: the sequential walk's control flow without touching a row.  In the steady state every
// level's merges read only that level's stored rows (level 0 also its incoming tokens), so the
// merges of all levels run at once (cascade_merge_kernel: carries of level l land in scratch
// buffer 1 as level l + 1's incoming rows) and then every level moves its survivors
// (cascade_move_kernel).  A level >= 1 whose merges would read incoming rows (carries of the
// level below) and the top level's fold need the levels in order: such lanes take the
// sequential walk.
// Block-wide: the lane's plan (written by the prepare kernel) into lp, its mode returned to every
// thread.  L2-coherent loads: the move kernel reads the plan before its grid dependency wait.
__device__ int plan_lane(const Geo& g, const Work& w, size_t lane, LevelPlan* lp) {
  __shared__ int sh_mode;
  const int tid = threadIdx.x;
  if (tid < g.L) {
    const int* src = reinterpret_cast<const int*>(w.lane_plan + lane * g.L + tid);
    lp[tid] = LevelPlan{__ldcg(src), __ldcg(src + 1), __ldcg(src + 2), __ldcg(src + 3), __ldcg(src + 4),
                        __ldcg(src + 5)};
  }
  if (tid == 32) sh_mode = __ldcg(w.lane_mode + lane);
  __syncthreads();
  return sh_mode;
}

// Source rows and metadata of pool row p of level l: a stored slot (p < cnt), else incoming row
// p - cnt: the lane's tokens (level 0, ordinary / new jobs), its staged re-inserts (level 0,
// delayed jobs: scratch buffer 0) or the carries of level l - 1 (scratch buffer 1).
template <typename T>
struct PoolRow {
  const T* k;
  const T* v;
  Meta m;
};
template <typename T>
__device__ PoolRow<T> pool_row(const LaneCtx<T>& x, const LevelPlan& p, int l, int row, bool late) {
  const Geo& g = x.g;
  if (row < p.cnt) {
    const size_t r = x.level_row(l, row);
    return PoolRow<T>{static_cast<const T*>(x.s.level_k) + r * g.D, static_cast<const T*>(x.s.level_v) + r * g.D,
                      Meta{x.s.level_w[r], x.s.level_p_lo[r], x.s.level_p_hi[r], x.s.level_sum_wp[r],
                           x.s.level_order[r], x.s.pad_mask[r]}};
  }
  const int i = row - p.cnt;
  Stage st{late || l > 0 ? 1 : 0, l > 0 ? 1 : 0, p.m};
  const int si = l > 0 ? p.in_off + i : i;
  return PoolRow<T>{x.stage_k(st, si), x.stage_v(st, si), st.kind == 0 ? x.stage_meta(st, i) : x.stage_meta(st, si)};
}

// Canonical-order cut of one 4-row group by one warp (the near-tie fallback of beta_cut_warp):
// lanes 0..11 each sum one (component, cut, side) loss, lanes 12..13 one component's energy, in
// the reference's order (beta_log_kv.select_cuts); the costs are then added comp-major as there.
// Returns the cut (2, 1 or 3); *best / *second / *second_cut describe the argmin for the tie log.
template <typename T, int DC>
__device__ int beta_cut_canonical_warp(const T* gk, const T* gv, const Meta* gm, int Drt, int lane, float* best_cost,
                                       float* second_cost, int* second_cut) {
  const int D = DC ? DC : Drt;
  float wv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) wv[i] = gm[i].w;
  float val = 0.f;
  if (lane < 14) {
    const int k = lane;
    const int comp = k < 12 ? k / 6 : k - 12;
    const T* base = comp == 0 ? gk : gv;
    if (k >= 12) {
      float e[4] = {0.f, 0.f, 0.f, 0.f};
      for (int d = 0; d < D; ++d)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float xv = Elem<T>::load(base + i * D + d);
          e[i] = fadd(e[i], fmul(xv, xv));
        }
      float tot = 0.f, acc = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) tot = fadd(tot, wv[i]);
      tot = fmaxf(tot, 1e-12f);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc = fadd(acc, fmul(e[i], wv[i]));
      val = fmaxf(fdiv(acc, tot), 1e-12f);
    } else {
      const int j = (k % 6) / 2, side = k % 2;
      const int cut = j == 0 ? 2 : (j == 1 ? 1 : 3);
      float om[4];
      float ws = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const bool in = side == 0 ? (i < cut) : (i >= cut);
        om[i] = fmul(wv[i], in ? 1.f : 0.f);
        ws = fadd(ws, om[i]);
      }
      const float den = fmaxf(ws, 1e-12f);
      float r[4] = {0.f, 0.f, 0.f, 0.f};
      for (int d = 0; d < D; ++d) {
        float xv[4];
        float sacc = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xv[i] = Elem<T>::load(base + i * D + d);
          sacc = fadd(sacc, fmul(xv[i], om[i]));
        }
        const float mean = fdiv(sacc, den);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float df = fsub(xv[i], mean);
          r[i] = fadd(r[i], fmul(df, df));
        }
      }
      float loss = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) loss = fadd(loss, fmul(r[i], om[i]));
      val = loss;
    }
  }
  float loss[12], ener[2];
#pragma unroll
  for (int k = 0; k < 12; ++k) loss[k] = __shfl_sync(0xffffffffu, val, k);
  ener[0] = __shfl_sync(0xffffffffu, val, 12);
  ener[1] = __shfl_sync(0xffffffffu, val, 13);
  float costs[3] = {0.f, 0.f, 0.f};
#pragma unroll
  for (int comp = 0; comp < 2; ++comp)
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int side = 0; side < 2; ++side) costs[j] = fadd(costs[j], fdiv(loss[comp * 6 + j * 2 + side], ener[comp]));
  int best = 0;
  if (costs[1] < costs[best]) best = 1;
  if (costs[2] < costs[best]) best = 2;
  const int r = best == 0 ? (costs[2] < costs[1] ? 2 : 1) : (best == 1 ? (costs[2] < costs[0] ? 2 : 0)
                                                                        : (costs[1] < costs[0] ? 1 : 0));
  *best_cost = costs[best];
  *second_cost = costs[r];
  *second_cut = r == 0 ? 2 : (r == 1 ? 1 : 3);
  return best == 0 ? 2 : (best == 1 ? 1 : 3);
}

// One merge group by one warp: pool rows r0 .. r0 + width - 1 of level `ell` (width 4, or 2 at a
// level's tail), staged as rows 0.. of gk / gv / gm, into merged rows r0 / 2 + j of scratch buffer 1
// from row out_off.  Pairwise: rows (0, 1) and (2, 3) merge count-weighted.  Beta: the cut is the
// certified warp cut, the canonical order on a near tie, or the update tape's; then every lane
// takes one (component, 16-byte column) pair of both sides.  Same arithmetic, in the same order,
// as merge_tile.
template <typename T, bool BETA, int DC>
__device__ void merge_group_warp(const LaneCtx<T>& x, const Geo& g, const Work& w, const T* gk, const T* gv,
                                 const Meta* gm, int r0, int width, int ell, int out_off, int lane) {
  constexpr int VN = Vec<T>::N;
  const int D = DC ? DC : g.D, DV = D / VN;
  T* SK = static_cast<T*>(w.sk);
  T* SV = static_cast<T*>(w.sv);
  const int orow = out_off + r0 / 2;
  if (!BETA) {
    const int np = width / 2;
    for (int item = lane; item < np * 2 * DV; item += 32) {
      const int j = item / (2 * DV), f = (item / DV) & 1, v = item % DV;
      const float wa = gm[2 * j].w, wb = gm[2 * j + 1].w;
      const float alpha = fdiv(wa, fmaxf(fadd(wa, wb), 1e-8f));
      const float beta = fsub(1.f, alpha);
      const T* base = f ? gv : gk;
      float a[VN], b[VN], o[VN];
      unpack(*reinterpret_cast<const uint4*>(base + 2 * j * D + v * VN), a, (const T*)nullptr);
      unpack(*reinterpret_cast<const uint4*>(base + (2 * j + 1) * D + v * VN), b, (const T*)nullptr);
#pragma unroll
      for (int e = 0; e < VN; ++e) o[e] = fadd(fmul(alpha, a[e]), fmul(beta, b[e]));
      *reinterpret_cast<uint4*>((f ? SV : SK) + x.scr_row(1, orow + j) * D + v * VN) = pack(o, (const T*)nullptr);
    }
    if (lane < np) x.put_scratch(1, orow + lane, merge_meta(gm[2 * lane], gm[2 * lane + 1]));
    return;
  }
  const bool two = width == 4;
  int cut = 1;
  bool finite = false;   // the certified warp cut saw every row finite (energies <= 1e30)
  uint8_t* tcut = g.tape != kTapeNone
                      ? w.tape_cuts + ((size_t)(w.tape_cut_lane >= 0 ? w.tape_cut_lane : (long long)x.lane) * g.L + ell) * tape_cut_stride(g) + r0 / 4
                      : nullptr;
  if (two) {
    if (g.tape == kTapeReplay) {
      cut = *tcut;
    } else {
      cut = beta_cut_warp<T, DC>(gk, gv, gm, 0, D, lane);
      finite = cut >= 0;
      if (cut < 0) {
        float bc, sc;
        int scut;
        cut = beta_cut_canonical_warp<T, DC>(gk, gv, gm, D, lane, &bc, &sc, &scut);
        if (lane == 0) {
          atomicAdd(&w.counters[kCntExactCuts], 1ull);
          if (near_tie(bc, sc))
            log_tie(w, LOGKV_TIE_BETA_CUT, x.b, x.grp, x.c, ell * 65536 + r0 / 4, cut, scut, rel_gap(bc, sc), bc);
        }
      }
    }
  }
  if (g.tape == kTapeRecord && lane == 0) *tcut = (uint8_t)cut;   // a 2-row tail records its sentinel 1
  // Apply: per output side, sum over member rows (row order) of w * x / max(mass, 1e-12); each
  // side keeps its own products (x * 0 for rows of the other side) and sums in row order.  With
  // finite rows the other side's products are skipped: each sum starts at +0, which adding
  // +-0 leaves unchanged, and a sum of products never becomes -0, so the bits are the same.
  if (finite) {
    for (int item = lane; item < 2 * DV; item += 32) {
      const int f = item / DV, v = item % DV;
      const T* base = f ? gv : gk;
      float acc0[VN], acc1[VN], mass0 = 0.f, mass1 = 0.f;
#pragma unroll
      for (int e = 0; e < VN; ++e) acc0[e] = acc1[e] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float xr[VN];
        unpack(*reinterpret_cast<const uint4*>(base + i * D + v * VN), xr, (const T*)nullptr);
        const float om = fmul(gm[i].w, 1.f);
        if (i < cut) {
          mass0 = fadd(mass0, om);
#pragma unroll
          for (int e = 0; e < VN; ++e) acc0[e] = fadd(acc0[e], fmul(xr[e], om));
        } else {
          mass1 = fadd(mass1, om);
#pragma unroll
          for (int e = 0; e < VN; ++e) acc1[e] = fadd(acc1[e], fmul(xr[e], om));
        }
      }
      const float den0 = fmaxf(mass0, 1e-12f), den1 = fmaxf(mass1, 1e-12f);
#pragma unroll
      for (int e = 0; e < VN; ++e) {
        acc0[e] = fdiv(acc0[e], den0);
        acc1[e] = fdiv(acc1[e], den1);
      }
      *reinterpret_cast<uint4*>((f ? SV : SK) + x.scr_row(1, orow) * D + v * VN) = pack(acc0, (const T*)nullptr);
      *reinterpret_cast<uint4*>((f ? SV : SK) + x.scr_row(1, orow + 1) * D + v * VN) = pack(acc1, (const T*)nullptr);
    }
  } else
  for (int item = lane; item < 2 * DV; item += 32) {
    const int f = item / DV, v = item % DV;
    const T* base = f ? gv : gk;
    float acc0[VN], acc1[VN], mass0 = 0.f, mass1 = 0.f;
#pragma unroll
    for (int e = 0; e < VN; ++e) acc0[e] = acc1[e] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const bool valid = i < width;
      const bool in0 = valid && (!two || i < cut), in1 = valid && two && i >= cut;
      const float wi = valid ? gm[i].w : 0.f;
      const float om0 = fmul(wi, in0 ? 1.f : 0.f), om1 = fmul(wi, in1 ? 1.f : 0.f);
      float xr[VN];
      if (valid) {
        unpack(*reinterpret_cast<const uint4*>(base + i * D + v * VN), xr, (const T*)nullptr);
      } else {
#pragma unroll
        for (int e = 0; e < VN; ++e) xr[e] = 0.f;
      }
      mass0 = fadd(mass0, om0);
      mass1 = fadd(mass1, om1);
#pragma unroll
      for (int e = 0; e < VN; ++e) {
        acc0[e] = fadd(acc0[e], fmul(xr[e], om0));
        acc1[e] = fadd(acc1[e], fmul(xr[e], om1));
      }
    }
    const float den0 = fmaxf(mass0, 1e-12f);
#pragma unroll
    for (int e = 0; e < VN; ++e) acc0[e] = fdiv(acc0[e], den0);
    *reinterpret_cast<uint4*>((f ? SV : SK) + x.scr_row(1, orow) * D + v * VN) = pack(acc0, (const T*)nullptr);
    if (two) {
      const float den1 = fmaxf(mass1, 1e-12f);
#pragma unroll
      for (int e = 0; e < VN; ++e) acc1[e] = fdiv(acc1[e], den1);
      *reinterpret_cast<uint4*>((f ? SV : SK) + x.scr_row(1, orow + 1) * D + v * VN) = pack(acc1, (const T*)nullptr);
    }
  }
  if (lane < (two ? 2 : 1)) {
    const int side = lane;
    float mass = 0.f;
    int64_t lo = INT64_MAX, hi = INT64_MIN, swp = 0, ord = INT64_MAX;
    uint8_t pad = 1;
    for (int i = 0; i < width; ++i) {
      const bool in = width == 2 ? side == 0 : (side == 0 ? i < cut : i >= cut);
      const Meta& r = gm[i];
      mass = fadd(mass, fmul(r.w, in ? 1.f : 0.f));
      if (!in) continue;
      if (r.w > 0.f) {
        lo = min(lo, r.lo);
        hi = max(hi, r.hi);
      }
      swp += r.swp;
      ord = min(ord, r.ord);
      pad &= r.pad;
    }
    x.put_scratch(1, orow + side, Meta{mass, mass > 0.f ? lo : 0, mass > 0.f ? hi : 0, swp, ord, pad});
  }
}

constexpr int kMergeWarps = 8;
constexpr int kMergeCtas = 4;  // CTAs per lane; the lane's merge groups are dealt to their warps

inline size_t merge_smem(int D, size_t esize) {
  return (size_t)kMergeWarps * 2 * (8 * (size_t)D * esize + 4 * sizeof(Meta));
}

// Grid (kMergeCtas, K, B * G).  The merge groups (4 pool rows; 2 at a level's tail) of every merging
// level of the lane, level by level, are dealt round-robin to the warps of the lane's CTAs.  A warp
// keeps two groups in flight: while it merges one (from its own shared rows) into the next level's
// incoming rows (scratch buffer 1), the next one's rows are arriving (16-byte cp.async).
template <typename T, bool BETA, int DC>
__global__ void __launch_bounds__(kMergeWarps * 32) cascade_merge_kernel(Geo g, logkv_state_t s, Work w) {
  // Launched right behind the prepare kernel, whose writes only delayed lanes read (their staged
  // re-inserts; new and delayed clusters, which prepare clears, merge no stored rows): those lanes
  // wait for it, the others run beside it.  CTA (0, 0, 0) always waits, so this grid completes
  // only after the prepare kernel has, and the move kernel's wait on this grid covers both.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bgi = blockIdx.z;
  const LaneCtx<T> x = make_ctx_at<T>(g, s, w, blockIdx.y, bgi % g.G, bgi / g.G);
  const bool late = __ldcg(w.plan_type + x.lane) == kJobLate;
  if (late || (blockIdx.x | blockIdx.y | blockIdx.z) == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ LevelPlan lp[kMaxLevels];
  __shared__ int gstart[kMaxLevels + 1];   // first group index of every level
  __shared__ const T* rowp[kMergeWarps][2][2][4];
  const int mode = plan_lane(g, w, x.lane, lp);
  if (tid == 0) {
    int ng = 0;
    for (int l = 0; l < g.L; ++l) {
      gstart[l] = ng;
      if (lp[l].kind == kLvlMerge) ng += (lp[l].npair + 3) / 4;
    }
    gstart[g.L] = ng;
    if (blockIdx.x == 0) {
      if (mode == 2) atomicAdd(&w.counters[kCntSeqLanes], 1ull);
      if (mode == 1) {
        unsigned long long carries = 0;
        for (int l = 0; l < g.L; ++l)
          if (lp[l].kind == kLvlMerge) carries += lp[l].npair / 2;
        if (carries) atomicAdd(&w.counters[kCntCarry], carries);
      }
    }
  }
  __syncthreads();
  if (mode != 1) return;
  constexpr int VN = Vec<T>::N;
  const int D = DC ? DC : g.D, DV = D / VN;
  extern __shared__ uint4 smem4[];
  T* rows = reinterpret_cast<T*>(smem4) + (size_t)warp * 2 * 8 * D;   // [2 buffers][4 K rows, 4 V rows][D]
  Meta* metas = reinterpret_cast<Meta*>(reinterpret_cast<T*>(smem4) + (size_t)kMergeWarps * 2 * 8 * D) + warp * 8;
  const int ng = gstart[g.L];
  const int stride = gridDim.x * kMergeWarps;
  // Group q -> (level, first pool row, width); issue its rows into buffer `buf`.
  auto locate = [&](int q, int& l, int& r0, int& width) {
    l = 0;
    while (gstart[l + 1] <= q) ++l;
    r0 = 4 * (q - gstart[l]);
    width = min(4, lp[l].npair - r0);
  };
  auto stage = [&](int q, int buf) {
    int l, r0, width;
    locate(q, l, r0, width);
    T* gk = rows + (size_t)buf * 8 * D;
    T* gv = gk + 4 * (size_t)D;
    if (lane < width) {
      const PoolRow<T> r = pool_row<T>(x, lp[l], l, r0 + lane, late);
      rowp[warp][buf][0][lane] = r.k;
      rowp[warp][buf][1][lane] = r.v;
      metas[buf * 4 + lane] = r.m;
    }
    __syncwarp();
    for (int item = lane; item < width * 2 * DV; item += 32) {
      const int r = item / (2 * DV), f = (item / DV) & 1, v = item % DV;
      cp_async16((f ? gv : gk) + r * D + v * VN, rowp[warp][buf][f][r] + v * VN);
    }
    cp_async_commit();
  };
  int q = blockIdx.x * kMergeWarps + warp, buf = 0;
  if (q < ng) stage(q, 0);
  for (; q < ng; q += stride, buf ^= 1) {
    const int qn = q + stride;
    if (qn < ng) {
      stage(qn, buf ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");   // the current group's rows have landed
    } else {
      cp_async_wait_all();
    }
    __syncwarp();
    int l, r0, width;
    locate(q, l, r0, width);
    const T* gk = rows + (size_t)buf * 8 * D;
    merge_group_warp<T, BETA, DC>(x, g, w, gk, gk + 4 * (size_t)D, metas + buf * 4, r0, width, l,
                                  lp[l + 1].in_off, lane);
    __syncwarp();  // buffer `buf` is free for the group after next
  }
}

constexpr int kMoveThreads = 256;
constexpr int kMoveWalkTile = 32;   // tile rows of a sequential walk inside the move kernel

inline size_t move_smem(const Geo& g, size_t esize) {
  const size_t moves = 2 * (size_t)g.Bs * g.D * esize + (size_t)g.Bs * sizeof(Meta) + 16;
  const size_t walk = walk_smem(g, esize, kMoveWalkTile);
  return moves > walk ? moves : walk;
}

// Grid (L, K, B * G): one CTA per (lane, level) of the lanes the merge kernel handles (and the
// level-0 CTA of every lane left to the sequential walk).  The rows the level writes (a filling level: its incoming rows,
// to slots cnt..; a merging level: all its survivors, pool rows npair.., to slots 0..) are first
// brought into shared memory by TMA bulk copies (the stored survivors and carried rows are
// contiguous runs, one copy each; level-0 token rows one copy per row), then written back with one
// bulk copy per K and V run, so no stored row is overwritten before it has been read.  The launch
// may overlap the merge kernel (programmatic dependent launch): the plan, the stored survivors
// (which the merge kernel only reads) and level-0 token rows are fetched before the grid
// dependency wait; carried rows, a delayed lane's staged rows and every write come after it.
// A merging level then zeroes its tail slots.  The copy wait is bounded: past the limit the
// status word gets kStatusCopyTimeout and nothing is written.
template <typename T, bool BETA, int DC>
__global__ void __launch_bounds__(kMoveThreads, 3) cascade_move_kernel(Geo g, logkv_state_t s, Work w) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x, nt = blockDim.x, l = blockIdx.x, bgi = blockIdx.z;
  const LaneCtx<T> x = make_ctx_at<T>(g, s, w, blockIdx.y, bgi % g.G, bgi / g.G);
  __shared__ LevelPlan lp[kMaxLevels];
  const int mode = plan_lane(g, w, x.lane, lp);
  if (mode == 2) {
    // A lane the parallel kernels leave alone: its level-0 CTA walks the levels in order, once
    // the prepare kernel (staged re-inserts, cleared clusters) has completed.
    if (l != 0) return;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    cascade_walk<T, BETA, DC, kMoveWalkTile>(x, g, s, w);
    return;
  }
  const LevelPlan p = lp[l];
  if (mode != 1 || (p.kind != kLvlFill && p.kind != kLvlMerge)) return;
  const int D = g.D, Bs = g.Bs;
  const bool late = w.plan_type[x.lane] == kJobLate;
  const bool fill = p.kind == kLvlFill;
  const int n = fill ? p.m : p.nsurv;                  // rows written, to slots dst0 ..
  const int dst0 = fill ? p.cnt : 0;
  const int nst = fill ? 0 : max(0, p.cnt - p.npair);  // stored survivors: slots npair .. cnt - 1
  const int src0 = fill ? p.cnt : p.npair;             // pool row of staged row 0
  const int in0 = src0 + nst - p.cnt;                   // incoming row of staged row nst
  const int nin = n - nst;
  const unsigned rowb = (unsigned)(D * sizeof(T));
  T* LK = static_cast<T*>(s.level_k);
  T* LV = static_cast<T*>(s.level_v);
  const size_t lrow0 = x.level_row(l, 0);
  extern __shared__ uint4 smem4[];
  T* tk = reinterpret_cast<T*>(smem4);                          // [Bs][D]
  T* tv = tk + (size_t)Bs * D;                                  // [Bs][D]
  Meta* tm = reinterpret_cast<Meta*>(tv + (size_t)Bs * D);      // [Bs]
  uint64_t* bar = reinterpret_cast<uint64_t*>(tm + Bs);
  const bool tokens = l == 0 && !late;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  if (tid == 0) mbar_arrive_expect_tx(bar, 2u * (unsigned)n * rowb);
  __syncthreads();
  auto issue_incoming = [&]() {
    if (tid == 0 && nin && !tokens) {
      const size_t r = x.scr_row(l > 0 ? 1 : 0, (l > 0 ? p.in_off : 0) + in0);
      bulk_load(tk + (size_t)nst * D, static_cast<const T*>(w.sk) + r * D, (unsigned)nin * rowb, bar);
      bulk_load(tv + (size_t)nst * D, static_cast<const T*>(w.sv) + r * D, (unsigned)nin * rowb, bar);
    }
    if (tokens)
      for (int i = tid; i < nin; i += nt) {
        const int src = x.token_src(in0 + i);
        bulk_load(tk + (size_t)(nst + i) * D, token_row<T>(g, x.snapk, x.reck, x.b, x.grp, src), rowb, bar);
        bulk_load(tv + (size_t)(nst + i) * D, token_row<T>(g, x.snapv, x.recv, x.b, x.grp, src), rowb, bar);
      }
    for (int r = nst + tid; r < n; r += nt) tm[r] = pool_row<T>(x, p, l, src0 + r, late).m;
  };
  if (tid == 0 && nst) {
    bulk_load(tk, LK + (lrow0 + p.npair) * D, (unsigned)nst * rowb, bar);
    bulk_load(tv, LV + (lrow0 + p.npair) * D, (unsigned)nst * rowb, bar);
  }
  for (int r = tid; r < nst; r += nt) tm[r] = pool_row<T>(x, p, l, src0 + r, late).m;
  if (tokens) issue_incoming();   // level-0 tokens: ready since the snapshot kernel
  asm volatile("griddepcontrol.wait;" ::: "memory");   // the merge (and so the prepare) kernel has completed
  if (!tokens) issue_incoming();  // carries of level l - 1, or a delayed lane's staged re-inserts
  const bool ok = mbar_wait_bounded(bar, 0);
  __syncthreads();
  if (!ok) {
    if (tid == 0) set_status(w.status, kStatusCopyTimeout);
    mbar_wait_bounded(bar, 0);   // give the copies in flight one more bounded wait before leaving
    return;
  }
  if (tid == 0 && n > 0) {
    fence_proxy_async();
    bulk_store(LK + (lrow0 + dst0) * D, tk, (unsigned)n * rowb);
    bulk_store(LV + (lrow0 + dst0) * D, tv, (unsigned)n * rowb);
    bulk_commit();
  }
  for (int r = tid; r < n; r += nt) x.put_level_meta(lrow0 + dst0 + r, tm[r]);
  if (!fill) {
    constexpr int VN = Vec<T>::N;
    const int DV = D / VN, nclr = Bs - n;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    for (int item = tid; item < nclr * DV * 2; item += nt) {
      const int r = item / (2 * DV), f = (item / DV) & 1, v = item % DV;
      *reinterpret_cast<uint4*>((f ? LV : LK) + (lrow0 + n + r) * D + v * VN) = zero;
    }
    for (int r = tid; r < nclr; r += nt) x.put_level_meta(lrow0 + n + r, Meta{0.f, 0, 0, 0, 0, 0});
  }
  if (tid == 0) {
    s.level_count[x.lane * g.L + l] = (int16_t)(fill ? p.cnt + p.m : n);
    atomicAdd(&w.counters[kCntStageRead], (unsigned long long)p.m);
    if (fill) {
      atomicAdd(&w.counters[kCntFill], (unsigned long long)p.m);
    } else {
      atomicAdd(&w.counters[kCntStorageRead], (unsigned long long)p.cnt);
      atomicAdd(&w.counters[kCntSurvivor], (unsigned long long)n);
      atomicAdd(&w.counters[kCntClear], (unsigned long long)(Bs - n));
    }
    bulk_wait_all();   // the shared rows stay allocated until the stores have read them
  }
}

}  // namespace logkv
