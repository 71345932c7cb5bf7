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

namespace logkv {

constexpr int kTileRows = 64;                 // multiple of 4 (Beta groups never straddle tiles)
constexpr int kTileGroups = kTileRows / 4;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

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

// Beta cut of one group of four rows by one warp, certified against the canonical cost.
//
// The canonical cost (beta_log_kv.select_cuts, beta_log_kv.py:29-46) of cut c for one
// component: energy = max(sum_i w_i E_i / max(sum w, 1e-12), 1e-12) with E_i = sum_d x_id^2;
// per side, mean_d = (sum_i om_i x_id) / max(sum om, 1e-12) (om = w on the side, else 0),
// loss = sum_i om_i sum_d (x_id - mean_d)^2; cost_c += loss / energy over sides and
// components, argmin over cuts (2, 1, 3) with ties to the earlier.  Rows off a side have
// om = 0 and add exactly zero, so only the side's rows are evaluated here.
//
// This warp evaluates the same quantities with three differences: sums over features run
// per lane and then across lanes (another order of adding non-negative terms); squares
// are accumulated with fused multiply-adds; and a side mean is the side's sum (the same
// rounded sum as the canonical one) times a rounded reciprocal of its mass, which lies
// within 3 u M_d of the canonical mean (u = 2^-24, M_d = max_i |x_id|), so each squared
// deviation moves by at most 32 u M_d^2 and a component's losses by 32 u (sum w)(sum_i E_i).
// All other differences are relative: at most about (4 D + 128) u of a cost.  With
// B = sum over components of 40 u (sum w)(sum_i E_i) / energy and rel = (4 D + 128) u,
// the returned cut is the canonical one whenever runner-up minus best exceeds
// 2 rel * runner-up + 2 B (plus a floor for subnormal rounding).  Otherwise, or when a
// row energy exceeds 1e30 (no overflow anywhere below that), -1 asks for the canonical
// evaluation.
template <typename T, int DC>
__device__ int beta_cut_warp(const T* tk, const T* tv, const Meta* tm, int start, int Drt, int lane) {
  const int D = DC ? DC : Drt;
  constexpr int NPL = (DC >= 32 && DC % 32 == 0) ? DC / 32 : 0;  // features per lane, compile time
  float wv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) wv[i] = tm[start + i].w;
  const float wsum = fadd(fadd(fadd(wv[0], wv[1]), wv[2]), wv[3]);
  const float tot = fmaxf(wsum, 1e-12f);
  // Side masses: left of cut c = w_0..w_{c-1}, right = w_c..w_3 (c = 1, 2, 3).
  const float wl1 = wv[0], wl2 = fadd(wv[0], wv[1]), wl3 = fadd(wl2, wv[2]);
  const float wr3 = wv[3], wr2 = fadd(wv[2], wv[3]), wr1 = fadd(fadd(wv[1], wv[2]), wv[3]);
  const float il1 = fdiv(1.f, fmaxf(wl1, 1e-12f)), il2 = fdiv(1.f, fmaxf(wl2, 1e-12f)),
              il3 = fdiv(1.f, fmaxf(wl3, 1e-12f));
  const float ir1 = fdiv(1.f, fmaxf(wr1, 1e-12f)), ir2 = fdiv(1.f, fmaxf(wr2, 1e-12f)),
              ir3 = fdiv(1.f, fmaxf(wr3, 1e-12f));
  float costs[3] = {0.f, 0.f, 0.f};
  float bound = 0.f;
  bool finite = true;
#pragma unroll
  for (int comp = 0; comp < 2; ++comp) {
    const T* base = (comp == 0 ? tk : tv) + start * D;
    // acc[0..3]: E_i; acc[4 + 4 jc + i]: squared deviations of row i for cut jc (cuts 2, 1, 3).
    float acc[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) acc[k] = 0.f;
    auto feature = [&](int d) {
      float x[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = Elem<T>::load(base + i * D + d);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = __fmaf_rn(x[i], x[i], acc[i]);
      const float p0 = __fmul_rn(x[0], wv[0]), p1 = __fmul_rn(x[1], wv[1]), p2 = __fmul_rn(x[2], wv[2]),
                  p3 = __fmul_rn(x[3], wv[3]);
      const float l2 = __fadd_rn(p0, p1), r2 = __fadd_rn(p2, p3);
      const float ml1 = __fmul_rn(p0, il1), ml2 = __fmul_rn(l2, il2), ml3 = __fmul_rn(__fadd_rn(l2, p2), il3);
      const float mr1 = __fmul_rn(__fadd_rn(__fadd_rn(p1, p2), p3), ir1), mr2 = __fmul_rn(r2, ir2), mr3 = __fmul_rn(p3, ir3);
      float df;
      // cut 2: rows 0,1 | 2,3
      df = __fsub_rn(x[0], ml2); acc[4] = __fmaf_rn(df, df, acc[4]);
      df = __fsub_rn(x[1], ml2); acc[5] = __fmaf_rn(df, df, acc[5]);
      df = __fsub_rn(x[2], mr2); acc[6] = __fmaf_rn(df, df, acc[6]);
      df = __fsub_rn(x[3], mr2); acc[7] = __fmaf_rn(df, df, acc[7]);
      // cut 1: row 0 | 1,2,3
      df = __fsub_rn(x[0], ml1); acc[8] = __fmaf_rn(df, df, acc[8]);
      df = __fsub_rn(x[1], mr1); acc[9] = __fmaf_rn(df, df, acc[9]);
      df = __fsub_rn(x[2], mr1); acc[10] = __fmaf_rn(df, df, acc[10]);
      df = __fsub_rn(x[3], mr1); acc[11] = __fmaf_rn(df, df, acc[11]);
      // cut 3: rows 0,1,2 | 3
      df = __fsub_rn(x[0], ml3); acc[12] = __fmaf_rn(df, df, acc[12]);
      df = __fsub_rn(x[1], ml3); acc[13] = __fmaf_rn(df, df, acc[13]);
      df = __fsub_rn(x[2], ml3); acc[14] = __fmaf_rn(df, df, acc[14]);
      df = __fsub_rn(x[3], mr3); acc[15] = __fmaf_rn(df, df, acc[15]);
    };
    if constexpr (NPL > 0) {
#pragma unroll
      for (int j = 0; j < NPL; ++j) feature(lane + 32 * j);
    } else {
#pragma unroll 1
      for (int d = lane; d < D; d += 32) feature(d);
    }
    warp_allreduce16(acc, lane);
    const float esum = acc[0] + acc[1] + acc[2] + acc[3];
    finite = finite && esum <= 1e30f;  // also false for NaN
    const float energy = fmaxf(fdiv(fadd(fadd(fadd(fmul(acc[0], wv[0]), fmul(acc[1], wv[1])), fmul(acc[2], wv[2])),
                                         fmul(acc[3], wv[3])),
                                    tot),
                               1e-12f);
    const float inv_e = fdiv(1.f, energy);
    // cut 2 (costs[0]), cut 1 (costs[1]), cut 3 (costs[2]); left side then right side.
    costs[0] += (acc[4] * wv[0] + acc[5] * wv[1]) * inv_e + (acc[6] * wv[2] + acc[7] * wv[3]) * inv_e;
    costs[1] += (acc[8] * wv[0]) * inv_e + (acc[9] * wv[1] + acc[10] * wv[2] + acc[11] * wv[3]) * inv_e;
    costs[2] += (acc[12] * wv[0] + acc[13] * wv[1] + acc[14] * wv[2]) * inv_e + (acc[15] * wv[3]) * inv_e;
    bound += 40.f * 5.9604645e-8f * wsum * esum * inv_e;
  }
  if (!finite) return -1;
  int best = 0;
  if (costs[1] < costs[best]) best = 1;
  if (costs[2] < costs[best]) best = 2;
  float second = INFINITY;
#pragma unroll
  for (int j = 0; j < 3; ++j)
    if (j != best) second = fminf(second, costs[j]);
  const float rel = (4.f * D + 128.f) * 5.9604645e-8f;
  const float margin = 2.f * rel * second + 2.f * bound + 1e-25f * (1.f + wsum);
  if (!(second - costs[best] > margin)) return -1;  // near tie (or NaN): canonical evaluation
  return best == 0 ? 2 : (best == 1 ? 1 : 3);
}

template <typename T, bool BETA, int DC>
__global__ void __launch_bounds__(512) cascade_kernel(Geo g, logkv_state_t s, Work w) {
  pdl_entry();
  LaneCtx<T> x = make_ctx<T>(g, s, w);
  const int type = w.plan_type[x.lane];
  if (type == kJobNone) return;
  constexpr int VN = Vec<T>::N;
  const int tid = threadIdx.x, nt = blockDim.x, Bs = g.Bs;
  // Compile-time head dim when DC != 0: every row/vector index map becomes shifts.
  const int D = DC ? DC : g.D, DV = D / VN;
  extern __shared__ uint4 smem4[];
  T* tkb = reinterpret_cast<T*>(smem4);                                 // [2][kTileRows][D]
  T* tvb = tkb + 2 * (size_t)kTileRows * D;                             // [2][kTileRows][D]
  Meta* tmb = reinterpret_cast<Meta*>(tvb + 2 * (size_t)kTileRows * D);  // [2][kTileRows]
  int64_t* tpos = reinterpret_cast<int64_t*>(tmb + 2 * kTileRows);      // [NW] token positions
  int* srcs = reinterpret_cast<int*>(tpos + g.NW);                      // [NW] token sources
  __shared__ float bloss[kTileGroups][12];
  __shared__ float bener[kTileGroups][2];
  __shared__ int bcut[kTileGroups];
  __shared__ int sh_exact;  // groups of the current tile needing the canonical cost order
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
      for (int j0 = 1; j0 < Bs; j0 += kTileRows - 1) {
        const int jn = min(kTileRows - 1, Bs - j0);
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
    auto issue = [&](int t0, int buf) {
      const int tn = min(kTileRows, total - t0);
      T* tk = tkb + (size_t)buf * kTileRows * D;
      T* tv = tvb + (size_t)buf * kTileRows * D;
      for (int item = tid; item < tn * DV * 2; item += nt) {
        const int r = item / (2 * DV), f = (item / DV) & 1, v = item % DV;
        cp_async16((f ? tv : tk) + r * D + v * VN, (f ? pool_v(t0 + r) : pool_k(t0 + r)) + v * VN);
      }
      cp_async_commit();
      if (tid < tn) pend = pool_m(t0 + tid);
    };
    issue(0, 0);
    int cur = 0;
    for (int t0 = 0; t0 < total; t0 += kTileRows) {
      const int tn = min(kTileRows, total - t0);
      T* tk = tkb + (size_t)cur * kTileRows * D;
      T* tv = tvb + (size_t)cur * kTileRows * D;
      Meta* tm = tmb + cur * kTileRows;
      cp_async_wait_all();
      if (tid < tn) tm[tid] = pend;
      __syncthreads();
      if (t0 + kTileRows < total) issue(t0 + kTileRows, cur ^ 1);
      const int mend = min(t0 + tn, npair);  // merge rows of this tile: [t0, mend)
      if (mend > t0) {
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
            *reinterpret_cast<uint4*>((f ? SV : SK) + x.scr_row(nb, j0 + j) * D + v * VN) = pack(o, (const T*)nullptr);
          }
          for (int j = tid; j < jn; j += nt) x.put_scratch(nb, j0 + j, merge_meta(tm[2 * j], tm[2 * j + 1]));
        } else {
          const int qn = (mend - t0 + 3) / 4;  // groups of this tile (tile rows 4q..4q+3)
          // Certified warp-parallel cut per group; near ties fall back to the canonical order below.
          const int warp = tid >> 5, lane = tid & 31, nwarps = nt >> 5;
          for (int q = warp; q < qn; q += nwarps) {
            const int width = min(4, npair - (t0 + 4 * q));
            const int cut = width == 4 ? beta_cut_warp<T, DC>(tk, tv, tm, 4 * q, D, lane) : 1;
            if (lane == 0) {
              bcut[q] = cut;
              if (cut < 0) atomicAdd(&sh_exact, 1);
            }
          }
          __syncthreads();
          if (sh_exact) {
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
          }
          __syncthreads();
          if (tid == 0) {
            atomicAdd(&w.counters[kCntExactCuts], (unsigned long long)sh_exact);
            sh_exact = 0;
          }
          }
          // Apply: per output side, sum over member rows (row order) of w*x / max(mass, 1e-12).
          for (int item = tid; item < qn * 2 * 2 * DV; item += nt) {
            const int q = item / (4 * DV), side = (item / (2 * DV)) & 1, f = (item / DV) & 1, v = item % DV;
            const int start = 4 * q;
            const int width = min(4, npair - (t0 + start));
            if (side == 1 && width != 4) continue;
            const int cut = bcut[q];
            const T* base = f ? tv : tk;
            float acc[VN], mass = 0.f;
#pragma unroll
            for (int e = 0; e < VN; ++e) acc[e] = 0.f;
            for (int i = 0; i < 4; ++i) {
              const bool valid = i < width;
              const bool in = valid && (width == 2 ? side == 0 : (side == 0 ? i < cut : i >= cut));
              const float om = fmul(valid ? tm[start + i].w : 0.f, in ? 1.f : 0.f);
              float xr[VN];
              if (valid) {
                unpack(*reinterpret_cast<const uint4*>(base + (start + i) * D + v * VN), xr, (const T*)nullptr);
              } else {
#pragma unroll
                for (int e = 0; e < VN; ++e) xr[e] = 0.f;
              }
              mass = fadd(mass, om);
#pragma unroll
              for (int e = 0; e < VN; ++e) acc[e] = fadd(acc[e], fmul(xr[e], om));
            }
            const float den = fmaxf(mass, 1e-12f);
#pragma unroll
            for (int e = 0; e < VN; ++e) acc[e] = fdiv(acc[e], den);
            const int outrow = (t0 + start) / 2 + side;
            *reinterpret_cast<uint4*>((f ? SV : SK) + x.scr_row(nb, outrow) * D + v * VN) = pack(acc, (const T*)nullptr);
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
            x.put_scratch(nb, (t0 + start) / 2 + side,
                          Meta{mass, mass > 0.f ? lo : 0, mass > 0.f ? hi : 0, swp, ord, pad});
          }
        }
      }
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

}  // namespace logkv
