// grad_x fallbacks: FFMA, TMA-pipelined and mma.sync (3xTF32) kernels for
// the shapes and layouts the tcgen05 kernel does not take (and static H).
// Part of the fused layer translation unit (included by layer.cu, in order).
#pragma once

#include <cuda_bf16.h>

#include "../common.cuh"
#include "../sinkhorn.cuh"
#include "../sinkhorn_lanes.cuh"
#include "../tma.cuh"

namespace mhc {
namespace {

// ---------------------------------------------------------------------------
// Backward 3: grad_x, and per-split partials of dphi and grad_w.
//   Thread = one column (stream i, channel c) of a CW-channel tile; the CTA
//   walks a contiguous token range.  phi for the thread's column and its
//   dphi accumulator stay in registers for the whole range.
//   grad_x[i,c] = sum_j M[j,i] g[j,c] + h_i (gy[c] w[c] / r - x_agg[c] beta)
//                 + sum_k d_p[k] phi[k, iC+c] + coef x[i,c]
//   dphi[k, iC+c] += d_p[k] x[i,c] ;  grad_w[c] += gy[c] x_agg[c] / r
// ---------------------------------------------------------------------------
constexpr int GX_CW = 64;   // channels per CTA tile
constexpr int GX_TB = 8;    // tokens staged per smem batch

template <int N, bool DYN>
__global__ void __launch_bounds__(GX_CW* N)
    grad_x_kernel(const float* __restrict__ g, const float* __restrict__ x,
                  const float* __restrict__ w, const float* __restrict__ phi_pre,
                  const float* __restrict__ phi_post, const float* __restrict__ phi_res,
                  const float* __restrict__ tokb, float* __restrict__ gx,
                  float* __restrict__ dphi_part,
                  float* __restrict__ gw_part, int64_t B, int64_t C, int ntiles, int nsplit) {
  using Lc = L<N>;
  constexpr int NH = Lc::NH, NHP = Lc::NHP;
  constexpr int TBS = Lc::TB;                // per-token row
  __shared__ __align__(16) float s_tok[GX_TB][TBS];
  const int tile = blockIdx.x % ntiles;
  const int split = blockIdx.x / ntiles;
  const int i = threadIdx.x / GX_CW;
  const int cl = threadIdx.x % GX_CW;
  const int64_t c = (int64_t)tile * GX_CW + cl;
  const bool cval = c < C;
  const int64_t nC = (int64_t)N * C;
  const int64_t col = (int64_t)i * C + c;
  // token range of this split
  const int64_t tb0 = B * split / nsplit, tb1 = B * (split + 1) / nsplit;

  float phi[DYN ? NHP : 1];
  float dph[DYN ? NHP : 1];
  if (DYN) {
#pragma unroll
    for (int k = 0; k < NHP; ++k) {
      phi[k] = (k < NH && cval) ? __ldg(phi_row(phi_pre, phi_post, phi_res, k, N, nC) + col) : 0.f;
      dph[k] = 0.f;
    }
  }
  const float wc = cval ? w[c] : 0.f;
  float gwacc = 0.f;

  for (int64_t t0 = tb0; t0 < tb1; t0 += GX_TB) {
    const int nt = (int)((tb1 - t0) < GX_TB ? (tb1 - t0) : GX_TB);
    __syncthreads();
    for (int e = threadIdx.x; e < nt * TBS; e += blockDim.x) {
      const int tt = e / TBS, f = e % TBS;
      s_tok[tt][f] = tokb[(t0 + tt) * TBS + f];
    }
    __syncthreads();
    if (!cval) continue;
    for (int tt = 0; tt < nt; ++tt) {
      const int64_t tok = t0 + tt;
      const float* st = s_tok[tt];
      const float beta = st[0], inv_r = st[1];
      const float* h = st + Lc::OFF_TH;
      const float* hp = st + Lc::OFF_THP;
      const float* m = st + Lc::OFF_TM;
      const float* gb = g + tok * nC + c;
      const float* xb = x + tok * nC + c;
      float gv[N], xv[N];
#pragma unroll
      for (int j = 0; j < N; ++j) { gv[j] = __ldg(gb + j * C); xv[j] = __ldg(xb + j * C); }
      float gy = 0.f, xa = 0.f, mix = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        gy = fmaf(hp[j], gv[j], gy);
        xa = fmaf(h[j], xv[j], xa);
        mix = fmaf(m[i * N + j], gv[j], mix);
      }
      const float xi = xv[i];
      float acc = mix + h[i] * (gy * wc * inv_r - xa * beta);
      if (DYN) {
        const float coef = st[2];
        const float* dp = st + 4;
        float2 a2 = make_float2(0.f, 0.f);
        const float2 x2 = make_float2(xi, xi);
#pragma unroll
        for (int k = 0; k < NHP; k += 2) {
          const float2 d2 = *reinterpret_cast<const float2*>(dp + k);
          const float2 p2 = make_float2(phi[k], phi[k + 1]);
          a2 = __ffma2_rn(d2, p2, a2);
          float2 q2 = make_float2(dph[k], dph[k + 1]);
          q2 = __ffma2_rn(d2, x2, q2);
          dph[k] = q2.x;
          dph[k + 1] = q2.y;
        }
        acc += (a2.x + a2.y) + coef * xi;
      }
      __stcs(gx + tok * nC + col, acc);
      if (i == 0) gwacc = fmaf(gy * xa, inv_r, gwacc);
    }
  }
  if (cval) {
    if (DYN) {
#pragma unroll
      for (int k = 0; k < NH; ++k) dphi_part[((int64_t)split * NH + k) * nC + col] = dph[k];
    }
    if (i == 0) gw_part[(int64_t)split * C + c] = gwacc;
  }
}

// ---------------------------------------------------------------------------
// Backward 3, TMA-pipelined (n <= 4, C % 4 == 0, 16-byte aligned tensors):
// same math and thread mapping as grad_x_kernel, but batches of GXT_TB tokens
// of grad_out, x and the per-token rows are brought into a GXT_STAGES-deep
// shared-memory ring by TMA (one elected thread issues the copies, an
// mbarrier per slot tracks arrival), so the bytes in flight no longer depend
// on how many warps are resident.
// ---------------------------------------------------------------------------
constexpr int GXT_TB = 8;      // tokens per stage
constexpr int GXT_STAGES = 4;

template <int N>
struct GxtCfg {
  static constexpr int ROWS = GXT_TB * N;                    // g / x rows per stage
  static constexpr int TILE_FLOATS = ROWS * GX_CW;           // one of g / x
  static constexpr int TOK_FLOATS = GXT_TB * L<N>::TB;
  static constexpr int STAGE_FLOATS = 2 * TILE_FLOATS + TOK_FLOATS;
  static constexpr uint32_t STAGE_BYTES = STAGE_FLOATS * 4;
  static constexpr size_t SMEM = (size_t)GXT_STAGES * STAGE_BYTES + 128 + 64;
};

template <int N, bool DYN>
__global__ void __launch_bounds__(GX_CW* N)
    grad_x_tma_kernel(const __grid_constant__ CUtensorMap gmap,
                      const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap tmap, const float* __restrict__ w,
                      const float* __restrict__ phi_pre, const float* __restrict__ phi_post,
                      const float* __restrict__ phi_res, float* __restrict__ gx,
                      float* __restrict__ dphi_part, float* __restrict__ gw_part, int64_t B,
                      int64_t C, int ntiles, int nsplit) {
  using Lc = L<N>;
  using Cf = GxtCfg<N>;
  constexpr int NH = Lc::NH, NHP = Lc::NHP, TBS = Lc::TB;
  extern __shared__ unsigned char smem_raw[];
  float* ring = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + GXT_STAGES * Cf::STAGE_FLOATS);

  const int tile = blockIdx.x % ntiles;
  const int split = blockIdx.x / ntiles;
  const int i = threadIdx.x / GX_CW;
  const int cl = threadIdx.x % GX_CW;
  const int64_t c = (int64_t)tile * GX_CW + cl;
  const bool cval = c < C;
  const int64_t nC = (int64_t)N * C;
  const int64_t col = (int64_t)i * C + c;
  const int64_t tb0 = B * split / nsplit, tb1 = B * (split + 1) / nsplit;
  const int nbatch = (int)((tb1 - tb0 + GXT_TB - 1) / GXT_TB);

  if (threadIdx.x == 0) {
    prefetch_tmap(&gmap);
    prefetch_tmap(&xmap);
    prefetch_tmap(&tmap);
    for (int st = 0; st < GXT_STAGES; ++st) mbar_init(&bars[st], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int j) {
    const int slot = j % GXT_STAGES;
    float* base = ring + slot * Cf::STAGE_FLOATS;
    const int t0 = (int)(tb0 + (int64_t)j * GXT_TB);
    mbar_expect_tx(&bars[slot], Cf::STAGE_BYTES);
    tma_load_2d(base, &gmap, tile * GX_CW, t0 * N, &bars[slot]);
    tma_load_2d(base + Cf::TILE_FLOATS, &xmap, tile * GX_CW, t0 * N, &bars[slot]);
    tma_load_2d(base + 2 * Cf::TILE_FLOATS, &tmap, 0, t0, &bars[slot]);
  };
  if (threadIdx.x == 0)
    for (int j = 0; j < GXT_STAGES && j < nbatch; ++j) issue(j);

  float phi[DYN ? NHP : 1];
  float dph[DYN ? NHP : 1];
  if (DYN) {
#pragma unroll
    for (int k = 0; k < NHP; ++k) {
      phi[k] = (k < NH && cval) ? __ldg(phi_row(phi_pre, phi_post, phi_res, k, N, nC) + col) : 0.f;
      dph[k] = 0.f;
    }
  }
  const float wc = cval ? w[c] : 0.f;
  float gwacc = 0.f;
  bool failed = false;

  for (int j = 0; j < nbatch; ++j) {
    const int slot = j % GXT_STAGES;
    const bool ok = threadIdx.x == 0 ? mbar_wait(&bars[slot], (uint32_t)((j / GXT_STAGES) & 1)) : true;
    if (__syncthreads_or(!ok)) { failed = true; break; }
    const float* gs = ring + slot * Cf::STAGE_FLOATS;
    const float* xs = gs + Cf::TILE_FLOATS;
    const float* ts = xs + Cf::TILE_FLOATS;
    const int64_t t0 = tb0 + (int64_t)j * GXT_TB;
    const int nt = (int)((tb1 - t0) < GXT_TB ? (tb1 - t0) : GXT_TB);
    if (cval) {
#pragma unroll 2
      for (int tt = 0; tt < nt; ++tt) {
        const int64_t tok = t0 + tt;
        const float* st = ts + tt * TBS;
        float beta, inv_r, coef, h[N], hp[N], mc[N];
        if constexpr (N == 4) {
          // per-token scalars as float4 broadcasts (row layout is 16-byte aligned at n = 4)
          const float4 s0 = *reinterpret_cast<const float4*>(st);
          const float4 h4 = *reinterpret_cast<const float4*>(st + Lc::OFF_TH);
          const float4 q4 = *reinterpret_cast<const float4*>(st + Lc::OFF_THP);
          const float4 m4 = *reinterpret_cast<const float4*>(st + Lc::OFF_TM + i * N);
          beta = s0.x; inv_r = s0.y; coef = s0.z;
          h[0] = h4.x; h[1] = h4.y; h[2] = h4.z; h[3] = h4.w;
          hp[0] = q4.x; hp[1] = q4.y; hp[2] = q4.z; hp[3] = q4.w;
          mc[0] = m4.x; mc[1] = m4.y; mc[2] = m4.z; mc[3] = m4.w;
        } else {
          beta = st[0]; inv_r = st[1]; coef = st[2];
#pragma unroll
          for (int jj = 0; jj < N; ++jj) {
            h[jj] = st[Lc::OFF_TH + jj];
            hp[jj] = st[Lc::OFF_THP + jj];
            mc[jj] = st[Lc::OFF_TM + i * N + jj];
          }
        }
        float gv[N], xv[N];
#pragma unroll
        for (int jj = 0; jj < N; ++jj) {
          gv[jj] = gs[(tt * N + jj) * GX_CW + cl];
          xv[jj] = xs[(tt * N + jj) * GX_CW + cl];
        }
        float gy = 0.f, xa = 0.f, mix = 0.f;
#pragma unroll
        for (int jj = 0; jj < N; ++jj) {
          gy = fmaf(hp[jj], gv[jj], gy);
          xa = fmaf(h[jj], xv[jj], xa);
          mix = fmaf(mc[jj], gv[jj], mix);
        }
        const float xi = xv[i];
        float acc = mix + h[i] * (gy * wc * inv_r - xa * beta);
        if (DYN) {
          const float4* dp4 = reinterpret_cast<const float4*>(st + 4);
          float2 a2 = make_float2(0.f, 0.f);
          const float2 x2 = make_float2(xi, xi);
#pragma unroll
          for (int k = 0; k < NHP; k += 4) {
            const float4 d4 = dp4[k / 4];
            const float2 da = make_float2(d4.x, d4.y), db = make_float2(d4.z, d4.w);
            a2 = __ffma2_rn(da, make_float2(phi[k], phi[k + 1]), a2);
            a2 = __ffma2_rn(db, make_float2(phi[k + 2], phi[k + 3]), a2);
            float2 q2 = __ffma2_rn(da, x2, make_float2(dph[k], dph[k + 1]));
            dph[k] = q2.x;
            dph[k + 1] = q2.y;
            q2 = __ffma2_rn(db, x2, make_float2(dph[k + 2], dph[k + 3]));
            dph[k + 2] = q2.x;
            dph[k + 3] = q2.y;
          }
          acc += (a2.x + a2.y) + coef * xi;
        }
        __stcs(gx + tok * nC + col, acc);
        if (i == 0) gwacc = fmaf(gy * xa, inv_r, gwacc);
      }
    }
    __syncthreads();  // slot fully consumed: refill it
    if (threadIdx.x == 0 && j + GXT_STAGES < nbatch) issue(j + GXT_STAGES);
  }
  if (failed) return;
  if (cval) {
    if (DYN) {
#pragma unroll
      for (int k = 0; k < NH; ++k) dphi_part[((int64_t)split * NH + k) * nC + col] = dph[k];
    }
    if (i == 0) gw_part[(int64_t)split * C + c] = gwacc;
  }
}

// ---------------------------------------------------------------------------
// 3xTF32 tensor-core helpers (m16n8k8, fp32 accumulate).  x = hi + lo with
// hi = tf32(x) (round to nearest) and lo = tf32(x - hi); a product is taken
// as hi*hi + hi*lo + lo*hi, which keeps ~fp32 accuracy (the dropped lo*lo
// term is below 2^-22 relative).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32_rna(x);
  lo = tf32_rna(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  // not volatile: a pure function of its operands, so the compiler may
  // interleave independent mma chains
  asm(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Backward 3 for n = 4 (C % 64 == 0, aligned): grad_x with tensor-core
// contractions.
//   CTA = 64 channels x 4 streams = 256 columns (col = i*64 + cl), 256
//   threads (8 warps, warp w owns columns 32w..32w+31), a contiguous token
//   range, TMA ring of 16-token stages.  Per stage:
//   (E) one thread per (token, channel): local terms of all 4 streams,
//       sum_j M[j,i] g_j + h_i (gy w / r - x_agg beta) + coef x_i -> smem,
//       and the stage's d_p split into tf32 hi/lo -> smem;
//   (C1) grad_x[tok, col] = local + (D_p[16 x 24] . Phi[24 x col]) with
//       mma.sync m16n8k8 3xTF32; the Phi fragments of the warp's columns stay
//       in registers for the whole token range;
//   (C2) dphi^T[col x k] += X^T[col x 16 tok] . D_p[16 tok x 24], same
//       instruction, accumulators persistent in registers.
// ---------------------------------------------------------------------------
constexpr int GX4_STAGES = 2;

struct Gx4Cfg {
  static constexpr int N = 4, CW = 64, COLS = N * CW, TOK = 16, TB = L<4>::TB;
  static constexpr int TILE = TOK * COLS;                 // g or x floats per stage
  static constexpr int STAGE = 2 * TILE + TOK * TB;
  static constexpr uint32_t STAGE_BYTES = STAGE * 4;
  static constexpr int NHP = L<4>::NHP;                   // 24
  // ring | gxl[TOK][COLS] | dph[TOK][NHP] | dpl[TOK][NHP] | gw[TOK/2][CW] | bars
  static constexpr size_t SMEM = ((size_t)GX4_STAGES * STAGE + TOK * COLS + 2 * TOK * NHP +
                                  (TOK / 2) * CW) * 4 + GX4_STAGES * 8 + 128;
};

template <bool DYN>
__global__ void __launch_bounds__(256, 2)
    grad_x4_kernel(const __grid_constant__ CUtensorMap gmap, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap omap,
                   const float* __restrict__ w,
                   const float* __restrict__ phi_pre, const float* __restrict__ phi_post,
                   const float* __restrict__ phi_res, float* __restrict__ gx,
                   float* __restrict__ dphi_part, float* __restrict__ gw_part, int64_t B,
                   int64_t C, int ntiles, int nsplit) {
  using F = Gx4Cfg;
  using Lc = L<4>;
  constexpr int N = 4, CW = F::CW, COLS = F::COLS, NHP = F::NHP, TB = F::TB, TOK = F::TOK;
  extern __shared__ unsigned char smem_raw[];
  float* ring = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  float* gxl = ring + GX4_STAGES * F::STAGE;
  uint32_t* dph_s = reinterpret_cast<uint32_t*>(gxl + TOK * COLS);   // [tok][k] hi
  uint32_t* dpl_s = dph_s + TOK * NHP;                               // [tok][k] lo
  float* gwS = reinterpret_cast<float*>(dpl_s + TOK * NHP);
  uint64_t* bars = reinterpret_cast<uint64_t*>(gwS + (TOK / 2) * CW);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int tile = blockIdx.x % ntiles;
  const int split = blockIdx.x / ntiles;
  const int64_t c0 = (int64_t)tile * CW;
  const int64_t nC = (int64_t)N * C;
  const int64_t tb0 = B * split / nsplit, tb1 = B * (split + 1) / nsplit;
  const int nbatch = (int)((tb1 - tb0 + TOK - 1) / TOK);

  if (tid == 0) {
    prefetch_tmap(&gmap);
    prefetch_tmap(&xmap);
    prefetch_tmap(&tmap);
    for (int st = 0; st < GX4_STAGES; ++st) mbar_init(&bars[st], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int j) {
    const int slot = j % GX4_STAGES;
    float* base = ring + slot * F::STAGE;
    const int t0 = (int)(tb0 + (int64_t)j * TOK);
    mbar_expect_tx(&bars[slot], F::STAGE_BYTES);
    tma_load_2d(base, &gmap, (int)c0, t0 * N, &bars[slot]);
    tma_load_2d(base + F::TILE, &xmap, (int)c0, t0 * N, &bars[slot]);
    tma_load_2d(base + 2 * F::TILE, &tmap, 0, t0, &bars[slot]);
  };
  if (tid == 0)
    for (int j = 0; j < GX4_STAGES && j < nbatch; ++j) issue(j);

  // warp columns: stream wi, channels wc0 .. wc0+31 of the tile
  const int wi = warp >> 1, wc0 = (warp & 1) * 32;
  // (C1) B fragments: Phi[k][col] for n-tile nt (8 columns), k-step ks
  uint32_t bph[4][3][2], bpl[4][3][2];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int ks = 0; ks < 3; ++ks)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int k = 8 * ks + t4 + 4 * h;
        float v = 0.f;
        if (DYN && k < Lc::NH)
          v = __ldg(phi_row(phi_pre, phi_post, phi_res, k, N, nC) + (int64_t)wi * C + c0 + wc0 + 8 * nt + g8);
        split_tf32(v, bph[nt][ks][h], bpl[nt][ks][h]);
      }
  // (C2) accumulators: dphi^T rows = columns (2 m-tiles of 16), cols = k (3 n-tiles of 8)
  float acc2[2][3][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 3; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc2[mt][nt][e] = 0.f;
  // (E) mapping: tokens ee and ee + 8, channels ce and ce + 32
  const int ee = tid >> 5, ce = tid & 31;
  const float w0 = __ldg(w + c0 + ce), w1 = __ldg(w + c0 + ce + 32);
  float gw0 = 0.f, gw1 = 0.f;

  bool failed = false;
  for (int j = 0; j < nbatch; ++j) {
    const int slot = j % GX4_STAGES;
    // one thread polls the barrier (after the previous grad_x store has read
    // gxl); the others park at the CTA barrier
    bool ok = true;
    if (tid == 0) {
      bulk_wait_read0();
      ok = mbar_wait(&bars[slot], (uint32_t)((j / GX4_STAGES) & 1));
    }
    if (__syncthreads_or(!ok)) { failed = true; break; }
    // every thread is past stage j-1: its slot can be refilled
    if (tid == 0 && j >= 1 && j - 1 + GX4_STAGES < nbatch) issue(j - 1 + GX4_STAGES);
    const float* gs = ring + slot * F::STAGE;
    const float* xs = gs + F::TILE;
    const float* ts = xs + F::TILE;
    const int64_t t0 = tb0 + (int64_t)j * TOK;
    const int nt_ = (int)((tb1 - t0) < TOK ? (tb1 - t0) : TOK);

    // d_p of the stage in tf32 hi/lo; tokens beyond the range contribute 0
    if (DYN) {
      for (int e = tid; e < TOK * NHP; e += 256) {
        const int tt = e / NHP, k = e % NHP;
        const float d = tt < nt_ ? ts[tt * TB + 4 + k] : 0.f;
        split_tf32(d, dph_s[e], dpl_s[e]);
      }
    }
    // (E) local terms
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int te = ee + 8 * r;
      if (te < nt_) {
        const float* st = ts + te * TB;
        const float4 s0 = *reinterpret_cast<const float4*>(st);
        const float4 h4 = *reinterpret_cast<const float4*>(st + Lc::OFF_TH);
        const float4 q4 = *reinterpret_cast<const float4*>(st + Lc::OFF_THP);
        const float h[4] = {h4.x, h4.y, h4.z, h4.w};
        const float hq[4] = {q4.x, q4.y, q4.z, q4.w};
        float mt[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 m4 = *reinterpret_cast<const float4*>(st + Lc::OFF_TM + 4 * i);
          mt[i][0] = m4.x; mt[i][1] = m4.y; mt[i][2] = m4.z; mt[i][3] = m4.w;
        }
        const float beta = s0.x, inv_r = s0.y, coef = DYN ? s0.z : 0.f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int cl = ce + 32 * half;
          float gv[4], xv[4];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            gv[jj] = gs[(te * 4 + jj) * CW + cl];
            xv[jj] = xs[(te * 4 + jj) * CW + cl];
          }
          float gy = 0.f, xa = 0.f;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) { gy = fmaf(hq[jj], gv[jj], gy); xa = fmaf(h[jj], xv[jj], xa); }
          const float wc = half ? w1 : w0;
          const float agg = gy * wc * inv_r - xa * beta;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float mix = 0.f;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) mix = fmaf(mt[i][jj], gv[jj], mix);
            gxl[te * COLS + i * CW + cl] = mix + h[i] * agg + coef * xv[i];
          }
          const float gwv = gy * xa * inv_r;
          if (half) gw1 += gwv; else gw0 += gwv;
        }
      }
    }
    __syncthreads();

    // (C1) grad_x: 4 n-tiles of 8 columns, rows = the 16 tokens
    uint32_t ah[3][4], al[3][4];
    if (DYN) {
#pragma unroll
      for (int ks = 0; ks < 3; ++ks) {
        const int k0 = 8 * ks + t4;
        ah[ks][0] = dph_s[g8 * NHP + k0];       al[ks][0] = dpl_s[g8 * NHP + k0];
        ah[ks][1] = dph_s[(g8 + 8) * NHP + k0]; al[ks][1] = dpl_s[(g8 + 8) * NHP + k0];
        ah[ks][2] = dph_s[g8 * NHP + k0 + 4];   al[ks][2] = dpl_s[g8 * NHP + k0 + 4];
        ah[ks][3] = dph_s[(g8 + 8) * NHP + k0 + 4]; al[ks][3] = dpl_s[(g8 + 8) * NHP + k0 + 4];
      }
    }
    float d1[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int colw = wi * CW + wc0 + 8 * nt + 2 * t4;   // column in the tile
      const float2 top = *reinterpret_cast<const float2*>(gxl + g8 * COLS + colw);
      const float2 bot = *reinterpret_cast<const float2*>(gxl + (g8 + 8) * COLS + colw);
      d1[nt][0] = top.x; d1[nt][1] = top.y; d1[nt][2] = bot.x; d1[nt][3] = bot.y;
    }
    if (DYN) {
      // k-step outer, n-tile inner: consecutive mma are independent
#pragma unroll
      for (int ks = 0; ks < 3; ++ks) {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma_tf32(d1[nt], al[ks], bph[nt][ks][0], bph[nt][ks][1]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma_tf32(d1[nt], ah[ks], bpl[nt][ks][0], bpl[nt][ks][1]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma_tf32(d1[nt], ah[ks], bph[nt][ks][0], bph[nt][ks][1]);
      }
    }
    if (nt_ == TOK) {
      // full stage: results back into gxl (same layout as the grad_x box), one TMA store
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int colw = wi * CW + wc0 + 8 * nt + 2 * t4;
        *reinterpret_cast<float2*>(gxl + g8 * COLS + colw) = make_float2(d1[nt][0], d1[nt][1]);
        *reinterpret_cast<float2*>(gxl + (g8 + 8) * COLS + colw) = make_float2(d1[nt][2], d1[nt][3]);
      }
      fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) {
        tma_store_2d(&omap, gxl, (int)c0, (int)(t0 * N));
        bulk_commit();
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        float* dst = gx + (t0 + g8) * nC + (int64_t)wi * C + c0 + wc0 + 8 * nt + 2 * t4;
        if (g8 < nt_) __stcs(reinterpret_cast<float2*>(dst), make_float2(d1[nt][0], d1[nt][1]));
        if (g8 + 8 < nt_) __stcs(reinterpret_cast<float2*>(dst + 8 * nC), make_float2(d1[nt][2], d1[nt][3]));
      }
    }
    // (C2) dphi^T += X^T . D_p over the 16 tokens (2 k-steps of 8 tokens)
    if (DYN) {
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const int tk = 8 * ks + t4;
        uint32_t bh[3][2], bl[3][2];
#pragma unroll
        for (int nt = 0; nt < 3; ++nt) {
          bh[nt][0] = dph_s[tk * NHP + 8 * nt + g8];       bl[nt][0] = dpl_s[tk * NHP + 8 * nt + g8];
          bh[nt][1] = dph_s[(tk + 4) * NHP + 8 * nt + g8]; bl[nt][1] = dpl_s[(tk + 4) * NHP + 8 * nt + g8];
        }
        uint32_t xh[2][4], xl[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const int cl = wc0 + 16 * mt + g8;   // channel of fragment row g8 (row g8+8 -> cl+8)
          split_tf32(xs[(tk * 4 + wi) * CW + cl], xh[mt][0], xl[mt][0]);
          split_tf32(xs[(tk * 4 + wi) * CW + cl + 8], xh[mt][1], xl[mt][1]);
          split_tf32(xs[((tk + 4) * 4 + wi) * CW + cl], xh[mt][2], xl[mt][2]);
          split_tf32(xs[((tk + 4) * 4 + wi) * CW + cl + 8], xh[mt][3], xl[mt][3]);
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < 3; ++nt) mma_tf32(acc2[mt][nt], xl[mt], bh[nt][0], bh[nt][1]);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < 3; ++nt) mma_tf32(acc2[mt][nt], xh[mt], bl[nt][0], bl[nt][1]);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int nt = 0; nt < 3; ++nt) mma_tf32(acc2[mt][nt], xh[mt], bh[nt][0], bh[nt][1]);
      }
    }
  }
  if (tid == 0) bulk_wait0();  // grad_x stores complete before the CTA's smem goes away
  if (failed) return;
  if (DYN) {
    // acc2[mt][nt]: rows = channels wc0+16mt+g8 (+8), cols = k 8nt+2t4 (+1)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 3; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 8 * nt + 2 * t4 + (e & 1);
          const int cl = wc0 + 16 * mt + g8 + (e >> 1) * 8;
          if (k < Lc::NH)
            dphi_part[((int64_t)split * Lc::NH + k) * nC + (int64_t)wi * C + c0 + cl] = acc2[mt][nt][e];
        }
  }
  // grad_w: reduce the 8 token lanes that share a channel (fixed order)
  gwS[ee * CW + ce] = gw0;
  gwS[ee * CW + ce + 32] = gw1;
  __syncthreads();
  if (tid < CW) {
    float sacc = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) sacc += gwS[k * CW + tid];
    gw_part[(int64_t)split * C + c0 + tid] = sacc;
  }
}

}  // namespace
}  // namespace mhc
