// Backward kernels 1 and 2: fp64 per-token moments and the closed-form
// per-token backward scalars (dynamic and static H).
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
// Backward 1: per-token moments gM = g x^T, W = g diag(w) x^T, G = x x^T.
//   One CTA (128 threads) per token, float4 over channel quads when VEC.
// ---------------------------------------------------------------------------
template <int V>
__device__ __forceinline__ void block_reduce_to_global(double (&acc)[V], double* smem,
                                                       double* __restrict__ dst) {
  // smem: [nwarps][V]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if constexpr (V == 32) {
    // transpose-reduce: each butterfly step hands half of the remaining values
    // to the partner lane, so after five steps lane l holds the warp's sum of
    // value l (31 shuffles instead of 32 x 5)
    double v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = acc[i];
#pragma unroll
    for (int o = 16, K = 32; o > 0; o >>= 1, K >>= 1) {
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < K / 2; ++i) {
        const double give = upper ? v[i] : v[i + K / 2];
        const double keep = upper ? v[i + K / 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, give, o);
      }
    }
    smem[warp * 32 + lane] = v[0];
    __syncthreads();
    if (threadIdx.x < 32) {
      double t = 0.0;
      for (int w = 0; w < nw; ++w) t += smem[w * 32 + threadIdx.x];
      dst[threadIdx.x] = t;
    }
    __syncthreads();
    return;
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    double s = acc[v];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) smem[warp * V + v] = s;
  }
  __syncthreads();
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    double s = 0.0;
    for (int w = 0; w < nw; ++w) s += smem[w * V + v];
    dst[v] = s;
  }
  __syncthreads();
}

template <int N, bool VEC, bool WITH_G, typename T = float>
__global__ void __launch_bounds__(128, 4)
    bwd_stats_kernel(const T* __restrict__ g, const T* __restrict__ x,
                     const float* __restrict__ w, double* __restrict__ stats, int64_t B,
                     int64_t C) {
  // Moments are accumulated in fp64: products of fp32 inputs are exact in
  // fp64, and the closed-form backward subtracts nearly equal moments (the
  // RMSNorm backward removes the radial component), which amplifies fp32
  // accumulation error by ~ the ratio |A_i| / |gh_i| (hundreds at cfg3).
  using Lc = L<N>;
  // dynamic H: the forward saved the fp64 Gram matrix, only gM and W are needed
  constexpr int NS1 = WITH_G ? Lc::NS1 : Lc::NSD;
  __shared__ double red[4 * NS1];
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    double acc[NS1];
#pragma unroll
    for (int v = 0; v < NS1; ++v) acc[v] = 0.0;
    const T* gb = g + b * N * C;
    const T* xb = x + b * N * C;
    auto accum = [&](const float (&gf)[N], const float (&xf)[N], float wf) {
      double gv[N], xv[N];
#pragma unroll
      for (int i = 0; i < N; ++i) { gv[i] = gf[i]; xv[i] = xf[i]; }
      const double wv = wf;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const double gw = gv[i] * wv;
#pragma unroll
        for (int j = 0; j < N; ++j) {
          acc[i * N + j] = fma(gv[i], xv[j], acc[i * N + j]);
          acc[N * N + i * N + j] = fma(gw, xv[j], acc[N * N + i * N + j]);
        }
      }
      if (WITH_G) {
        int e = 2 * N * N;
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int j = i; j < N; ++j) { acc[e] = fma(xv[i], xv[j], acc[e]); ++e; }
      }
    };
    if (VEC && !WITH_G) {
      // float4 per stream: with the Gram matrix left to the forward, 32
      // accumulators leave room for twice the loads in flight.
#pragma unroll 1
      for (int64_t q = threadIdx.x; q < C / 4; q += blockDim.x) {
        float4 g4[N], x4[N];
#pragma unroll
        for (int i = 0; i < N; ++i) {
          g4[i] = IO<T>::load4(gb + i * C, q);
          x4[i] = IO<T>::load4(xb + i * C, q);
        }
        const float4 w4 = __ldg(reinterpret_cast<const float4*>(w) + q);
        float gv[N], xv[N];
#pragma unroll
        for (int i = 0; i < N; ++i) { gv[i] = g4[i].x; xv[i] = x4[i].x; }
        accum(gv, xv, w4.x);
#pragma unroll
        for (int i = 0; i < N; ++i) { gv[i] = g4[i].y; xv[i] = x4[i].y; }
        accum(gv, xv, w4.y);
#pragma unroll
        for (int i = 0; i < N; ++i) { gv[i] = g4[i].z; xv[i] = x4[i].z; }
        accum(gv, xv, w4.z);
#pragma unroll
        for (int i = 0; i < N; ++i) { gv[i] = g4[i].w; xv[i] = x4[i].w; }
        accum(gv, xv, w4.w);
      }
    } else if constexpr (sizeof(T) == 4) {
      if (VEC) {
      // float2 per stream: keeps the live load registers low enough for
      // 4 CTAs (16 warps) per SM next to the 42 fp64 accumulators.
#pragma unroll 2
      for (int64_t q = threadIdx.x; q < C / 2; q += blockDim.x) {
        float2 g2[N], x2[N];
#pragma unroll
        for (int i = 0; i < N; ++i) {
          g2[i] = __ldcs(reinterpret_cast<const float2*>(gb + i * C) + q);
          x2[i] = __ldcs(reinterpret_cast<const float2*>(xb + i * C) + q);
        }
        const float2 w2 = __ldg(reinterpret_cast<const float2*>(w) + q);
        float gv[N], xv[N];
#pragma unroll
        for (int i = 0; i < N; ++i) { gv[i] = g2[i].x; xv[i] = x2[i].x; }
        accum(gv, xv, w2.x);
#pragma unroll
        for (int i = 0; i < N; ++i) { gv[i] = g2[i].y; xv[i] = x2[i].y; }
        accum(gv, xv, w2.y);
      }
    } else {
      for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
        float gv[N], xv[N];
#pragma unroll
        for (int i = 0; i < N; ++i) { gv[i] = gb[i * C + c]; xv[i] = xb[i * C + c]; }
        accum(gv, xv, w[c]);
      }
    }
    }
    block_reduce_to_global<NS1>(acc, red, stats + b * NS1);
  }
}

// Backward 1 of MHCResidualWrapper (dynamic H, fp32): the moments gM and W of
// the layer's streams without the streams in memory.  The layer's upstream
// gradient is the mean's reverse, g[i, c] = gmean[c] / n for every stream
// (as the framework's mean backward divides), and stream j is sc.s[j] *
// residual (j != 1) or the branch output, as the forward packed them.
template <int N>
__global__ void __launch_bounds__(128, 4)
    wrap_bwd_stats_kernel(const float* __restrict__ gmean, const float* __restrict__ res,
                          const float* __restrict__ br, WrapScales sc,
                          const float* __restrict__ w, double* __restrict__ stats, int64_t B,
                          int64_t C) {
  using Lc = L<N>;
  constexpr int NS = Lc::NSD;
  __shared__ double red[4 * NS];
  const float nf = (float)N;
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    double acc[NS];
#pragma unroll
    for (int v = 0; v < NS; ++v) acc[v] = 0.0;
    const float4* gb = reinterpret_cast<const float4*>(gmean + b * C);
    const float4* rb = reinterpret_cast<const float4*>(res + b * C);
    const float4* bb = reinterpret_cast<const float4*>(br + b * C);
    auto accum = [&](float gq, float rq, float bq, float wq) {
      const float gv = gq / nf;
      double xv[N];
#pragma unroll
      for (int j = 0; j < N; ++j) xv[j] = (double)(j == 1 ? bq : sc.s[j] * rq);
      const double g = gv, gw = (double)gv * (double)wq;
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = 0; j < N; ++j) {
          acc[i * N + j] = fma(g, xv[j], acc[i * N + j]);
          acc[N * N + i * N + j] = fma(gw, xv[j], acc[N * N + i * N + j]);
        }
    };
    const int64_t C4 = C / 4, NT = blockDim.x;
    float4 g0, r0, b0, g1, r1, b1;
    int64_t q = threadIdx.x;
    if (q < C4) { g0 = __ldcs(gb + q); r0 = __ldcs(rb + q); b0 = __ldcs(bb + q); }
#pragma unroll 1
    for (; q < C4; q += 2 * NT) {
      if (q + NT < C4) { g1 = __ldcs(gb + q + NT); r1 = __ldcs(rb + q + NT); b1 = __ldcs(bb + q + NT); }
      {
        const float4 w4 = __ldg(reinterpret_cast<const float4*>(w) + q);
        accum(g0.x, r0.x, b0.x, w4.x); accum(g0.y, r0.y, b0.y, w4.y);
        accum(g0.z, r0.z, b0.z, w4.z); accum(g0.w, r0.w, b0.w, w4.w);
      }
      if (q + 2 * NT < C4) { g0 = __ldcs(gb + q + 2 * NT); r0 = __ldcs(rb + q + 2 * NT); b0 = __ldcs(bb + q + 2 * NT); }
      if (q + NT < C4) {
        const float4 w4 = __ldg(reinterpret_cast<const float4*>(w) + q + NT);
        accum(g1.x, r1.x, b1.x, w4.x); accum(g1.y, r1.y, b1.y, w4.y);
        accum(g1.z, r1.z, b1.z, w4.z); accum(g1.w, r1.w, b1.w, w4.w);
      }
    }
    block_reduce_to_global<NS>(acc, red, stats + b * NS);
  }
}

// ---------------------------------------------------------------------------
// Backward 2 (dynamic): per-token closed-form scalars, one group of lanes per
// token (the Sinkhorn reverse runs one matrix row per lane, the rest is
// evaluated alike by every lane of the group and written by its first lane),
// in fp64.  With W = g diag(w) x^T, G = x x^T, gM = g x^T (sums over c):
//     ghp_i = (W h)_i / r                     (= sum_c g_i y)
//     dot   = hp^T W h                        (= sum_c gy w x_agg)
//     A_i   = (W^T hp)_i                      (= sum_c gy w x_i)
//     Q_i   = (G h)_i                         (= sum_c x_agg x_i)
//     beta  = dot / (C r^3);  gh_i = A_i / r - beta Q_i   (= sum_c gx_agg x_i)
//   then the gate derivatives, the Sinkhorn reverse on gM, and the projection
//   backward: d_p = dt alpha / rms_h, coef = -(sum dt alpha p) / (rms_h^3 nC).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo);
__host__ __device__ __forceinline__ uint32_t umma_kmaj_off(int r, int k, int R);

// Operand image of each token block from the per-token backward rows:
// D_p hi/lo as the K-major [TOK tokens x 24] B operand of D1 and as the
// K-major [32 (k, zero-padded) x TOK tokens] B operand of D2, and 32 scalars
// per token (beta, inv_r, coef, 0, h[4], h_post[4], M^T[16], 0[4]).  Tokens
// past B are zero.
__device__ __forceinline__ void gx_image_row(const float* __restrict__ tb, float* __restrict__ img,
                                             int64_t t) {
  // tb: the token's backward row, or nullptr for a padding token (zeros)
  using Lc = L<4>;
  using F = Gx6Cfg;
  const bool live = tb != nullptr;
  float* im = img + (t / F::TOK) * F::IMG_FLOATS;
  const int tt = (int)(t % F::TOK);
#pragma unroll
  for (int k = 0; k < F::KP; ++k) {
    const float d = (live && k < F::NH) ? tb[4 + k] : 0.f;
    uint32_t hi, lo;
    split_tf32(d, hi, lo);
    if (k < F::NH) {
      const uint32_t o1 = umma_kmaj_off(tt, k, F::TOK) / 4;
      im[F::IMG_B1H + o1] = __uint_as_float(hi);
      im[F::IMG_B1L + o1] = __uint_as_float(lo);
    }
    const uint32_t o2 = umma_kmaj_off(k, tt, F::KP) / 4;
    im[F::IMG_B2H + o2] = __uint_as_float(hi);
    im[F::IMG_B2L + o2] = __uint_as_float(lo);
  }
  float* sc = im + F::IMG_SC + tt * 32;
  float v[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) v[e] = 0.f;
  if (live) {
    v[0] = tb[0]; v[1] = tb[1]; v[2] = tb[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) { v[4 + i] = tb[Lc::OFF_TH + i]; v[8 + i] = tb[Lc::OFF_THP + i]; }
#pragma unroll
    for (int e = 0; e < 16; ++e) v[12 + e] = tb[Lc::OFF_TM + e];
  }
#pragma unroll
  for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4*>(sc + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
}

template <int N>
__global__ void __launch_bounds__(128)
    token_bwd_lanes_kernel(const double* __restrict__ stats, const float* __restrict__ rec,
                     const float* __restrict__ a_pre, const float* __restrict__ a_post,
                     const float* __restrict__ a_res, const float* __restrict__ b_pre,
                     const float* __restrict__ b_post, const float* __restrict__ b_res,
                     float* __restrict__ tokb, double* __restrict__ tokr, int64_t B, int64_t C,
                     int iters, float s_eps, float r_eps, unsigned int* __restrict__ counter,
                     float* __restrict__ img, int64_t img_tokens) {
  using Lc = L<N>;
  constexpr int NH = Lc::NH, NSD = Lc::NSD;
  if (blockIdx.x == 0 && threadIdx.x == 0) *counter = 0u;  // arrival counter of finish_dyn_bwd
  constexpr int LG = N <= 2 ? 2 : (N <= 4 ? 4 : 8);  // lanes per token
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int row = (int)(threadIdx.x & (LG - 1));
  const int base = (int)(threadIdx.x & 31) & ~(LG - 1);
  const int64_t b = gt / LG;
  const bool live = b < B;
  // every lane of the warp takes part in the shuffles: dead groups evaluate
  // the last token and write nothing
  const int64_t bb = live ? b : B - 1;
  const double* st = stats + bb * NSD;
  const float* rc = rec + bb * Lc::REC;
  const double* G = reinterpret_cast<const double*>(rc + Lc::OFF_G64);  // fp64 Gram saved by the forward
  // The H_pre gradient is the small difference of two large moments (the
  // RMSNorm backward removes the radial part of the upstream gradient), so it
  // is sensitive to the exact gate values: recompute rms_h, h, hp and r in
  // fp64 from the saved projections p and the forward's fp64 Gram matrix
  // instead of reusing the fp32 values of the forward record.
  double tr_g = 0.0;
#pragma unroll
  for (int i = 0; i < N; ++i) tr_g += G[gram_index(i, i, N)];
  const double rms_h = sqrt(tr_g / (double)(N * C) + (double)r_eps);
  const double inv_h = 1.0 / rms_h;
  const double ap = *a_pre, aq = *a_post, ar = *a_res;
  // gate `row` on this lane, then shared over the group
  const int gi = row < N ? row : 0;
  const double h_mine = 1.0 / (1.0 + exp(-((ap * (double)rc[Lc::OFF_P + gi]) * inv_h + (double)b_pre[gi])));
  const double hp_mine = 2.0 / (1.0 + exp(-((aq * (double)rc[Lc::OFF_P + N + gi]) * inv_h + (double)b_post[gi])));
  double h[N], hp[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    h[i] = __shfl_sync(0xffffffffu, h_mine, base + i);
    hp[i] = __shfl_sync(0xffffffffu, hp_mine, base + i);
  }
  double q = 0.0;
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) q += h[i] * h[j] * G[gram_index(i, j, N)];
  const double r = sqrt(q / (double)C + (double)r_eps);
  const double inv_r = 1.0 / r;
  double dt[NH];
  double dot = 0.0;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    double wh = 0.0;
#pragma unroll
    for (int j = 0; j < N; ++j) wh = fma(st[N * N + i * N + j], h[j], wh);
    dot = fma(hp[i], wh, dot);
    dt[N + i] = wh * inv_r * hp[i] * (1.0 - 0.5 * hp[i]);
  }
  const double beta = dot / ((double)C * r * r * r);
#pragma unroll
  for (int i = 0; i < N; ++i) {
    double A = 0.0, Q = 0.0;
#pragma unroll
    for (int k = 0; k < N; ++k) A = fma(hp[k], st[N * N + k * N + i], A);
#pragma unroll
    for (int j = 0; j < N; ++j) Q = fma(G[gram_index(i, j, N)], h[j], Q);
    dt[i] = (A * inv_r - beta * Q) * h[i] * (1.0 - h[i]);
  }
  // Sinkhorn reverse with lane `row` of the group holding that row
  double e0[N], gm[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    e0[j] = row < N ? exp((ar * (double)rc[Lc::OFF_P + 2 * N + row * N + j]) * inv_h + (double)b_res[row * N + j]) : 0.0;
    gm[j] = row < N ? st[row * N + j] : 0.0;
  }
  skl_backward<N, LG, double>(e0, gm, iters, (double)s_eps, row);
#pragma unroll
  for (int rr = 0; rr < N; ++rr)
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const double v = __shfl_sync(0xffffffffu, gm[j] * e0[j], base + rr);
      dt[2 * N + rr * N + j] = v;
    }
  if (row != 0) return;
  if (!live) {
    // padding tokens of the last operand-image block
    if constexpr (N == 4) { if (img != nullptr && b < img_tokens) gx_image_row(nullptr, img, b); }
    return;
  }
  float* tb = tokb + b * Lc::TB;
  double* tr = tokr + b * Lc::NR;
  double s = 0.0, da0 = 0.0, da1 = 0.0, da2 = 0.0;
#pragma unroll
  for (int k = 0; k < NH; ++k) {
    const double a = k < N ? ap : (k < 2 * N ? aq : ar);
    const double pk = rc[Lc::OFF_P + k];
    tb[4 + k] = (float)(dt[k] * a * inv_h);
    s = fma(dt[k] * a, pk, s);
    const double dak = dt[k] * pk * inv_h;
    if (k < N) da0 += dak; else if (k < 2 * N) da1 += dak; else da2 += dak;
    tr[k] = dt[k];
  }
#pragma unroll
  for (int k = NH; k < Lc::NHP; ++k) tb[4 + k] = 0.f;
  tb[0] = (float)beta;
  tb[1] = (float)inv_r;
  tb[2] = (float)(-s * inv_h * inv_h * inv_h / (double)(N * C));
  tb[3] = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    tb[Lc::OFF_TH + i] = (float)h[i];
    tb[Lc::OFF_THP + i] = (float)hp[i];
  }
#pragma unroll
  for (int e = 0; e < N * N; ++e) tb[Lc::OFF_TM + (e % N) * N + e / N] = rc[Lc::OFF_M + e];
#pragma unroll
  for (int e = Lc::OFF_TM + N * N; e < Lc::TB; ++e) tb[e] = 0.f;
  tr[NH + 0] = da0;
  tr[NH + 1] = da1;
  tr[NH + 2] = da2;
  if constexpr (N == 4) {
    if (img != nullptr) gx_image_row(tb, img, b);
  }
}

// Static-H per-token scalars (fp64): beta, inv_r for grad_x, and per-token
// gate gradients (dt_pre, dt_post) and gM for the reductions over the batch.
template <int N>
__global__ void __launch_bounds__(128)
    token_bwd_static_kernel(const double* __restrict__ stats, const float* __restrict__ H_pre,
                            const float* __restrict__ H_post, const float* __restrict__ rec,
                            float* __restrict__ tokb,
                            double* __restrict__ tokr, int64_t B, int64_t C, float r_eps) {
  using Lc = L<N>;
  constexpr int NS1 = Lc::NS1;
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const double* st = stats + b * NS1;
  const double* G = st + 2 * N * N;
  // gates and r in fp64 (see token_bwd_lanes_kernel for why)
  double h[N], hp[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    h[i] = 1.0 / (1.0 + exp(-(double)H_pre[i]));
    hp[i] = 2.0 / (1.0 + exp(-(double)H_post[i]));
  }
  double q = 0.0;
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) q += h[i] * h[j] * G[gram_index(i, j, N)];
  const double r = sqrt(q / (double)C + (double)r_eps);
  const double inv_r = 1.0 / r;
  double* tr = tokr + b * Lc::NRS;
  double dot = 0.0;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    double wh = 0.0;
#pragma unroll
    for (int j = 0; j < N; ++j) wh = fma(st[N * N + i * N + j], h[j], wh);
    dot = fma(hp[i], wh, dot);
    tr[N + i] = wh * inv_r * hp[i] * (1.0 - 0.5 * hp[i]);
  }
  const double beta = dot / ((double)C * r * r * r);
#pragma unroll
  for (int i = 0; i < N; ++i) {
    double A = 0.0, Q = 0.0;
#pragma unroll
    for (int k = 0; k < N; ++k) A = fma(hp[k], st[N * N + k * N + i], A);
#pragma unroll
    for (int j = 0; j < N; ++j) Q = fma(st[2 * N * N + gram_index(i, j, N)], h[j], Q);
    tr[i] = (A * inv_r - beta * Q) * h[i] * (1.0 - h[i]);
  }
#pragma unroll
  for (int e = 0; e < N * N; ++e) tr[2 * N + e] = st[e];
  float* tb = tokb + b * Lc::TB;
  tb[0] = (float)beta;
  tb[1] = (float)inv_r;
  tb[2] = 0.f;
  tb[3] = 0.f;
#pragma unroll
  for (int k = 0; k < Lc::NHP; ++k) tb[4 + k] = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    tb[Lc::OFF_TH + i] = (float)h[i];
    tb[Lc::OFF_THP + i] = (float)hp[i];
  }
#pragma unroll
  for (int e = 0; e < N * N; ++e) tb[Lc::OFF_TM + (e % N) * N + e / N] = rec[Lc::OFF_M + e];
#pragma unroll
  for (int e = Lc::OFF_TM + N * N; e < Lc::TB; ++e) tb[e] = 0.f;
}

}  // namespace
}  // namespace mhc
