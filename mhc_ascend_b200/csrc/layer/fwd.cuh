// Forward kernels: FFMA / TMA projections (fallbacks), per-token gates and
// Sinkhorn, the streaming output pass, and the static-H forward.
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
// Forward 1: projections and Gram moments, split over channel ranges.
//   CTA = 8 warps; warp w owns TPW tokens, lane owns one channel of each
//   32-channel chunk.  phi for the chunk is staged in shared memory
//   [32 ch][N][NHP] (row stride = SROW floats, == 4 mod 32 for conflict-free
//   float4 reads) and reused by the CTA's 8*TPW tokens.
// ---------------------------------------------------------------------------
template <int N>
struct ProjCfg {
  static constexpr int TPW = N <= 4 ? 4 : 1;
  static constexpr int TT = 8 * TPW;  // tokens per CTA
  static constexpr int ROW = N * L<N>::NHP;
  static constexpr int SROW = (ROW + 27) / 32 * 32 + 4;  // >= ROW, == 4 (mod 32)
  static constexpr int SMEM_FLOATS = 2 * 32 * SROW;
};

template <int N>
__global__ void __launch_bounds__(256, 1)
    proj_stats_kernel(const float* __restrict__ x, const float* __restrict__ phi_pre,
                      const float* __restrict__ phi_post, const float* __restrict__ phi_res,
                      float* __restrict__ ppart, float* __restrict__ gpart, int64_t B, int64_t C,
                      int cps) {
  using Lc = L<N>;
  using P = ProjCfg<N>;
  constexpr int NHP = Lc::NHP, NH = Lc::NH, NG = Lc::NG, TPW = P::TPW, SROW = P::SROW;
  extern __shared__ float smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t nC = (int64_t)N * C;
  const int64_t t0 = (int64_t)blockIdx.x * P::TT + warp * TPW;
  const int split = blockIdx.y;
  const int64_t c_begin = (int64_t)split * cps;
  int64_t c_end = c_begin + cps;
  if (c_end > C) c_end = C;

  float acc[TPW][NHP];
  float gacc[TPW][NG];
#pragma unroll
  for (int t = 0; t < TPW; ++t) {
#pragma unroll
    for (int k = 0; k < NHP; ++k) acc[t][k] = 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g) gacc[t][g] = 0.f;
  }

  // cooperative phi staging: element e of the chunk -> (k, i, ch)
  auto stage = [&](int buf, int64_t cc) {
    float* dst = smem + buf * 32 * SROW;
    for (int e = threadIdx.x; e < NHP * N * 32; e += blockDim.x) {
      const int ch = e & 31;
      const int ki = e >> 5;  // k * N + i
      const int k = ki / N, i = ki % N;
      const int64_t c = cc + ch;
      float v = 0.f;
      if (k < NH && c < c_end) v = __ldg(phi_row(phi_pre, phi_post, phi_res, k, N, nC) + i * C + c);
      dst[ch * SROW + i * NHP + k] = v;
    }
  };

  float xv[TPW][N], xn[TPW][N];
  auto load_x = [&](float (&dst)[TPW][N], int64_t cc) {
    const int64_t c = cc + lane;
#pragma unroll
    for (int t = 0; t < TPW; ++t) {
      const int64_t tok = t0 + t;
#pragma unroll
      for (int i = 0; i < N; ++i)
        dst[t][i] = (tok < B && c < c_end) ? __ldcs(x + tok * nC + (int64_t)i * C + c) : 0.f;
    }
  };

  if (c_begin < c_end) {
    stage(0, c_begin);
    load_x(xv, c_begin);
  }
  __syncthreads();
  int buf = 0;
  for (int64_t cc = c_begin; cc < c_end; cc += 32) {
    const bool more = cc + 32 < c_end;
    if (more) {
      stage(buf ^ 1, cc + 32);
      load_x(xn, cc + 32);
    }
    const float* row = smem + buf * 32 * SROW + lane * SROW;
#pragma unroll
    for (int i = 0; i < N; ++i) {
#pragma unroll
      for (int k4 = 0; k4 < NHP / 4; ++k4) {
        const float4 f = *reinterpret_cast<const float4*>(row + i * NHP + 4 * k4);
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
          acc[t][4 * k4 + 0] = fmaf(xv[t][i], f.x, acc[t][4 * k4 + 0]);
          acc[t][4 * k4 + 1] = fmaf(xv[t][i], f.y, acc[t][4 * k4 + 1]);
          acc[t][4 * k4 + 2] = fmaf(xv[t][i], f.z, acc[t][4 * k4 + 2]);
          acc[t][4 * k4 + 3] = fmaf(xv[t][i], f.w, acc[t][4 * k4 + 3]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < TPW; ++t) {
      int g = 0;
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = i; j < N; ++j) {
          gacc[t][g] = fmaf(xv[t][i], xv[t][j], gacc[t][g]);
          ++g;
        }
    }
    if (more) {
#pragma unroll
      for (int t = 0; t < TPW; ++t)
#pragma unroll
        for (int i = 0; i < N; ++i) xv[t][i] = xn[t][i];
    }
    __syncthreads();
    buf ^= 1;
  }

  // reduce over the 32 lanes (channels) and write this split's partials
#pragma unroll
  for (int t = 0; t < TPW; ++t) {
    const int64_t tok = t0 + t;
#pragma unroll
    for (int k = 0; k < NHP; ++k) {
      const float v = warp_sum(acc[t][k]);
      if (lane == (k & 31) && tok < B) ppart[((int64_t)split * B + tok) * NHP + k] = v;
    }
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const float v = warp_sum(gacc[t][g]);
      if (lane == (g & 31) && tok < B) gpart[((int64_t)split * B + tok) * NG + g] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Forward 1, TMA-pipelined (n <= 4, C % 4 == 0, 16-byte aligned x): the same
// split-K projection + Gram as proj_stats_kernel, with the x chunk
// [32 tokens x n streams][32 channels] and the transposed phi chunk
// [32 channels][PROW] brought into a PJT_STAGES-deep ring by TMA.  phiT is
// phi rearranged per channel: phiT[c][i*NHP + k] = phi_k[i*C + c], rows padded
// to PROW = n*NHP + 4 floats so the per-lane float4 reads hit distinct banks.
// ---------------------------------------------------------------------------
constexpr int PJT_STAGES = 4;

template <int N>
struct PjtCfg {
  static constexpr int NHP = L<N>::NHP;
  static constexpr int PROW = N * NHP + 4;
  static constexpr int TT = 32;                           // tokens per CTA
  static constexpr int XF = TT * N * 32;                  // x floats per stage
  static constexpr int PF = 32 * PROW;                    // phiT floats per stage
  static constexpr uint32_t STAGE_BYTES = (XF + PF) * 4;
  static constexpr size_t SMEM = (size_t)PJT_STAGES * STAGE_BYTES + 128 + 64;
};

template <int N>
__global__ void phi_transpose_kernel(const float* __restrict__ pp, const float* __restrict__ pq,
                                     const float* __restrict__ pr, float* __restrict__ phiT,
                                     int64_t C) {
  using P = PjtCfg<N>;
  constexpr int NH = L<N>::NH, NHP = L<N>::NHP;
  const int64_t total = C * P::PROW;
  const int64_t nC = (int64_t)N * C;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = e / P::PROW;
    const int f = (int)(e % P::PROW);
    float v = 0.f;
    if (f < N * NHP) {
      const int i = f / NHP, k = f % NHP;
      if (k < NH) v = phi_row(pp, pq, pr, k, N, nC)[(int64_t)i * C + c];
    }
    phiT[e] = v;
  }
}

constexpr int PJT_THREADS = 512;  // 16 warps x 2 tokens

template <int N>
__global__ void __launch_bounds__(PJT_THREADS, 1)
    proj_stats_tma_kernel(const __grid_constant__ CUtensorMap xmap,
                          const __grid_constant__ CUtensorMap pmap, float* __restrict__ ppart,
                          float* __restrict__ gpart, int64_t B, int64_t C, int cps) {
  using Lc = L<N>;
  using P = PjtCfg<N>;
  constexpr int NHP = Lc::NHP, NG = Lc::NG, TPW = P::TT / (PJT_THREADS / 32), PROW = P::PROW;
  extern __shared__ unsigned char smem_raw[];
  float* ring = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + PJT_STAGES * (P::XF + P::PF));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t tile_t0 = (int64_t)blockIdx.x * P::TT;
  const int64_t t0 = tile_t0 + warp * TPW;
  const int split = blockIdx.y;
  const int64_t c_begin = (int64_t)split * cps;
  const int64_t c_end = c_begin + cps < C ? c_begin + cps : C;
  const int nchunks = c_begin < c_end ? (int)((c_end - c_begin + 31) / 32) : 0;

  if (threadIdx.x == 0) {
    prefetch_tmap(&xmap);
    prefetch_tmap(&pmap);
    for (int st = 0; st < PJT_STAGES; ++st) mbar_init(&bars[st], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int k) {
    const int slot = k % PJT_STAGES;
    float* base = ring + slot * (P::XF + P::PF);
    const int cc = (int)(c_begin + 32 * k);
    mbar_expect_tx(&bars[slot], P::STAGE_BYTES);
    tma_load_2d(base, &xmap, cc, (int)(tile_t0 * N), &bars[slot]);
    tma_load_2d(base + P::XF, &pmap, 0, cc, &bars[slot]);
  };
  if (threadIdx.x == 0)
    for (int k = 0; k < PJT_STAGES && k < nchunks; ++k) issue(k);

  float acc[TPW][NHP];
  float gacc[TPW][NG];
#pragma unroll
  for (int t = 0; t < TPW; ++t) {
#pragma unroll
    for (int k = 0; k < NHP; ++k) acc[t][k] = 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g) gacc[t][g] = 0.f;
  }
  for (int k = 0; k < nchunks; ++k) {
    const int slot = k % PJT_STAGES;
    const bool ok = threadIdx.x == 0 ? mbar_wait(&bars[slot], (uint32_t)((k / PJT_STAGES) & 1)) : true;
    if (__syncthreads_or(!ok)) return;
    const float* xs = ring + slot * (P::XF + P::PF);
    const float* row = xs + P::XF + lane * PROW;
    float xv[TPW][N];
#pragma unroll
    for (int t = 0; t < TPW; ++t)
#pragma unroll
      for (int i = 0; i < N; ++i) xv[t][i] = xs[((warp * TPW + t) * N + i) * 32 + lane];
#pragma unroll
    for (int i = 0; i < N; ++i) {
#pragma unroll
      for (int k4 = 0; k4 < NHP / 4; ++k4) {
        const float4 f = *reinterpret_cast<const float4*>(row + i * NHP + 4 * k4);
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
          acc[t][4 * k4 + 0] = fmaf(xv[t][i], f.x, acc[t][4 * k4 + 0]);
          acc[t][4 * k4 + 1] = fmaf(xv[t][i], f.y, acc[t][4 * k4 + 1]);
          acc[t][4 * k4 + 2] = fmaf(xv[t][i], f.z, acc[t][4 * k4 + 2]);
          acc[t][4 * k4 + 3] = fmaf(xv[t][i], f.w, acc[t][4 * k4 + 3]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < TPW; ++t) {
      int g = 0;
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = i; j < N; ++j) {
          gacc[t][g] = fmaf(xv[t][i], xv[t][j], gacc[t][g]);
          ++g;
        }
    }
    __syncthreads();  // slot consumed: refill it
    if (threadIdx.x == 0 && k + PJT_STAGES < nchunks) issue(k + PJT_STAGES);
  }
#pragma unroll
  for (int t = 0; t < TPW; ++t) {
    const int64_t tok = t0 + t;
#pragma unroll
    for (int k = 0; k < NHP; ++k) {
      const float v = warp_sum(acc[t][k]);
      if (lane == (k & 31) && tok < B) ppart[((int64_t)split * B + tok) * NHP + k] = v;
    }
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const float v = warp_sum(gacc[t][g]);
      if (lane == (g & 31) && tok < B) gpart[((int64_t)split * B + tok) * NG + g] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Forward 2: per-token gates, Sinkhorn and RMS (a group of lanes per token:
// the Sinkhorn runs one row of M per lane, the rest is written by the first).
// ---------------------------------------------------------------------------
// SUMSQ: the projection supplied only the sum of squares per split
// (gpart = [ks][B]); r is then computed by stream_fwd_r_kernel.
template <int N, bool SUMSQ = false>
__global__ void __launch_bounds__(128)
    token_fwd_lanes_kernel(const float* __restrict__ ppart, const float* __restrict__ gpart, int ks,
                     const float* __restrict__ a_pre, const float* __restrict__ a_post,
                     const float* __restrict__ a_res, const float* __restrict__ b_pre,
                     const float* __restrict__ b_post, const float* __restrict__ b_res,
                     float* __restrict__ rec, int64_t B, int64_t C, int iters, float s_eps,
                     float r_eps) {
  using Lc = L<N>;
  constexpr int NH = Lc::NH, NHP = Lc::NHP, NG = Lc::NG;
  constexpr int LG = N <= 2 ? 2 : (N <= 4 ? 4 : 8);  // lanes per token
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int row = (int)(threadIdx.x & (LG - 1));
  const int64_t bt = gt / LG;
  const bool live = bt < B;
  // every lane of the warp takes part in the shuffles: dead groups evaluate
  // the last token and write nothing
  const int64_t b = live ? bt : B - 1;
  float p[NH], G[SUMSQ ? 1 : NG];
#pragma unroll
  for (int k = 0; k < NH; ++k) p[k] = 0.f;
#pragma unroll
  for (int g = 0; g < (SUMSQ ? 1 : NG); ++g) G[g] = 0.f;
  for (int s = 0; s < ks; ++s) {
    const float* pp = ppart + ((int64_t)s * B + b) * NHP;
#pragma unroll
    for (int k = 0; k < NH; ++k) p[k] += pp[k];
    if constexpr (SUMSQ) {
      G[0] += gpart[(int64_t)s * B + b];
    } else {
      const float* gp = gpart + ((int64_t)s * B + b) * NG;
#pragma unroll
      for (int g = 0; g < NG; ++g) G[g] += gp[g];
    }
  }
  float ss = 0.f;
  if constexpr (SUMSQ) {
    ss = G[0];
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) ss += G[gram_index(i, i, N)];
  }
  const float rms_h = sqrtf(ss / (float)(N * C) + r_eps);
  const float inv_h = 1.f / rms_h;
  const float ap = *a_pre, aq = *a_post, ar = *a_res;
  float h[N], hp[N], m[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    h[i] = sigmoidf_((ap * p[i]) * inv_h + b_pre[i]);
    hp[i] = 2.f * sigmoidf_((aq * p[N + i]) * inv_h + b_post[i]);
  }
  // Sinkhorn with lane `row` of the group holding that row of M
#pragma unroll
  for (int j = 0; j < N; ++j)
    m[j] = row < N ? expf((ar * p[2 * N + row * N + j]) * inv_h + b_res[row * N + j]) : 0.f;
  skl_forward<N, LG, float>(m, iters, s_eps, row);
  if (!live) return;
  float* o = rec + b * Lc::REC;
  if (row < N) {
#pragma unroll
    for (int j = 0; j < N; ++j) o[Lc::OFF_M + row * N + j] = m[j];
  }
  if (row != 0) return;
  o[0] = rms_h;
  if constexpr (!SUMSQ) {
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) q += h[i] * h[j] * G[gram_index(i, j, N)];
    o[1] = sqrtf(fmaxf(q, 0.f) / (float)C + r_eps);
  }
#pragma unroll
  for (int i = 0; i < N; ++i) {
    o[Lc::OFF_H + i] = h[i];
    o[Lc::OFF_HP + i] = hp[i];
  }
#pragma unroll
  for (int k = 0; k < NH; ++k) o[Lc::OFF_P + k] = p[k];
}

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> struct IO;
template <> struct IO<float> {
  // raw4: four elements as stored (kept in registers until used)
  using raw4 = float4;
  static __device__ __forceinline__ raw4 load_raw4(const float* p, int64_t q) {
    return __ldcs(reinterpret_cast<const float4*>(p) + q);
  }
  static __device__ __forceinline__ float4 to_f4(raw4 r) { return r; }
  static __device__ __forceinline__ float4 load4(const float* p, int64_t q) {
    return __ldcs(reinterpret_cast<const float4*>(p) + q);
  }
  static __device__ __forceinline__ void store4(float* p, int64_t q, float4 v) {
    __stcs(reinterpret_cast<float4*>(p) + q, v);
  }
};
template <> struct IO<__nv_bfloat16> {
  using raw4 = uint2;
  static __device__ __forceinline__ raw4 load_raw4(const __nv_bfloat16* p, int64_t q) {
    return __ldcs(reinterpret_cast<const uint2*>(p) + q);
  }
  static __device__ __forceinline__ float4 to_f4(raw4 u) {
    // bf16 -> fp32 is a 16-bit shift
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
  }
  static __device__ __forceinline__ float4 load4(const __nv_bfloat16* p, int64_t q) {
    const uint2 u = __ldcs(reinterpret_cast<const uint2*>(p) + q);
    __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
    return make_float4(a.x, a.y, b.x, b.y);
  }
  static __device__ __forceinline__ void store4(__nv_bfloat16* p, int64_t q, float4 v) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    __stcs(reinterpret_cast<uint2*>(p) + q, u);
  }
};

// ---------------------------------------------------------------------------
// Forward 3: out[i,c] = sum_j M_ij x[j,c] + hp_i * (w_c / r) * sum_j h_j x[j,c]
//   One CTA per token (grid-stride over tokens); per-token record in smem;
//   rec_stride 0 = one shared record (static H) with per-token r from rms[].
// ---------------------------------------------------------------------------
template <int N, bool VEC, bool GRAM, typename T = float>
__global__ void __launch_bounds__(256)
    stream_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w,
                      const float* __restrict__ rec, int rec_stride,
                      const float* __restrict__ rms, T* __restrict__ out, int64_t B,
                      int64_t C, float* __restrict__ rec_w) {
  static_assert(VEC || sizeof(T) == 4, "bf16 streams use the vector path");
  // GRAM (dynamic H): also the token's Gram matrix in fp64 from exact
  // products, for the backward -- FP64 work hidden under this HBM-bound pass.
  using Lc = L<N>;
  constexpr int NG = Lc::NG;
  __shared__ float s_rec[Lc::REC];
  __shared__ double s_g[GRAM ? 8 * NG : 1];
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    __syncthreads();
    for (int e = threadIdx.x; e < Lc::REC; e += blockDim.x) s_rec[e] = rec[b * rec_stride + e];
    __syncthreads();
    const float r = rms ? rms[b] : s_rec[1];
    const float inv_r = 1.f / r;
    const float* h = s_rec + Lc::OFF_H;
    const float* hp = s_rec + Lc::OFF_HP;
    const float* m = s_rec + Lc::OFF_M;
    const T* xb = x + b * N * C;
    T* ob = out + b * N * C;
    double gacc[NG];
#pragma unroll
    for (int g = 0; g < NG; ++g) gacc[g] = 0.0;
    if (VEC) {
      for (int64_t q = threadIdx.x; q < C / 4; q += blockDim.x) {
        float4 xv[N];
#pragma unroll
        for (int j = 0; j < N; ++j) xv[j] = IO<T>::load4(xb + j * C, q);
        if (GRAM) {
          int g = 0;
#pragma unroll
          for (int i = 0; i < N; ++i)
#pragma unroll
            for (int j = i; j < N; ++j) {
              gacc[g] = fma((double)xv[i].x, (double)xv[j].x, gacc[g]);
              gacc[g] = fma((double)xv[i].y, (double)xv[j].y, gacc[g]);
              gacc[g] = fma((double)xv[i].z, (double)xv[j].z, gacc[g]);
              gacc[g] = fma((double)xv[i].w, (double)xv[j].w, gacc[g]);
              ++g;
            }
        }
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + q);
        float4 xa = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < N; ++j) {
          xa.x = fmaf(h[j], xv[j].x, xa.x); xa.y = fmaf(h[j], xv[j].y, xa.y);
          xa.z = fmaf(h[j], xv[j].z, xa.z); xa.w = fmaf(h[j], xv[j].w, xa.w);
        }
        float4 y;
        y.x = (xa.x * inv_r) * wv.x; y.y = (xa.y * inv_r) * wv.y;
        y.z = (xa.z * inv_r) * wv.z; y.w = (xa.w * inv_r) * wv.w;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          float4 o;
          o.x = hp[i] * y.x; o.y = hp[i] * y.y; o.z = hp[i] * y.z; o.w = hp[i] * y.w;
#pragma unroll
          for (int j = 0; j < N; ++j) {
            const float mij = m[i * N + j];
            o.x = fmaf(mij, xv[j].x, o.x); o.y = fmaf(mij, xv[j].y, o.y);
            o.z = fmaf(mij, xv[j].z, o.z); o.w = fmaf(mij, xv[j].w, o.w);
          }
          IO<T>::store4(ob + i * C, q, o);
        }
      }
    } else if constexpr (sizeof(T) == 4) {
      for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
        float xv[N];
#pragma unroll
        for (int j = 0; j < N; ++j) xv[j] = xb[j * C + c];
        if (GRAM) {
          int g = 0;
#pragma unroll
          for (int i = 0; i < N; ++i)
#pragma unroll
            for (int j = i; j < N; ++j) { gacc[g] = fma((double)xv[i], (double)xv[j], gacc[g]); ++g; }
        }
        float xa = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) xa = fmaf(h[j], xv[j], xa);
        const float y = (xa * inv_r) * w[c];
#pragma unroll
        for (int i = 0; i < N; ++i) {
          float o = hp[i] * y;
#pragma unroll
          for (int j = 0; j < N; ++j) o = fmaf(m[i * N + j], xv[j], o);
          ob[i * C + c] = o;
        }
      }
    }
    if (GRAM) {
      // block sum of the fp64 Gram entries, in a fixed order
      const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const double v = warp_sum_d(gacc[g]);
        if (lane == 0) s_g[warp * NG + g] = v;
      }
      __syncthreads();
      if (threadIdx.x < NG) {
        double t = 0.0;
        for (int wi = 0; wi < (int)(blockDim.x >> 5); ++wi) t += s_g[wi * NG + threadIdx.x];
        reinterpret_cast<double*>(rec_w + b * Lc::REC + Lc::OFF_G64)[threadIdx.x] = t;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Forward 3 for the tensor-core projection (which supplies only sum(x^2)):
// one CTA per token computes r = sqrt(mean_c x_agg^2 + eps) itself, then
// out[i,c] = sum_j M_ij x[j,c] + hp_i * (w_c / r) * x_agg[c].
//   QPT > 0: the token stays in registers (QPT channel quads per thread and
//            stream, loaded up front), so x is read from HBM once;
//   QPT = 0: any C -- the second loop reads x again (from L2: the CTA read it
//            microseconds earlier).
// Also the token's Gram matrix in fp64 (exact products) for the backward when
// the record is kept.  Writes r into the record.
// ---------------------------------------------------------------------------
template <int N, int QPT, bool GRAM, typename T = float, int THREADS = 256>
__global__ void __launch_bounds__(THREADS, THREADS <= 256 ? (sizeof(T) == 2 ? 3 : 2) : 1)
    stream_fwd_r_kernel(const T* __restrict__ x, const float* __restrict__ w,
                        float* __restrict__ rec, T* __restrict__ out, int64_t B, int64_t C,
                        float r_eps) {
  using Lc = L<N>;
  constexpr int NG = Lc::NG;
  __shared__ float s_rec[Lc::REC];
  __shared__ float red[32];
  __shared__ double s_g[GRAM ? 32 * NG : 1];
  const int64_t C4 = C / 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const T* xb = x + b * N * C;
    T* ob = out + b * N * C;
    // issue this token's loads before anything waits
    typename IO<T>::raw4 xv[QPT > 0 ? QPT : 1][N];
#pragma unroll
    for (int u = 0; u < QPT; ++u) {
      const int64_t q = threadIdx.x + (int64_t)u * blockDim.x;
      if (q < C4) {
#pragma unroll
        for (int j = 0; j < N; ++j) xv[u][j] = IO<T>::load_raw4(xb + j * C, q);
      }
    }
    __syncthreads();  // s_rec / red of the previous token are no longer read
    for (int e = threadIdx.x; e < Lc::REC; e += blockDim.x) s_rec[e] = rec[b * Lc::REC + e];
    __syncthreads();
    const float* h = s_rec + Lc::OFF_H;
    const float* hp = s_rec + Lc::OFF_HP;
    const float* m = s_rec + Lc::OFF_M;
    double gacc[GRAM ? NG : 1];
#pragma unroll
    for (int g = 0; g < (GRAM ? NG : 1); ++g) gacc[g] = 0.0;
    float sq = 0.f;
    auto moments = [&](const float4 (&xf)[N]) {
      if constexpr (GRAM) {
        int g = 0;
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int j = i; j < N; ++j) {
            gacc[g] = fma((double)xf[i].x, (double)xf[j].x, gacc[g]);
            gacc[g] = fma((double)xf[i].y, (double)xf[j].y, gacc[g]);
            gacc[g] = fma((double)xf[i].z, (double)xf[j].z, gacc[g]);
            gacc[g] = fma((double)xf[i].w, (double)xf[j].w, gacc[g]);
            ++g;
          }
      }
      float4 xa = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < N; ++j) {
        xa.x = fmaf(h[j], xf[j].x, xa.x); xa.y = fmaf(h[j], xf[j].y, xa.y);
        xa.z = fmaf(h[j], xf[j].z, xa.z); xa.w = fmaf(h[j], xf[j].w, xa.w);
      }
      sq += xa.x * xa.x + xa.y * xa.y + xa.z * xa.z + xa.w * xa.w;
      return xa;
    };
    float4 xa_keep[QPT > 0 ? QPT : 1];
    if constexpr (QPT > 0) {
#pragma unroll
      for (int u = 0; u < QPT; ++u) {
        const int64_t q = threadIdx.x + (int64_t)u * blockDim.x;
        xa_keep[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q < C4) {
          float4 xf[N];
#pragma unroll
          for (int j = 0; j < N; ++j) xf[j] = IO<T>::to_f4(xv[u][j]);
          xa_keep[u] = moments(xf);
        }
      }
    } else {
      for (int64_t q = threadIdx.x; q < C4; q += blockDim.x) {
        float4 xf[N];
#pragma unroll
        for (int j = 0; j < N; ++j) xf[j] = IO<T>::to_f4(IO<T>::load_raw4(xb + j * C, q));
        moments(xf);
      }
    }
    // block sums: x_agg^2 (fp32) and the fp64 Gram, fixed order
    sq = warp_sum(sq);
    if (lane == 0) red[warp] = sq;
    if constexpr (GRAM) {
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const double v = warp_sum_d(gacc[g]);
        if (lane == 0) s_g[warp * NG + g] = v;
      }
    }
    __syncthreads();
    float tot = 0.f;
    for (int k = 0; k < nw; ++k) tot += red[k];
    const float r = sqrtf(tot / (float)C + r_eps);
    const float inv_r = 1.f / r;
    if (threadIdx.x == 0) rec[b * Lc::REC + 1] = r;
    if constexpr (GRAM) {
      if (threadIdx.x < NG) {
        double t = 0.0;
        for (int k = 0; k < nw; ++k) t += s_g[k * NG + threadIdx.x];
        reinterpret_cast<double*>(rec + b * Lc::REC + Lc::OFF_G64)[threadIdx.x] = t;
      }
    }
    auto emit = [&](int64_t q, const float4 (&xf)[N], float4 xa) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + q);
      float4 y;
      y.x = (xa.x * inv_r) * wv.x; y.y = (xa.y * inv_r) * wv.y;
      y.z = (xa.z * inv_r) * wv.z; y.w = (xa.w * inv_r) * wv.w;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float4 o;
        o.x = hp[i] * y.x; o.y = hp[i] * y.y; o.z = hp[i] * y.z; o.w = hp[i] * y.w;
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const float mij = m[i * N + j];
          o.x = fmaf(mij, xf[j].x, o.x); o.y = fmaf(mij, xf[j].y, o.y);
          o.z = fmaf(mij, xf[j].z, o.z); o.w = fmaf(mij, xf[j].w, o.w);
        }
        IO<T>::store4(ob + i * C, q, o);
      }
    };
    if constexpr (QPT > 0) {
#pragma unroll
      for (int u = 0; u < QPT; ++u) {
        const int64_t q = threadIdx.x + (int64_t)u * blockDim.x;
        if (q < C4) {
          float4 xf[N];
#pragma unroll
          for (int j = 0; j < N; ++j) xf[j] = IO<T>::to_f4(xv[u][j]);
          emit(q, xf, xa_keep[u]);
        }
      }
    } else {
      for (int64_t q = threadIdx.x; q < C4; q += blockDim.x) {
        float4 xf[N];
        float4 xa = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < N; ++j) {
          xf[j] = IO<T>::to_f4(IO<T>::load_raw4(xb + j * C, q));
          xa.x = fmaf(h[j], xf[j].x, xa.x); xa.y = fmaf(h[j], xf[j].y, xa.y);
          xa.z = fmaf(h[j], xf[j].z, xa.z); xa.w = fmaf(h[j], xf[j].w, xa.w);
        }
        emit(q, xf, xa);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Forward 3 of MHCResidualWrapper (fp32): the layer's streams are never in
// memory -- stream j is sc.s[j] * residual, stream 1 the branch output, built
// in registers exactly as the reference's packing rounds them -- and the
// output is the wrapper's stream mean, (sum_i out[i, c]) / n, not the
// [T, n, C] layer output.  Otherwise as stream_fwd_r_kernel (r, fp64 Gram).
// PRE: the next branch's input RMSNorm is written by the same pass (a
// pre-norm block normalises this hidden state before its attention / MLP):
// normed[c] = mean[c] / rms2 * w2[c], rms2 = sqrt(mean_c mean^2 + eps2) over
// the mean exactly as stored, rms2 kept per token for the backward; the mean
// is recomputed from the token's registers rather than read back from HBM.
// ---------------------------------------------------------------------------
struct PreNorm {
  const float* w2 = nullptr;  // [C] weight of the next branch's RMSNorm
  float eps2 = 0.f;
  float* normed = nullptr;    // [B, C]
  float* rms2 = nullptr;      // [B]
};

template <int N, int QPT, bool GRAM, int THREADS = 256, bool PRE = false>
__global__ void __launch_bounds__(THREADS, THREADS <= 256 ? 2 : 1)
    wrap_fwd_r_kernel(const float* __restrict__ res, const float* __restrict__ br, WrapScales sc,
                      const float* __restrict__ w, float* __restrict__ rec,
                      float* __restrict__ mean, int64_t B, int64_t C, float r_eps,
                      PreNorm pn = PreNorm{}) {
  using Lc = L<N>;
  constexpr int NG = Lc::NG;
  __shared__ float s_rec[Lc::REC];
  __shared__ float red[32];
  __shared__ double s_g[GRAM ? 32 * NG : 1];
  const int64_t C4 = C / 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  auto streams = [&](float4 rv, float4 bv, float4 (&xf)[N]) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      if (j == 1) { xf[j] = bv; continue; }
      const float sj = sc.s[j];
      xf[j] = make_float4(sj * rv.x, sj * rv.y, sj * rv.z, sj * rv.w);
    }
  };
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const float4* rb = reinterpret_cast<const float4*>(res + b * C);
    const float4* bb = reinterpret_cast<const float4*>(br + b * C);
    float4 rv[QPT > 0 ? QPT : 1], bv[QPT > 0 ? QPT : 1];
#pragma unroll
    for (int u = 0; u < QPT; ++u) {
      const int64_t q = threadIdx.x + (int64_t)u * blockDim.x;
      if (q < C4) { rv[u] = __ldcs(rb + q); bv[u] = __ldcs(bb + q); }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < Lc::REC; e += blockDim.x) s_rec[e] = rec[b * Lc::REC + e];
    __syncthreads();
    const float* h = s_rec + Lc::OFF_H;
    const float* hp = s_rec + Lc::OFF_HP;
    const float* m = s_rec + Lc::OFF_M;
    double gacc[GRAM ? NG : 1];
#pragma unroll
    for (int g = 0; g < (GRAM ? NG : 1); ++g) gacc[g] = 0.0;
    float sq = 0.f;
    auto moments = [&](const float4 (&xf)[N]) {
      if constexpr (GRAM) {
        int g = 0;
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int j = i; j < N; ++j) {
            gacc[g] = fma((double)xf[i].x, (double)xf[j].x, gacc[g]);
            gacc[g] = fma((double)xf[i].y, (double)xf[j].y, gacc[g]);
            gacc[g] = fma((double)xf[i].z, (double)xf[j].z, gacc[g]);
            gacc[g] = fma((double)xf[i].w, (double)xf[j].w, gacc[g]);
            ++g;
          }
      }
      float4 xa = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < N; ++j) {
        xa.x = fmaf(h[j], xf[j].x, xa.x); xa.y = fmaf(h[j], xf[j].y, xa.y);
        xa.z = fmaf(h[j], xf[j].z, xa.z); xa.w = fmaf(h[j], xf[j].w, xa.w);
      }
      sq += xa.x * xa.x + xa.y * xa.y + xa.z * xa.z + xa.w * xa.w;
      return xa;
    };
    if constexpr (QPT > 0) {
#pragma unroll
      for (int u = 0; u < QPT; ++u) {
        const int64_t q = threadIdx.x + (int64_t)u * blockDim.x;
        if (q < C4) { float4 xf[N]; streams(rv[u], bv[u], xf); moments(xf); }
      }
    } else {
      for (int64_t q = threadIdx.x; q < C4; q += blockDim.x) {
        float4 xf[N];
        streams(__ldg(rb + q), __ldg(bb + q), xf);
        moments(xf);
      }
    }
    sq = warp_sum(sq);
    if (lane == 0) red[warp] = sq;
    if constexpr (GRAM) {
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const double v = warp_sum_d(gacc[g]);
        if (lane == 0) s_g[warp * NG + g] = v;
      }
    }
    __syncthreads();
    float tot = 0.f;
    for (int k = 0; k < nw; ++k) tot += red[k];
    const float r = sqrtf(tot / (float)C + r_eps);
    const float inv_r = 1.f / r;
    if (threadIdx.x == 0) rec[b * Lc::REC + 1] = r;
    if constexpr (GRAM) {
      if (threadIdx.x < NG) {
        double t = 0.0;
        for (int k = 0; k < nw; ++k) t += s_g[k * NG + threadIdx.x];
        reinterpret_cast<double*>(rec + b * Lc::REC + Lc::OFF_G64)[threadIdx.x] = t;
      }
    }
    float4* mb = reinterpret_cast<float4*>(mean + b * C);
    const float nf = (float)N;
    float sq2 = 0.f;                         // PRE: sum of the mean's squares
    auto mean_of = [&](int64_t q, float4 rq, float4 bq) {
      float4 xf[N];
      streams(rq, bq, xf);
      float4 xa = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < N; ++j) {
        xa.x = fmaf(h[j], xf[j].x, xa.x); xa.y = fmaf(h[j], xf[j].y, xa.y);
        xa.z = fmaf(h[j], xf[j].z, xa.z); xa.w = fmaf(h[j], xf[j].w, xa.w);
      }
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + q);
      float4 y;
      y.x = (xa.x * inv_r) * wv.x; y.y = (xa.y * inv_r) * wv.y;
      y.z = (xa.z * inv_r) * wv.z; y.w = (xa.w * inv_r) * wv.w;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float4 o;
        o.x = hp[i] * y.x; o.y = hp[i] * y.y; o.z = hp[i] * y.z; o.w = hp[i] * y.w;
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const float mij = m[i * N + j];
          o.x = fmaf(mij, xf[j].x, o.x); o.y = fmaf(mij, xf[j].y, o.y);
          o.z = fmaf(mij, xf[j].z, o.z); o.w = fmaf(mij, xf[j].w, o.w);
        }
        if (i == 0) acc = o;
        else { acc.x += o.x; acc.y += o.y; acc.z += o.z; acc.w += o.w; }
      }
      return make_float4(acc.x / nf, acc.y / nf, acc.z / nf, acc.w / nf);
    };
    auto emit = [&](int64_t q, float4 rq, float4 bq) {
      const float4 mv = mean_of(q, rq, bq);
      __stcs(mb + q, mv);
      if constexpr (PRE) sq2 += mv.x * mv.x + mv.y * mv.y + mv.z * mv.z + mv.w * mv.w;
    };
    if constexpr (QPT > 0) {
#pragma unroll
      for (int u = 0; u < QPT; ++u) {
        const int64_t q = threadIdx.x + (int64_t)u * blockDim.x;
        if (q < C4) emit(q, rv[u], bv[u]);
      }
    } else {
      for (int64_t q = threadIdx.x; q < C4; q += blockDim.x) emit(q, __ldg(rb + q), __ldg(bb + q));
    }
    if constexpr (PRE) {
      // second block sum (red is free: every thread has read it for r)
      __syncthreads();
      sq2 = warp_sum(sq2);
      if (lane == 0) red[warp] = sq2;
      __syncthreads();
      float tot2 = 0.f;
      for (int k = 0; k < nw; ++k) tot2 += red[k];
      const float r2 = sqrtf(tot2 / (float)C + pn.eps2);
      const float inv2 = 1.f / r2;
      if (threadIdx.x == 0) pn.rms2[b] = r2;
      float4* nb = reinterpret_cast<float4*>(pn.normed + b * C);
      auto emit2 = [&](int64_t q, float4 rq, float4 bq) {
        const float4 mv = mean_of(q, rq, bq);
        const float4 wv = __ldg(reinterpret_cast<const float4*>(pn.w2) + q);
        __stcs(nb + q, make_float4((mv.x * inv2) * wv.x, (mv.y * inv2) * wv.y,
                                   (mv.z * inv2) * wv.z, (mv.w * inv2) * wv.w));
      };
      if constexpr (QPT > 0) {
#pragma unroll
        for (int u = 0; u < QPT; ++u) {
          const int64_t q = threadIdx.x + (int64_t)u * blockDim.x;
          if (q < C4) emit2(q, rv[u], bv[u]);
        }
      } else {
        for (int64_t q = threadIdx.x; q < C4; q += blockDim.x) emit2(q, __ldg(rb + q), __ldg(bb + q));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Forward 3, shared-memory staged (n <= 4 dynamic H after the tensor-core
// projection, and static H): a persistent CTA per SM walks tokens b =
// blockIdx.x + k gridDim.x.  One thread keeps NBUF-1 tokens in flight with
// bulk copies (one per stream row) into a ring of token buffers, so HBM is
// busy while the CTA reduces and writes the current token; per token
//   r = sqrt(mean_c x_agg^2 + eps), x_agg = sum_j h_j x[j,c]
//   out[i,c] = sum_j M_ij x[j,c] + hp_i (w_c / r) x_agg[c]
// DYN: h, hp, M from the token's record, r and (GRAM) the fp64 Gram matrix
// written back into it; static: one shared record, r into rms[] (optional).
// Needs C * sizeof(T) % 16 == 0 and 16-byte aligned x / out / w.
// ---------------------------------------------------------------------------
constexpr int kTsThreads = 512;

template <int N, typename T, bool DYN, bool GRAM>
__global__ void __launch_bounds__(kTsThreads, 1)
    token_stream_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w,
                            float* __restrict__ rec, float* __restrict__ rms,
                            T* __restrict__ out, int64_t B, int64_t C, float r_eps, int nbuf) {
  using Lc = L<N>;
  constexpr int NG = Lc::NG;
  extern __shared__ __align__(16) unsigned char ts_smem[];
  // a token buffer: the n stream rows, then (DYN) the token's record
  const uint32_t tok_bytes = (uint32_t)(N * C * sizeof(T));
  constexpr uint32_t REC_BYTES = DYN ? Lc::REC * 4 : 0;
  const uint32_t tok_stride = (tok_bytes + REC_BYTES + 127) & ~127u;
  uint64_t* full = reinterpret_cast<uint64_t*>(ts_smem + (size_t)nbuf * tok_stride);
  __shared__ float s_rec0[DYN ? 1 : Lc::REC];
  __shared__ float red[32];
  __shared__ double s_g[GRAM ? 16 * NG : 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t C4 = C / 4;
  const int64_t first = blockIdx.x, step = gridDim.x;
  auto fetch = [&](int64_t b, int slot) {
    mbar_expect_tx(&full[slot], tok_bytes + REC_BYTES);
#pragma unroll
    for (int i = 0; i < N; ++i)
      bulk_load(ts_smem + (size_t)slot * tok_stride + (size_t)i * C * sizeof(T),
                x + (b * N + i) * C, (uint32_t)(C * sizeof(T)), &full[slot]);
    if (DYN)  // the record travels with its token
      bulk_load(ts_smem + (size_t)slot * tok_stride + tok_bytes, rec + b * Lc::REC, REC_BYTES,
                &full[slot]);
  };
  if (tid == 0) {
    for (int q = 0; q < nbuf; ++q) mbar_init(&full[q], 1);
    fence_mbar_init();
    for (int q = 0; q < nbuf; ++q)
      if (first + q * step < B) fetch(first + q * step, q);
  }
  if (!DYN) {
    for (int e = tid; e < Lc::REC; e += blockDim.x) s_rec0[e] = rec[e];
  }
  __syncthreads();
  int k = 0;
  for (int64_t b = first; b < B; b += step, ++k) {
    const int slot = k % nbuf;
    const T* xs = reinterpret_cast<const T*>(ts_smem + (size_t)slot * tok_stride);
    const float* s_rec = DYN ? reinterpret_cast<const float*>(ts_smem + (size_t)slot * tok_stride + tok_bytes) : s_rec0;
    const float* h = s_rec + Lc::OFF_H;
    const float* hp = s_rec + Lc::OFF_HP;
    const float* m = s_rec + Lc::OFF_M;
    if (!mbar_wait(&full[slot], (uint32_t)((k / nbuf) & 1))) break;  // bounded; error word set
    double gacc[GRAM ? NG : 1];
#pragma unroll
    for (int g = 0; g < (GRAM ? NG : 1); ++g) gacc[g] = 0.0;
    float sq = 0.f;
    for (int64_t q = tid; q < C4; q += blockDim.x) {
      float4 xf[N];
#pragma unroll
      for (int j = 0; j < N; ++j) xf[j] = IO<T>::to_f4(*reinterpret_cast<const typename IO<T>::raw4*>(xs + j * C + 4 * q));
      if constexpr (GRAM) {
        int g = 0;
#pragma unroll
        for (int i = 0; i < N; ++i)
#pragma unroll
          for (int j = i; j < N; ++j) {
            gacc[g] = fma((double)xf[i].x, (double)xf[j].x, gacc[g]);
            gacc[g] = fma((double)xf[i].y, (double)xf[j].y, gacc[g]);
            gacc[g] = fma((double)xf[i].z, (double)xf[j].z, gacc[g]);
            gacc[g] = fma((double)xf[i].w, (double)xf[j].w, gacc[g]);
            ++g;
          }
      }
      float4 xa = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < N; ++j) {
        xa.x = fmaf(h[j], xf[j].x, xa.x); xa.y = fmaf(h[j], xf[j].y, xa.y);
        xa.z = fmaf(h[j], xf[j].z, xa.z); xa.w = fmaf(h[j], xf[j].w, xa.w);
      }
      sq += xa.x * xa.x + xa.y * xa.y + xa.z * xa.z + xa.w * xa.w;
    }
    // block sums in a fixed order
    sq = warp_sum(sq);
    if (lane == 0) red[warp] = sq;
    if constexpr (GRAM) {
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const double v = warp_sum_d(gacc[g]);
        if (lane == 0) s_g[warp * NG + g] = v;
      }
    }
    __syncthreads();
    float tot = 0.f;
    for (int q = 0; q < (int)(blockDim.x >> 5); ++q) tot += red[q];
    const float r = sqrtf(tot / (float)C + r_eps);
    const float inv_r = 1.f / r;
    if (tid == 0) {
      if (DYN) rec[b * Lc::REC + 1] = r;
      else if (rms) rms[b] = r;
    }
    if constexpr (GRAM) {
      if (tid < NG) {
        double t = 0.0;
        for (int q = 0; q < (int)(blockDim.x >> 5); ++q) t += s_g[q * NG + tid];
        reinterpret_cast<double*>(rec + b * Lc::REC + Lc::OFF_G64)[tid] = t;
      }
    }
    T* ob = out + b * N * C;
    for (int64_t q = tid; q < C4; q += blockDim.x) {
      float4 xf[N];
#pragma unroll
      for (int j = 0; j < N; ++j) xf[j] = IO<T>::to_f4(*reinterpret_cast<const typename IO<T>::raw4*>(xs + j * C + 4 * q));
      float4 xa = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < N; ++j) {
        xa.x = fmaf(h[j], xf[j].x, xa.x); xa.y = fmaf(h[j], xf[j].y, xa.y);
        xa.z = fmaf(h[j], xf[j].z, xa.z); xa.w = fmaf(h[j], xf[j].w, xa.w);
      }
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + q);
      float4 y;
      y.x = (xa.x * inv_r) * wv.x; y.y = (xa.y * inv_r) * wv.y;
      y.z = (xa.z * inv_r) * wv.z; y.w = (xa.w * inv_r) * wv.w;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float4 o;
        o.x = hp[i] * y.x; o.y = hp[i] * y.y; o.z = hp[i] * y.z; o.w = hp[i] * y.w;
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const float mij = m[i * N + j];
          o.x = fmaf(mij, xf[j].x, o.x); o.y = fmaf(mij, xf[j].y, o.y);
          o.z = fmaf(mij, xf[j].z, o.z); o.w = fmaf(mij, xf[j].w, o.w);
        }
        IO<T>::store4(ob + i * C, q, o);
      }
    }
    __syncthreads();  // the buffer and red are free again
    if (tid == 0 && b + (int64_t)nbuf * step < B) fetch(b + (int64_t)nbuf * step, slot);
  }
}

// ---------------------------------------------------------------------------
// Static-H forward, single pass: one CTA per token holds the token in
// registers (QPT float4 channel quads per thread), block-reduces sum(x_agg^2)
// and writes out.  T = float or __nv_bfloat16 (fp32 arithmetic either way).
// ---------------------------------------------------------------------------
struct bf16x4 { __nv_bfloat162 a, b; };

template <int N, int QPT, typename T>
__global__ void __launch_bounds__(256, sizeof(T) == 2 ? 3 : 2)
    static_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w,
                      const float* __restrict__ rec, float* __restrict__ rms,
                      T* __restrict__ out, int64_t B, int64_t C, float r_eps) {
  using Lc = L<N>;
  __shared__ float s_rec[Lc::REC];
  __shared__ float red[8];
  for (int e = threadIdx.x; e < Lc::REC; e += blockDim.x) s_rec[e] = rec[e];
  __syncthreads();
  const float* h = s_rec + Lc::OFF_H;
  const float* hp = s_rec + Lc::OFF_HP;
  const float* m = s_rec + Lc::OFF_M;
  const int64_t C4 = C / 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const T* xb = x + b * N * C;
    T* ob = out + b * N * C;
    typename IO<T>::raw4 xv[QPT][N];   // as stored: bf16 tokens take half the registers
    float4 xa[QPT];
    float sq = 0.f;
#pragma unroll
    for (int u = 0; u < QPT; ++u) {
      const int64_t q = threadIdx.x + (int64_t)u * blockDim.x;
      xa[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (q < C4) {
#pragma unroll
        for (int j = 0; j < N; ++j) xv[u][j] = IO<T>::load_raw4(xb + j * C, q);
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const float4 xf = IO<T>::to_f4(xv[u][j]);
          xa[u].x = fmaf(h[j], xf.x, xa[u].x); xa[u].y = fmaf(h[j], xf.y, xa[u].y);
          xa[u].z = fmaf(h[j], xf.z, xa[u].z); xa[u].w = fmaf(h[j], xf.w, xa[u].w);
        }
        sq += xa[u].x * xa[u].x + xa[u].y * xa[u].y + xa[u].z * xa[u].z + xa[u].w * xa[u].w;
      }
    }
    sq = warp_sum(sq);
    if (lane == 0) red[warp] = sq;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    __syncthreads();
    const float r = sqrtf(tot / (float)C + r_eps);
    const float inv_r = 1.f / r;
    if (threadIdx.x == 0 && rms) rms[b] = r;
#pragma unroll
    for (int u = 0; u < QPT; ++u) {
      const int64_t q = threadIdx.x + (int64_t)u * blockDim.x;
      if (q < C4) {
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + q);
        float4 y;
        y.x = (xa[u].x * inv_r) * wv.x; y.y = (xa[u].y * inv_r) * wv.y;
        y.z = (xa[u].z * inv_r) * wv.z; y.w = (xa[u].w * inv_r) * wv.w;
#pragma unroll
        for (int i = 0; i < N; ++i) {
          float4 o;
          o.x = hp[i] * y.x; o.y = hp[i] * y.y; o.z = hp[i] * y.z; o.w = hp[i] * y.w;
#pragma unroll
          for (int j = 0; j < N; ++j) {
            const float mij = m[i * N + j];
            const float4 xf = IO<T>::to_f4(xv[u][j]);
            o.x = fmaf(mij, xf.x, o.x); o.y = fmaf(mij, xf.y, o.y);
            o.z = fmaf(mij, xf.z, o.z); o.w = fmaf(mij, xf.w, o.w);
          }
          IO<T>::store4(ob + i * C, q, o);
        }
      }
    }
  }
}

// Scalar fallback for the static forward (C not a multiple of 4 or too large
// for the register-resident kernel): two passes over the token, the second
// one served by L1/L2.
template <int N, typename T>
__global__ void __launch_bounds__(256)
    static_fwd_generic_kernel(const T* __restrict__ x, const float* __restrict__ w,
                              const float* __restrict__ rec, float* __restrict__ rms,
                              T* __restrict__ out, int64_t B, int64_t C, float r_eps) {
  using Lc = L<N>;
  __shared__ float s_rec[Lc::REC];
  __shared__ float red[8];
  for (int e = threadIdx.x; e < Lc::REC; e += blockDim.x) s_rec[e] = rec[e];
  __syncthreads();
  const float* h = s_rec + Lc::OFF_H;
  const float* hp = s_rec + Lc::OFF_HP;
  const float* m = s_rec + Lc::OFF_M;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t b = blockIdx.x; b < B; b += gridDim.x) {
    const T* xb = x + b * N * C;
    T* ob = out + b * N * C;
    float sq = 0.f;
    for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
      float xa = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) xa = fmaf(h[j], (float)xb[j * C + c], xa);
      sq += xa * xa;
    }
    sq = warp_sum(sq);
    if (lane == 0) red[warp] = sq;
    __syncthreads();
    float tot = 0.f;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) tot += red[k];
    __syncthreads();
    const float r = sqrtf(tot / (float)C + r_eps);
    const float inv_r = 1.f / r;
    if (threadIdx.x == 0 && rms) rms[b] = r;
    for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
      float xv[N];
      float xa = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        xv[j] = (float)xb[j * C + c];
        xa = fmaf(h[j], xv[j], xa);
      }
      const float y = (xa * inv_r) * w[c];
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float o = hp[i] * y;
#pragma unroll
        for (int j = 0; j < N; ++j) o = fmaf(m[i * N + j], xv[j], o);
        ob[i * C + c] = (T)o;
      }
    }
  }
}

// Shared record for static H: h = sigmoid(H_pre), hp = 2 sigmoid(H_post),
// M = Sinkhorn(exp(H_res)).  Written into rec (REC floats).
template <int N>
__global__ void static_prep_kernel(const float* __restrict__ H_pre,
                                   const float* __restrict__ H_post,
                                   const float* __restrict__ H_res, float* __restrict__ rec,
                                   int iters, float s_eps) {
  using Lc = L<N>;
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float m[N * N];
#pragma unroll
  for (int e = 0; e < N * N; ++e) m[e] = expf(H_res[e]);
  sk_forward<N, float>(m, iters, s_eps);
  for (int e = 0; e < Lc::REC; ++e) rec[e] = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    rec[Lc::OFF_H + i] = sigmoidf_(H_pre[i]);
    rec[Lc::OFF_HP + i] = 2.f * sigmoidf_(H_post[i]);
  }
#pragma unroll
  for (int e = 0; e < N * N; ++e) rec[Lc::OFF_M + e] = m[e];
}

}  // namespace
}  // namespace mhc
