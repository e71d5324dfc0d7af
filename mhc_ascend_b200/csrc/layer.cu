// Fused mHC layer: dynamic-H and static-H forward and backward for sm_100a.
//
// Replaces the reference's host orchestration mhc_layer_fwd_dynamic
// (bindings.cpp:880-952) and mhc_layer_bwd_dynamic (bindings.cpp:600-874),
// which run ~10 kernels + ~35 ATen ops with a host sync before every launch,
// and the static-H composition of layer.py:142-170.
//
// Math (per token, x[i,c] for n streams i and C channels; xf = flattened x):
//   rms_h = sqrt(mean(xf^2) + eps_r)          p = xf @ phi^T  (phi: [n^2+2n, nC])
//   t = alpha * p / rms_h + b ;  h = sigmoid(t_pre), hp = 2 sigmoid(t_post),
//   M = Sinkhorn(exp(t_res)) ;  x_agg[c] = sum_i h_i x[i,c]
//   r = sqrt(mean_c(x_agg^2) + eps_r) ;  y[c] = x_agg[c] / r * w[c]
//   out[i,c] = hp_i y[c] + sum_j M[i,j] x[j,c]
//
// Every token-wide reduction is expressed through per-token "moments" that a
// single pass over the token's data produces:
//   forward : p (n^2+2n dots with phi) and the n x n Gram matrix G = x x^T
//             (sum(xf^2) = trace G, sum_c x_agg^2 = h^T G h);
//   backward: gM = g x^T, W = g diag(w) x^T and G again; from these every
//             per-token scalar of the backward follows in closed form (see
//             token_bwd_lanes_kernel).
// So the forward reads x twice and writes out once; the backward reads g and
// x twice and writes grad_x once; parameter gradients are fixed-order
// reductions (no atomics: bitwise reproducible).
//
// Kernels (launch order):
//   fwd : proj_stats   -> token_fwd (gates, Sinkhorn, r) -> stream_fwd
//   bwd : bwd_stats    -> token_bwd (Sinkhorn reverse, d_p) -> grad_x (gx, dphi/gw
//         partials) -> reduce_* (fixed-order sums over splits / tokens)
#include "common.cuh"
#include "sinkhorn.cuh"
#include "sinkhorn_lanes.cuh"
#include "tma.cuh"
#include <cuda_bf16.h>

namespace mhc {
namespace {

// ---------------------------------------------------------------------------
// Layout constants
// ---------------------------------------------------------------------------
template <int N>
struct L {
  static constexpr int NH = N * N + 2 * N;              // projections (pre|post|res)
  static constexpr int NHP = (NH + 3) / 4 * 4;           // padded to float4
  static constexpr int NG = N * (N + 1) / 2;             // Gram upper triangle
  static constexpr int REC_RAW = 2 + 2 * N + N * N + NH;  // token_state record
  // then the Gram matrix in fp64 (exact products), written by the dynamic
  // stream_fwd for the backward, at an 8-byte offset
  static constexpr int OFF_G64 = (REC_RAW + 1) / 2 * 2;
  static constexpr int REC = (OFF_G64 + 2 * NG + 3) / 4 * 4;
  static constexpr int OFF_H = 2, OFF_HP = 2 + N, OFF_M = 2 + 2 * N, OFF_P = 2 + 2 * N + N * N;
  static constexpr int NS1 = 2 * N * N + NG;             // static bwd moments: gM, W, G
  static constexpr int NSD = 2 * N * N;                  // dynamic bwd moments: gM, W
  // bwd per-token row read by grad_x: beta, inv_r, coef, -, d_p[NHP], h[N], hp[N], M^T[N*N]
  static constexpr int OFF_TH = 4 + NHP, OFF_THP = OFF_TH + N, OFF_TM = OFF_THP + N;
  static constexpr int TB = (OFF_TM + N * N + 3) / 4 * 4;
  static constexpr int NR = NH + 3;                       // bwd per-token reduce: dt, dalpha
  static constexpr int NRS = 2 * N + N * N;               // static per-token reduce: dt_pre, dt_post, gM
};

__host__ __device__ inline int rec_stride(int n) {
  const int raw = 2 + 2 * n + n * n + (n * n + 2 * n);
  const int og = (raw + 1) / 2 * 2;
  return (og + n * (n + 1) + 3) / 4 * 4;
}

// Layout of the warp-specialised n = 4 grad_x (kernel comment at grad_x6_kernel).
struct Gx6Cfg {
  static constexpr int CW = 32, COLS = 128, TOK = 32, NH = 24, KP = 32;
  static constexpr int SG = 3, SI = 3, ND = 2, E_WARPS = 16, TPE = TOK / E_WARPS, THREADS = 32 * (2 + E_WARPS + 4 + 1 + 4);
  static constexpr int D2_WARP = 2 + E_WARPS + 4;          // issues the D2 MMAs
  static constexpr int XT_WARP0 = D2_WARP + 1;             // first of the four X^T warps
  // operand image of one token block (floats)
  static constexpr int IMG_B1H = 0, IMG_B1L = TOK * NH, IMG_B2H = 2 * TOK * NH, IMG_B2L = IMG_B2H + KP * TOK;
  static constexpr int IMG_SC = IMG_B2L + KP * TOK, IMG_FLOATS = IMG_SC + TOK * 32;
  static constexpr uint32_t IMG = IMG_FLOATS * 4;
  static constexpr uint32_t LOCB = TOK * COLS * 4;         // local terms [tokens][128 columns]
  static constexpr int NBAR = 2 * SG + 2 * SI + 6 * ND + 2;
  // tensor memory: D1[b] [TOK b, +TOK); D2 [64, 96); Phi^T hi [96, 120), lo [128, 152);
  // X^T[b] [256 + 2 TOK b, +2 TOK) hi|lo
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t D2_COL = 64, A1_COL = 96, A1L_COL = 128, XT_COL = 256;
  static_assert(ND * TOK <= 64 && XT_COL + 2 * TOK * ND <= TMEM_COLS && TOK % 16 == 0, "tensor-memory plan");
};

// Shared-memory plan of grad_x6 for stream element type T (fp32 or bf16 I/O).
template <typename T>
struct Gx6S {
  using F = Gx6Cfg;
  static constexpr bool BF16 = sizeof(T) == 2;
  static constexpr uint32_t GB = F::TOK * 4 * F::CW * sizeof(T);   // g (or x) tile bytes
  static constexpr uint32_t OFF_IMG = F::SG * 2 * GB;              // g/x ring, then the image ring
  static constexpr uint32_t OFF_LOC = OFF_IMG + F::SI * F::IMG;    // [ND buffers]
  static constexpr uint32_t STGB = BF16 ? F::TOK * F::COLS * 2 : 0; // bf16 grad_x staging tile
  static constexpr uint32_t OFF_STG = OFF_LOC + F::ND * F::LOCB;   // [ND buffers]
  static constexpr uint32_t OFF_GW = OFF_STG + F::ND * STGB;       // grad-w partials [E warps][32]
  static constexpr uint32_t OFF_BAR = OFF_GW + F::E_WARPS * F::CW * 4;
  static constexpr size_t SMEM = OFF_BAR + F::NBAR * 8 + 16 + 128;
};

__device__ __forceinline__ int gram_index(int i, int j, int N) {
  // upper triangle, row-major: (0,0),(0,1)..(0,N-1),(1,1)...
  if (i > j) { int t = i; i = j; j = t; }
  return i * N - i * (i - 1) / 2 + (j - i);
}

__device__ __forceinline__ const float* phi_row(const float* pre, const float* post,
                                                const float* res, int k, int N, int64_t nC) {
  if (k < N) return pre + (int64_t)k * nC;
  if (k < 2 * N) return post + (int64_t)(k - N) * nC;
  return res + (int64_t)(k - 2 * N) * nC;
}

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
template <int N>
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
  float p[NH], G[NG];
#pragma unroll
  for (int k = 0; k < NH; ++k) p[k] = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g) G[g] = 0.f;
  for (int s = 0; s < ks; ++s) {
    const float* pp = ppart + ((int64_t)s * B + b) * NHP;
    const float* gp = gpart + ((int64_t)s * B + b) * NG;
#pragma unroll
    for (int k = 0; k < NH; ++k) p[k] += pp[k];
#pragma unroll
    for (int g = 0; g < NG; ++g) G[g] += gp[g];
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) ss += G[gram_index(i, i, N)];
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
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) q += h[i] * h[j] * G[gram_index(i, j, N)];
  const float r = sqrtf(fmaxf(q, 0.f) / (float)C + r_eps);
  o[0] = rms_h;
  o[1] = r;
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

// ---------------------------------------------------------------------------
// Backward 1: per-token moments gM = g x^T, W = g diag(w) x^T, G = x x^T.
//   One CTA (128 threads) per token, float4 over channel quads when VEC.
// ---------------------------------------------------------------------------
template <int V>
__device__ __forceinline__ void block_reduce_to_global(double (&acc)[V], double* smem,
                                                       double* __restrict__ dst) {
  // smem: [nwarps][V]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
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

// ---------------------------------------------------------------------------
// tcgen05 (UMMA) helpers: kind::tf32, operands in shared memory in the
// K-major "interleaved" (no swizzle) layout -- 8 rows x 16 bytes core
// matrices -- accumulators in tensor memory.
// ---------------------------------------------------------------------------
// byte offset of element (row r, k) in an R-row K-major operand
__host__ __device__ __forceinline__ uint32_t umma_kmaj_off(int r, int k, int R) {
  return (uint32_t)((k >> 2) * (R >> 3) * 128 + (r >> 3) * 128 + (r & 7) * 16 + (k & 3) * 4);
}
// smem matrix descriptor: start address, leading (K-chunk) and stride (8-row
// group) byte offsets, sm100 descriptor version, no swizzle
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}
// descriptor of K-step s (k in [8s, 8s+8)) of an R-row operand, rows from rb
__device__ __forceinline__ uint64_t umma_desc_k(uint32_t base, int R, int s, int rb) {
  return umma_desc(base + (uint32_t)(2 * s * (R >> 3) * 128 + (rb >> 3) * 128), (uint32_t)((R >> 3) * 128), 128);
}
// instruction descriptor: D f32, A/B tf32, both K-major, M x N
__host__ __device__ constexpr uint32_t umma_idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 32 lanes x 16 columns of fp32 from tensor memory (this warp's lane quadrant)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

// 32 lanes x 16 columns of 32-bit values into tensor memory (this warp's lane quadrant)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// D (tmem) (+)= A (tmem, M lanes x 8 columns) . B (smem descriptor)^T, kind::tf32
__device__ __forceinline__ void umma_tf32_at(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ---------------------------------------------------------------------------
// Forward 1 on tcgen05: projection p = x_flat . phi^T and the per-token Gram
// matrix of the n streams, for n <= 4 (C % 4 == 0, x 16-byte aligned).
//   CTA = 128 tokens (one M=128 MMA tile) x one split of the channels, two
//   CTAs per SM, warp-specialised: warp 0 issues TMA, warp 1 issues MMAs,
//   warps 2..9 (two threads per token, one per half of a 128-byte row)
//   prepare the A operand.  A stage is one stream x 32 channels: x[128 tokens
//   x 32] and phi_hi / phi_lo[NB rows x 32] (phi split once per call), both
//   128-byte-swizzled as TMA writes them.  The operand threads read their
//   token's row, keep the values of the n streams of a channel block in
//   registers for the Gram entries, and store the row split into tf32 hi/lo
//   into tensor memory with tcgen05.st (lane = token, column = channel: the
//   A operand, no proxy fence); the MMA warp adds x_lo.phi_hi + x_hi.phi_lo +
//   x_hi.phi_hi (3xTF32) into the accumulator in tensor memory.  Barriers:
//   full (TMA bytes), empty (operand warps done with x + MMA done with phi),
//   aready / afree per tensor-memory A buffer.
// ---------------------------------------------------------------------------
template <int N, typename T = float>
struct PumCfg {
  static constexpr int NH = L<N>::NH, NHP = L<N>::NHP, NG = L<N>::NG;
  static constexpr int NB = (NH + 15) / 16 * 16;           // MMA N (padded phi rows)
  // a stage is one 128-byte row of x per token: 32 fp32 or 64 bf16 channels
  static constexpr int TOK = 128, CH = 128 / (int)sizeof(T), THREADS = 320;
  static constexpr int PSUB = CH / 32;                     // 32-channel phi sub-tiles per stage
  static constexpr bool BF16 = sizeof(T) == 2;             // bf16 x is exact in tf32: no lo part
  static constexpr uint32_t XB = TOK * 128;                // x tile of one stage
  static constexpr uint32_t PB = NB * CH * 4;              // phi tile (fp32) of one stage
  static constexpr uint32_t SLOT = XB + 2 * PB;            // x, phi_hi, phi_lo
  static constexpr uint32_t OFF_PH = XB, OFF_PL = XB + PB;
  static constexpr uint32_t TX = SLOT;                     // bytes TMA brings per stage
  static constexpr int STAGES = BF16 ? 3 : 4, NA = 2;      // smem stages, tensor-memory A buffers
  static constexpr uint32_t TCOLS = 256;                   // D [0, 32); A[a] = [64 + 64 a, +64): fp32 hi|lo, bf16 hi
  static constexpr uint32_t ACOL = 64;
  static constexpr uint32_t OFF_GX = STAGES * SLOT;        // Gram exchange [128][NG]
  static constexpr uint32_t OFF_BAR = OFF_GX + TOK * NG * 4;
  static constexpr size_t SMEM = OFF_BAR + (2 * STAGES + 2 * NA + 1) * 8 + 16 + 1024;
  static_assert(NB <= 32, "one 32-column accumulator");
  static_assert(XB % 1024 == 0 && PB % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
};

// phi_hi / phi_lo [NB rows x nC]: rows k < NH hold phi_k split into tf32 hi +
// tf32 lo, the padding rows are zero.
template <int N>
__global__ void __launch_bounds__(256)
    phi_split_kernel(const float* __restrict__ pp, const float* __restrict__ pq,
                     const float* __restrict__ pr, float* __restrict__ ph,
                     float* __restrict__ pl, int64_t C, bool vec) {
  // blockIdx.y = row k; float4 columns when every row start is 16-byte aligned
  using P = PumCfg<N>;
  const int64_t nC = (int64_t)N * C;
  const int k = blockIdx.y;
  const float* src = k < P::NH ? phi_row(pp, pq, pr, k, N, nC) : nullptr;
  float* dh = ph + (int64_t)k * nC;
  float* dl = pl + (int64_t)k * nC;
  if (vec) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nC / 4;
         q += (int64_t)gridDim.x * blockDim.x) {
      const float4 v = src ? __ldg(reinterpret_cast<const float4*>(src) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      uint4 hi, lo;
      split_tf32(v.x, hi.x, lo.x); split_tf32(v.y, hi.y, lo.y);
      split_tf32(v.z, hi.z, lo.z); split_tf32(v.w, hi.w, lo.w);
      reinterpret_cast<uint4*>(dh)[q] = hi;
      reinterpret_cast<uint4*>(dl)[q] = lo;
    }
  } else {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nC;
         e += (int64_t)gridDim.x * blockDim.x) {
      uint32_t hi, lo;
      split_tf32(src ? src[e] : 0.f, hi, lo);
      dh[e] = __uint_as_float(hi);
      dl[e] = __uint_as_float(lo);
    }
  }
}

// smem descriptor of a K-major, 128-byte-swizzled operand (8-row groups
// 1024 B apart); the start may advance by 32 B per K-step inside the atom
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Bounded mbarrier wait that also gives up once another role of the CTA has
// raised the abort word.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity,
                                                   const volatile int* abort_word) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 255) == 255 && *abort_word) return false;
  }
  atomicExch(&g_mhc_device_error, 1);
  return false;
}

template <int N, typename T = float>
__global__ void __launch_bounds__(320, 2)
    proj_umma_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap hmap,
                     const __grid_constant__ CUtensorMap lmap, float* __restrict__ ppart,
                     float* __restrict__ gpart, int64_t B, int64_t C, int cps) {
  using P = PumCfg<N, T>;
  constexpr int NG = P::NG, NHP = P::NHP, S = P::STAGES, NA = P::NA;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* gx_s = reinterpret_cast<float*>(sm + P::OFF_GX);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + P::OFF_BAR);
  uint64_t* empty = full + S;
  uint64_t* aready = empty + S;
  uint64_t* afree = aready + NA;
  uint64_t* done = afree + NA;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t sbase = smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t t0 = (int64_t)blockIdx.x * P::TOK;
  const int split = blockIdx.y;
  const int64_t c_begin = (int64_t)split * cps;
  const int64_t c_end = c_begin + cps < C ? c_begin + cps : C;
  const int nblocks = c_begin < c_end ? (int)((c_end - c_begin + P::CH - 1) / P::CH) : 0;
  const int nchunks = nblocks * N;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(P::TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 32) {
    prefetch_tmap(&xmap);
    prefetch_tmap(&hmap);
    prefetch_tmap(&lmap);
    for (int st = 0; st < S; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 1 + 8);
    }
    for (int a = 0; a < NA; ++a) {
      mbar_init(&aready[a], 8);
      mbar_init(&afree[a], 1);
    }
    mbar_init(done, 1);
    *abort_word = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int k = 0; k < nchunks; ++k) {
        const int slot = k % S;
        if (k >= S && !mbar_wait_or_abort(&empty[slot], (uint32_t)(((k / S) - 1) & 1), abort_word)) {
          *abort_word = 1;
          break;
        }
        issued = k + 1;
        unsigned char* base = sm + slot * P::SLOT;
        const int c = (int)(c_begin + (int64_t)(k / N) * P::CH);
        const int i = k % N;
        mbar_expect_tx(&full[slot], P::TX);
        tma_load_3d(base, &xmap, c, i, (int)t0, &full[slot]);
#pragma unroll
        for (int ps = 0; ps < P::PSUB; ++ps) {
          tma_load_3d(base + P::OFF_PH + ps * P::NB * 128, &hmap, c + 32 * ps, i, 0, &full[slot]);
          tma_load_3d(base + P::OFF_PL + ps * P::NB * 128, &lmap, c + 32 * ps, i, 0, &full[slot]);
        }
      }
      // no copy may still be landing when the CTA exits (bounded)
      for (int q = issued > S ? issued - S : 0; q < issued; ++q)
        mbar_wait(&full[q % S], (uint32_t)((q / S) & 1));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t ID = umma_idesc_tf32(128, P::NB);
      for (int k = 0; k < nchunks; ++k) {
        const int slot = k % S, a = k % NA;
        if (!mbar_wait_or_abort(&full[slot], (uint32_t)((k / S) & 1), abort_word) ||
            !mbar_wait_or_abort(&aready[a], (uint32_t)((k / NA) & 1), abort_word)) {
          *abort_word = 1;
          break;
        }
        tc_fence_after();
        const uint32_t sb = sbase + slot * P::SLOT;
        const uint32_t at = tmem + P::ACOL + 64 * a;
#pragma unroll
        for (int st = 0; st < P::CH / 8; ++st) {
          const uint32_t boff = (st / 4) * P::NB * 128 + 32 * (st % 4);
          const uint64_t bh = umma_desc_sw128(sb + P::OFF_PH + boff);
          const uint64_t bl = umma_desc_sw128(sb + P::OFF_PL + boff);
          if constexpr (P::BF16) {
            umma_tf32_at(tmem, at + 8 * st, bh, ID, (k > 0 || st > 0) ? 1u : 0u);
            umma_tf32_at(tmem, at + 8 * st, bl, ID, 1u);
          } else {
            umma_tf32_at(tmem, at + 32 + 8 * st, bh, ID, (k > 0 || st > 0) ? 1u : 0u);
            umma_tf32_at(tmem, at + 8 * st, bl, ID, 1u);
            umma_tf32_at(tmem, at + 8 * st, bh, ID, 1u);
          }
        }
        umma_commit(&empty[slot]);
        umma_commit(&afree[a]);
      }
      umma_commit(done);
    }
  } else {
    // ---------------- A operand (tensor memory) + Gram ----------------
    const int cw = warp - 2;               // 0..7
    const int h = cw >> 2;                 // half of the 128-byte row
    const int qd = warp & 3;               // tensor-memory lane quadrant
    const int r = 32 * qd + lane;          // token row = tensor-memory lane
    const uint32_t rowoff = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
    uint32_t choff[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) choff[j] = rowoff + (uint32_t)((((4 * h + j) ^ (r & 7))) * 16);
    float gacc[NG];
#pragma unroll
    for (int g = 0; g < NG; ++g) gacc[g] = 0.f;
    bool ok = true;
    for (int b = 0; b < nblocks && ok; ++b) {
      // this thread's 16 (fp32) or 32 (bf16) channels of each stream, as stored
      uint4 v[N][4];
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int k = b * N + i;
        const int slot = k % S, a = k % NA;
        const unsigned char* base = sm + slot * P::SLOT;
        if (!mbar_wait_or_abort(&full[slot], (uint32_t)((k / S) & 1), abort_word)) { ok = false; break; }
#pragma unroll
        for (int j = 0; j < 4; ++j) v[i][j] = *reinterpret_cast<const uint4*>(base + choff[j]);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);  // x of this stage now lives in registers
        if (k >= NA && !mbar_wait_or_abort(&afree[a], (uint32_t)(((k / NA) - 1) & 1), abort_word)) { ok = false; break; }
        tc_fence_after();
        if constexpr (P::BF16) {
          // bf16 -> fp32 is exact and already a tf32 value: hi only
          const uint32_t ta = tmem + ((uint32_t)(32 * qd) << 16) + P::ACOL + 64 * a + 32 * h;
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            uint32_t hi[16];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const uint32_t w2 = (&v[i][2 * hf].x)[e];   // channels 2e, 2e+1 of chunks 2hf, 2hf+1
              hi[2 * e] = w2 << 16;
              hi[2 * e + 1] = w2 & 0xFFFF0000u;
            }
            tmem_st16(ta + 16 * hf, hi);
          }
        } else {
          const uint32_t ta = tmem + ((uint32_t)(32 * qd) << 16) + P::ACOL + 64 * a + 16 * h;
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            uint32_t hi[8], lo[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) split_tf32(__uint_as_float((&v[i][2 * hf].x)[e]), hi[e], lo[e]);
            tmem_st8(ta + 8 * hf, hi);
            tmem_st8(ta + 32 + 8 * hf, lo);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&aready[a]);
      }
      if (!ok) break;
      // Gram of this block first, then the running sum: the rounding error
      // grows with the number of blocks, not of channels
      int g = 0;
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = i; j < N; ++j) {
          float blk = 0.f;
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const uint32_t ui = (&v[i][0].x)[q], uj = (&v[j][0].x)[q];
            if constexpr (P::BF16) {
              blk = fmaf(__uint_as_float(ui << 16), __uint_as_float(uj << 16), blk);
              blk = fmaf(__uint_as_float(ui & 0xFFFF0000u), __uint_as_float(uj & 0xFFFF0000u), blk);
            } else {
              blk = fmaf(__uint_as_float(ui), __uint_as_float(uj), blk);
            }
          }
          gacc[g] += blk;
          ++g;
        }
    }
    if (!ok) *abort_word = 1;
    // results: D columns [16h, 16h + 16) of this token, Gram halves summed
    bool have = ok && nchunks > 0 && mbar_wait_or_abort(done, 0u, abort_word);
    have = __all_sync(0xffffffffu, have);
    tc_fence_after();
    const int64_t tok = t0 + r;
    if (16 * h < NHP) {
      float d[16];
      if (have) {
        tmem_ld16(tmem + ((uint32_t)(32 * qd) << 16) + 16 * h, d);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) d[e] = 0.f;
      }
      if (tok < B && (have || nchunks == 0)) {
        float* pd = ppart + ((int64_t)split * B + tok) * NHP + 16 * h;
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (16 * h + e < NHP) pd[e] = d[e];
      }
    }
    if (h == 1) {
#pragma unroll
      for (int g = 0; g < NG; ++g) gx_s[r * NG + g] = gacc[g];
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (h == 0 && tok < B && (have || nchunks == 0)) {
#pragma unroll
      for (int g = 0; g < NG; ++g)
        gpart[((int64_t)split * B + tok) * NG + g] = gacc[g] + gx_s[r * NG + g];
    }
  }
  // the MMA issuer drains its last batch before tensor memory is released
  if (warp == 1 && lane == 0 && nchunks > 0) mbar_wait_or_abort(done, 0u, abort_word);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P::TCOLS));
}

// ---------------------------------------------------------------------------
// Backward 3 for n = 4, dynamic H, on tcgen05 with warp specialisation.
//   CTA = 32 channels x 4 streams = 128 columns (col = 32 i + c) = one M=128
//   MMA tile, a contiguous range of 32-token blocks; 27 warps: warp 0 TMA,
//   warp 1 issues D1, warps 2..17 "E" (two tokens each, lane = channel, all
//   four streams), warps 18..21 epilogue and warps 23..26 X^T (stream = the
//   tensor-memory lane quadrant of the warp, lane = channel), warp 22 issues
//   D2.  Per block j:
//     TMA:  g, x [32 tokens x 4 streams x 32 channels] and the block's
//           operand image (d_p split into tf32 hi/lo in both the B layout of
//           D1 and of D2, plus the per-token scalars), written by
//           token_bwd (gx_image_row) in the exact K-major shared-memory layout;
//     MMA:  D1[b] = Phi^T[col x 24] . D_p^T      (M=128, N=32, 3xTF32)
//           D2   += X^T[col x 32 tok] . D_p      (M=128, N=32, 3xTF32)
//           with Phi^T resident in shared memory, X^T (A of D2) and D1 in
//           tensor memory, ND-deep;
//     X^T:  x of the warp's stream split into tf32 hi/lo and stored into
//           tensor memory (tcgen05.st: lane = column, column = token), which
//           transposes for free and needs no proxy fence;
//     E:    the local terms of all four streams into a shared buffer
//           (overlapping the MMAs);
//     epilogue: grad_x = D1 + local term, added in place in the local-term
//           buffer (its [token][stream][channel] layout is the grad_x tile)
//           and written with one TMA store.
//   After the range: D2 -> this split's dphi partial, sum of gy.xa.inv_r ->
//   this split's grad-w partial.
// ---------------------------------------------------------------------------


template <typename T>
__global__ void __launch_bounds__(Gx6Cfg::THREADS, 1)
    grad_x6_kernel(const __grid_constant__ CUtensorMap gmap, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap omap, const float* __restrict__ img, const float* __restrict__ w,
                   const float* __restrict__ phi_pre, const float* __restrict__ phi_post,
                   const float* __restrict__ phi_res, T* __restrict__ gx,
                   float* __restrict__ dphi_part, float* __restrict__ gw_part, int64_t B,
                   int64_t C, int ntiles, int nsplit, int64_t nblk) {
  using F = Gx6Cfg;
  using SM = Gx6S<T>;
  constexpr int SG = F::SG, SI = F::SI, ND = F::ND, CW = F::CW, COLS = F::COLS, TOK = F::TOK;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint64_t* gfull = reinterpret_cast<uint64_t*>(sm + SM::OFF_BAR);
  uint64_t* gfree = gfull + SG;
  uint64_t* ifull = gfree + SG;
  uint64_t* ifree = ifull + SI;
  uint64_t* a2_ready = ifree + SI;
  uint64_t* a2_free = a2_ready + ND;
  uint64_t* d1_full = a2_free + ND;
  uint64_t* d1_free = d1_full + ND;
  uint64_t* loc_ready = d1_free + ND;
  uint64_t* loc_free = loc_ready + ND;
  uint64_t* d2_done = loc_free + ND;
  uint64_t* phi_ready = d2_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(phi_ready + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t sbase = smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x % ntiles;
  const int split = blockIdx.x / ntiles;
  const int64_t c0 = (int64_t)tile * CW;
  const int64_t nC = 4 * C;
  const int64_t blk0 = nblk * split / nsplit, blk1 = nblk * (split + 1) / nsplit;
  const int nb = (int)(blk1 - blk0);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(F::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 32) {
    prefetch_tmap(&gmap);
    prefetch_tmap(&xmap);
    prefetch_tmap(&omap);
    for (int st = 0; st < SG; ++st) { mbar_init(&gfull[st], 1); mbar_init(&gfree[st], F::E_WARPS + 4); }
    for (int st = 0; st < SI; ++st) { mbar_init(&ifull[st], 1); mbar_init(&ifree[st], 2 + F::E_WARPS); }
    for (int b = 0; b < ND; ++b) {
      mbar_init(&a2_ready[b], 4);
      mbar_init(&a2_free[b], 1);
      mbar_init(&d1_full[b], 1);
      mbar_init(&d1_free[b], 4);
      mbar_init(&loc_ready[b], F::E_WARPS);
      mbar_init(&loc_free[b], 1);
    }
    mbar_init(d2_done, 1);
    mbar_init(phi_ready, 4);
    *abort_word = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int gi = 0, ii = 0;
      for (int j = 0; j < nb; ++j) {
        const int sg = j % SG, si = j % SI;
        if (j >= SG && !mbar_wait_or_abort(&gfree[sg], (uint32_t)(((j / SG) - 1) & 1), abort_word)) {
          *abort_word = 1;
          break;
        }
        const int64_t blk = blk0 + j;
        const int row = (int)(blk * TOK * 4);
        unsigned char* gb = sm + sg * 2 * SM::GB;
        mbar_expect_tx(&gfull[sg], 2 * SM::GB);
        tma_load_2d(gb, &gmap, (int)c0, row, &gfull[sg]);
        tma_load_2d(gb + SM::GB, &xmap, (int)c0, row, &gfull[sg]);
        gi = j + 1;
        if (j >= SI && !mbar_wait_or_abort(&ifree[si], (uint32_t)(((j / SI) - 1) & 1), abort_word)) {
          *abort_word = 1;
          break;
        }
        mbar_expect_tx(&ifull[si], F::IMG);
        bulk_load(sm + SM::OFF_IMG + si * F::IMG, img + blk * F::IMG_FLOATS, F::IMG, &ifull[si]);
        ii = j + 1;
      }
      // no copy may still be landing when the CTA exits (bounded)
      for (int q = gi > SG ? gi - SG : 0; q < gi; ++q) mbar_wait(&gfull[q % SG], (uint32_t)((q / SG) & 1));
      for (int q = ii > SI ? ii - SI : 0; q < ii; ++q) mbar_wait(&ifull[q % SI], (uint32_t)((q / SI) & 1));
    }
  } else if (warp == 1) {
    // ---------------- D1 issuer ----------------
    if (lane == 0) {
      constexpr uint32_t ID1 = umma_idesc_tf32(128, TOK);
      if (nb > 0 && !mbar_wait_or_abort(phi_ready, 0u, abort_word)) *abort_word = 1;
      for (int j = 0; j < nb && !*abort_word; ++j) {
        const int si = j % SI, b = j % ND;
        if (!mbar_wait_or_abort(&ifull[si], (uint32_t)((j / SI) & 1), abort_word)) { *abort_word = 1; break; }
        if (j >= ND && !mbar_wait_or_abort(&d1_free[b], (uint32_t)(((j / ND) - 1) & 1), abort_word)) {
          *abort_word = 1;
          break;
        }
        tc_fence_after();
        const uint32_t im = sbase + SM::OFF_IMG + si * F::IMG;
#pragma unroll
        for (int ks = 0; ks < 3; ++ks) {
          const uint32_t ah = tmem + F::A1_COL + 8 * ks, al = tmem + F::A1L_COL + 8 * ks;
          const uint64_t bh = umma_desc_k(im + F::IMG_B1H * 4, TOK, ks, 0);
          const uint64_t bl = umma_desc_k(im + F::IMG_B1L * 4, TOK, ks, 0);
          umma_tf32_at(tmem + TOK * b, al, bh, ID1, ks > 0 ? 1u : 0u);
          umma_tf32_at(tmem + TOK * b, ah, bl, ID1, 1u);
          umma_tf32_at(tmem + TOK * b, ah, bh, ID1, 1u);
        }
        umma_commit(&d1_full[b]);
        umma_commit(&ifree[si]);
      }
    }
  } else if (warp == F::D2_WARP) {
    // ---------------- D2 issuer ----------------
    if (lane == 0) {
      constexpr uint32_t ID2 = umma_idesc_tf32(128, F::KP);
      for (int j = 0; j < nb; ++j) {
        const int si = j % SI, b = j % ND;
        if (!mbar_wait_or_abort(&ifull[si], (uint32_t)((j / SI) & 1), abort_word)) { *abort_word = 1; break; }
        if (!mbar_wait_or_abort(&a2_ready[b], (uint32_t)((j / ND) & 1), abort_word)) { *abort_word = 1; break; }
        tc_fence_after();
        const uint32_t im = sbase + SM::OFF_IMG + si * F::IMG;
        const uint32_t a2 = tmem + F::XT_COL + 2 * TOK * b;
#pragma unroll
        for (int ks = 0; ks < TOK / 8; ++ks) {
          const uint32_t ah = a2 + 8 * ks, al = a2 + TOK + 8 * ks;
          const uint64_t bh = umma_desc_k(im + F::IMG_B2H * 4, F::KP, ks, 0);
          const uint64_t bl = umma_desc_k(im + F::IMG_B2L * 4, F::KP, ks, 0);
          if constexpr (SM::BF16) {
            umma_tf32_at(tmem + F::D2_COL, ah, bl, ID2, (j > 0 || ks > 0) ? 1u : 0u);
            umma_tf32_at(tmem + F::D2_COL, ah, bh, ID2, 1u);
          } else {
            umma_tf32_at(tmem + F::D2_COL, al, bh, ID2, (j > 0 || ks > 0) ? 1u : 0u);
            umma_tf32_at(tmem + F::D2_COL, ah, bl, ID2, 1u);
            umma_tf32_at(tmem + F::D2_COL, ah, bh, ID2, 1u);
          }
        }
        umma_commit(&a2_free[b]);
        umma_commit(&ifree[si]);
      }
      umma_commit(d2_done);
    }
  } else if (warp >= F::XT_WARP0) {
    // ---------------- X^T operand into tensor memory ----------------
    const int q = warp & 3;                  // stream = tensor-memory lane quadrant
    {
      // resident Phi^T (A of D1): lane = column (stream q, channel lane), column = k
      const float* ph = nullptr;
      uint32_t hi[24], lo[24];
#pragma unroll
      for (int k = 0; k < F::NH; ++k) {
        ph = phi_row(phi_pre, phi_post, phi_res, k, 4, nC);
        split_tf32(__ldg(ph + (int64_t)q * C + c0 + lane), hi[k], lo[k]);
      }
      const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16);
#pragma unroll
      for (int k8 = 0; k8 < 3; ++k8) {
        tmem_st8(ta + F::A1_COL + 8 * k8, *reinterpret_cast<const uint32_t(*)[8]>(hi + 8 * k8));
        tmem_st8(ta + F::A1L_COL + 8 * k8, *reinterpret_cast<const uint32_t(*)[8]>(lo + 8 * k8));
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(phi_ready);
    }
    for (int j = 0; j < nb; ++j) {
      const int sg = j % SG, b = j % ND;
      if (!mbar_wait_or_abort(&gfull[sg], (uint32_t)((j / SG) & 1), abort_word)) { *abort_word = 1; break; }
      const T* xs = reinterpret_cast<const T*>(sm + sg * 2 * SM::GB) + SM::GB / sizeof(T);
      float xv[TOK];
#pragma unroll
      for (int t = 0; t < TOK; ++t) xv[t] = to_f32(xs[(t * 4 + q) * CW + lane]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&gfree[sg]);
      if (j >= ND && !mbar_wait_or_abort(&a2_free[b], (uint32_t)(((j / ND) - 1) & 1), abort_word)) { *abort_word = 1; break; }
      tc_fence_after();
      const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + F::XT_COL + 2 * TOK * b;
#pragma unroll
      for (int hf = 0; hf < TOK / 16; ++hf) {
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          if constexpr (SM::BF16) hi[t] = __float_as_uint(xv[16 * hf + t]);   // exact in tf32
          else split_tf32(xv[16 * hf + t], hi[t], lo[t]);
        }
        tmem_st16(ta + 16 * hf, hi);
        if constexpr (!SM::BF16) tmem_st16(ta + TOK + 16 * hf, lo);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a2_ready[b]);
    }
  } else {
    const int64_t c = c0 + lane;
    float* locs = reinterpret_cast<float*>(sm + SM::OFF_LOC);
    float* gws = reinterpret_cast<float*>(sm + SM::OFF_GW);
    bool ok = true;
    constexpr int TPE = F::TPE;
    if (warp < 2 + F::E_WARPS) {
      // ---------------- E: X^T operand and local terms ----------------
      const int e = warp - 2;                // tokens TPE e .. TPE e + TPE - 1
      const float wc = __ldg(w + c);
      float gwacc = 0.f;
      for (int j = 0; j < nb; ++j) {
        const int sg = j % SG, si = j % SI, b = j % ND;
        if (!mbar_wait_or_abort(&gfull[sg], (uint32_t)((j / SG) & 1), abort_word)) { ok = false; break; }
        const T* gs = reinterpret_cast<const T*>(sm + sg * 2 * SM::GB);
        const T* xs = gs + SM::GB / sizeof(T);
        float gv[TPE][4], xv[TPE][4];        // [token][stream]
#pragma unroll
        for (int u = 0; u < TPE; ++u)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            gv[u][jj] = to_f32(gs[((TPE * e + u) * 4 + jj) * CW + lane]);
            xv[u][jj] = to_f32(xs[((TPE * e + u) * 4 + jj) * CW + lane]);
          }
        __syncwarp();
        if (lane == 0) mbar_arrive(&gfree[sg]);   // g, x now live in registers
        if (!mbar_wait_or_abort(&ifull[si], (uint32_t)((j / SI) & 1), abort_word)) { ok = false; break; }
        const float* sc = reinterpret_cast<const float*>(sm + SM::OFF_IMG + si * F::IMG) + F::IMG_SC;
        // local terms of the four streams
        if (j >= ND && !mbar_wait_or_abort(&loc_free[b], (uint32_t)(((j / ND) - 1) & 1), abort_word)) { ok = false; break; }
        float* lb = locs + b * (F::LOCB / 4);
#pragma unroll
        for (int u = 0; u < TPE; ++u) {
          const int t = TPE * e + u;
          const float* st = sc + t * 32;
          const float4 s0 = *reinterpret_cast<const float4*>(st);
          const float4 h4 = *reinterpret_cast<const float4*>(st + 4);
          const float4 q4 = *reinterpret_cast<const float4*>(st + 8);
          const float gy = q4.x * gv[u][0] + q4.y * gv[u][1] + q4.z * gv[u][2] + q4.w * gv[u][3];
          const float xa = h4.x * xv[u][0] + h4.y * xv[u][1] + h4.z * xv[u][2] + h4.w * xv[u][3];
          const float agg = gy * wc * s0.y - xa * s0.x;
          const float hh[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 m4 = *reinterpret_cast<const float4*>(st + 12 + 4 * i);
            const float mix = m4.x * gv[u][0] + m4.y * gv[u][1] + m4.z * gv[u][2] + m4.w * gv[u][3];
            lb[t * COLS + i * CW + lane] = mix + hh[i] * agg + s0.z * xv[u][i];
          }
          gwacc = fmaf(gy * xa, s0.y, gwacc);
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&loc_ready[b]);
          mbar_arrive(&ifree[si]);
        }
      }
      gws[e * CW + lane] = gwacc;
    } else {
      // ---------------- epilogue: grad_x = D1 + local term ----------------
      const int i = warp & 3;                // stream = tensor-memory lane quadrant
      const bool leader = warp == 2 + F::E_WARPS && lane == 0;
      for (int j = 0; j < nb; ++j) {
        const int b = j % ND;
        if (!mbar_wait_or_abort(&d1_full[b], (uint32_t)((j / ND) & 1), abort_word)) { ok = false; break; }
        if (!mbar_wait_or_abort(&loc_ready[b], (uint32_t)((j / ND) & 1), abort_word)) { ok = false; break; }
        tc_fence_after();
        float* lb = locs + b * (F::LOCB / 4) + i * CW + lane;
        __nv_bfloat16* sb16 = reinterpret_cast<__nv_bfloat16*>(sm + SM::OFF_STG + b * SM::STGB) + i * CW + lane;
#pragma unroll
        for (int hf = 0; hf < TOK / 16; ++hf) {
          float d[16];
          tmem_ld16(tmem + ((uint32_t)(32 * i) << 16) + TOK * b + 16 * hf, d);
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            if constexpr (SM::BF16) sb16[(16 * hf + t) * COLS] = __float2bfloat16_rn(lb[(16 * hf + t) * COLS] + d[t]);
            else lb[(16 * hf + t) * COLS] += d[t];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d1_free[b]);
        fence_proxy_async_smem();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (leader) {
          tma_store_2d(&omap, SM::BF16 ? static_cast<const void*>(sm + SM::OFF_STG + b * SM::STGB)
                                       : static_cast<const void*>(locs + b * (F::LOCB / 4)),
                       (int)c0, (int)((blk0 + j) * TOK * 4));
          bulk_commit();
          // the previous block's buffer may be refilled once its store has read it
          if (j > 0) {
            asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
            mbar_arrive(&loc_free[(j - 1) % ND]);
          }
        }
      }
      if (leader) {
        bulk_wait0();
        if (ok && nb > 0) mbar_arrive(&loc_free[(nb - 1) % ND]);
      }
    }
    if (!ok) *abort_word = 1;
    asm volatile("bar.sync 1, %0;" ::"r"(32 * (F::E_WARPS + 4)) : "memory");
    ok = *abort_word == 0;
    if (warp >= 2 + F::E_WARPS) {
      const int i = warp & 3;
      bool have = ok && nb > 0 && mbar_wait_or_abort(d2_done, 0u, abort_word);
      have = __all_sync(0xffffffffu, have);
      const bool write = have || (ok && nb == 0);
      tc_fence_after();
      float a[16], bb[16];
      if (have) {
        tmem_ld16(tmem + ((uint32_t)(32 * i) << 16) + F::D2_COL, a);
        tmem_ld16(tmem + ((uint32_t)(32 * i) << 16) + F::D2_COL + 16, bb);
      } else {
#pragma unroll
        for (int q = 0; q < 16; ++q) { a[q] = 0.f; bb[q] = 0.f; }
      }
      if (write) {
        float* dd = dphi_part + (int64_t)split * F::NH * nC + (int64_t)i * C + c;
#pragma unroll
        for (int k = 0; k < 16; ++k) dd[(int64_t)k * nC] = a[k];
#pragma unroll
        for (int k = 16; k < F::NH; ++k) dd[(int64_t)k * nC] = bb[k - 16];
        if (i == 0) {
          float gsum = 0.f;
#pragma unroll
          for (int q = 0; q < F::E_WARPS; ++q) gsum += gws[q * CW + lane];
          gw_part[(int64_t)split * C + c] = gsum;
        }
      }
    }
  }
  if (warp == F::D2_WARP && lane == 0 && nb > 0) mbar_wait_or_abort(d2_done, 0u, abort_word);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(F::TMEM_COLS));
}

// out[l] = sum_s part[s * L + l]   (fixed order over splits)
__global__ void __launch_bounds__(256)
    reduce_splits_kernel(const float* __restrict__ part, int nsplit, int64_t L,
                         float* __restrict__ out) {
  for (int64_t l = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; l < L;
       l += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < nsplit; ++k) s += part[(int64_t)k * L + l];
    out[l] = s;
  }
}


// One CTA per column v of a [B, stride] fp64 table: total[v] = sum_b tab[b, v]
// (fixed order: thread-strided partials, then a fixed tree).
__global__ void __launch_bounds__(256)
    reduce_tokens_kernel(const double* __restrict__ tab, int64_t B, int stride,
                         double* __restrict__ out) {
  __shared__ double red[8];
  const int v = blockIdx.x;
  double s = 0.0;
  for (int64_t b = threadIdx.x; b < B; b += blockDim.x) s += tab[b * stride + v];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[k];
    out[v] = t;
  }
}


// Tail of the dynamic backward in one launch.  Blocks [0, nb_dphi) sum the
// dphi split partials into the three phi gradients, the next nb_gw blocks the
// grad-w split partials, the last nb_tok blocks reduce the per-token rows
// [B, NR] (dt, dalpha) to block partials; the last of those to finish sums
// the partials in block order and scatters the bias / alpha gradients.  The
// arrival counter is zeroed by token_bwd earlier on the same stream.  Every
// sum runs in a fixed order (bitwise reproducible).
template <int N>
__global__ void __launch_bounds__(256)
    finish_dyn_bwd_kernel(const float* __restrict__ dphi_part, const float* __restrict__ gw_part,
                          int nsplit, int64_t C, float* __restrict__ d_pre,
                          float* __restrict__ d_post, float* __restrict__ d_res,
                          float* __restrict__ gw, const double* __restrict__ tokr, int64_t B,
                          double* __restrict__ tok_part, unsigned int* __restrict__ counter,
                          int nb_dphi, int nb_gw, int nb_tok, float* __restrict__ gbp,
                          float* __restrict__ gbq, float* __restrict__ gbr, float* __restrict__ gap,
                          float* __restrict__ gaq, float* __restrict__ gar) {
  constexpr int NH = L<N>::NH, NR = L<N>::NR, RL = 256 / NR;
  const int64_t nC = (int64_t)N * C;
  const int bid = blockIdx.x, tid = threadIdx.x;
  if (bid < nb_dphi) {
    const int64_t Ld = (int64_t)NH * nC;
    for (int64_t l = (int64_t)bid * 256 + tid; l < Ld; l += (int64_t)nb_dphi * 256) {
      float sacc = 0.f;
      for (int k = 0; k < nsplit; ++k) sacc += dphi_part[(int64_t)k * Ld + l];
      const int64_t kk = l / nC, cc = l % nC;
      float* dst = kk < N ? d_pre + kk * nC : (kk < 2 * N ? d_post + (kk - N) * nC : d_res + (kk - 2 * N) * nC);
      dst[cc] = sacc;
    }
    return;
  }
  if (bid < nb_dphi + nb_gw) {
    for (int64_t l = (int64_t)(bid - nb_dphi) * 256 + tid; l < C; l += (int64_t)nb_gw * 256) {
      float sacc = 0.f;
      for (int k = 0; k < nsplit; ++k) sacc += gw_part[(int64_t)k * C + l];
      gw[l] = sacc;
    }
    return;
  }
  // token rows: thread = (column v, row lane rl), rows of this block's range
  __shared__ double red[256];
  __shared__ bool last;
  const int kb = bid - nb_dphi - nb_gw;
  const int64_t r0 = B * kb / nb_tok, r1 = B * (kb + 1) / nb_tok;
  const int v = tid % NR, rl = tid / NR;
  double sacc = 0.0;
  if (rl < RL)
    for (int64_t r = r0 + rl; r < r1; r += RL) sacc += tokr[r * NR + v];
  red[tid] = sacc;
  __syncthreads();
  if (tid < NR) {
    double t = 0.0;
    for (int q = 0; q < RL; ++q) t += red[q * NR + tid];
    tok_part[(int64_t)kb * NR + tid] = t;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(counter, 1u) == (unsigned)(nb_tok - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (tid < NR) {
    double t = 0.0;
    for (int q = 0; q < nb_tok; ++q) t += *(volatile const double*)(tok_part + (int64_t)q * NR + tid);
    if (tid < N) gbp[tid] = (float)t;
    else if (tid < 2 * N) gbq[tid - N] = (float)t;
    else if (tid < NH) gbr[tid - 2 * N] = (float)t;
    else if (tid == NH) *gap = (float)t;
    else if (tid == NH + 1) *gaq = (float)t;
    else *gar = (float)t;
  }
  if (tid == 0) *counter = 0u;
}

// Static-H parameter gradients from the token totals [dt_pre, dt_post, gM]:
// the Sinkhorn reverse runs once on the batch-summed gM (M is shared).
template <int N>
__global__ void static_param_grads_kernel(const double* __restrict__ tot,
                                          const float* __restrict__ H_res,
                                          float* __restrict__ gHp, float* __restrict__ gHq,
                                          float* __restrict__ gHr, int iters, float s_eps) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  for (int i = 0; i < N; ++i) { gHp[i] = (float)tot[i]; gHq[i] = (float)tot[N + i]; }
  double e0[N * N], gm[N * N];
#pragma unroll
  for (int e = 0; e < N * N; ++e) { e0[e] = exp((double)H_res[e]); gm[e] = tot[2 * N + e]; }
  sk_backward<N, double>(e0, gm, iters, (double)s_eps);
#pragma unroll
  for (int e = 0; e < N * N; ++e) gHr[e] = (float)(gm[e] * e0[e]);
}

// ---------------------------------------------------------------------------
// Host-side planning
// ---------------------------------------------------------------------------
inline size_t align_up(size_t v) { return (v + 255) & ~(size_t)255; }

struct Carve {
  char* base;
  size_t off = 0;
  explicit Carve(void* p) : base((char*)p) {}
  float* take(size_t floats) {
    float* p = base ? (float*)(base + off) : nullptr;
    off += align_up(floats * sizeof(float));
    return p;
  }
};

int choose_ksplit(int64_t tiles, int64_t C, int sms) {
  const int64_t max_ks = (C + 31) / 32;
  int best = 1;
  double best_eff = -1.0;
  for (int ks = 1; ks <= 32 && ks <= max_ks; ++ks) {
    const int64_t total = tiles * ks;
    const int64_t waves = (total + sms - 1) / sms;
    double eff = (double)total / (double)(waves * sms);
    if (total < 2 * sms) eff *= (double)total / (2.0 * sms);  // too little parallelism
    if (eff > best_eff + 0.02) { best_eff = eff; best = ks; }
  }
  return best;
}

// Channel splits of the tensor-core projection: minimise waves x (32-channel
// blocks per CTA + a fixed per-CTA cost), at most 1024 channels per split.
int choose_proj_splits(int64_t tiles, int64_t C, int slots) {
  const int64_t nblk = (C + 31) / 32;
  int64_t lo = (C + 1023) / 1024;
  if (lo < 1) lo = 1;
  const int64_t hi = nblk < 64 ? nblk : 64;
  int best = (int)lo;
  double best_cost = 1e300;
  for (int64_t ks = lo; ks <= hi || ks == lo; ++ks) {
    const int64_t waves = (tiles * ks + slots - 1) / slots;
    const int64_t blocks = (nblk + ks - 1) / ks;
    const double cost = (double)waves * (double)(blocks + 3);
    if (cost < best_cost) { best_cost = cost; best = (int)ks; }
  }
  return best;
}

int choose_gx_splits(int64_t tiles, int64_t B, int sms, int per_sm) {
  const int64_t slots = (int64_t)sms * per_sm;
  int best = 1;
  double best_eff = -1.0;
  const int64_t max_s = B < 1 ? 1 : (B < 1024 ? B : 1024);
  for (int64_t s = 1; s <= max_s; ++s) {
    const int64_t total = tiles * s;
    const int64_t waves = (total + slots - 1) / slots;
    double eff = (double)total / (double)(waves * slots);
    if (waves > 8) break;
    // prefer fewer splits (less partial traffic) unless clearly better balanced
    if (eff > best_eff + 0.01) { best_eff = eff; best = (int)s; }
  }
  return best;
}

struct FwdPlan {
  int ks, cps;
  int64_t tiles;
  int uks, ucps;     // splits of the tensor-core projection (n <= 4, C % 8 == 0)
  int64_t utiles;
  size_t ppart, gpart, rec_tmp, phiT;
};

template <int N>
FwdPlan plan_fwd(int64_t B, int64_t C) {
  FwdPlan p;
  p.tiles = (B + ProjCfg<N>::TT - 1) / ProjCfg<N>::TT;
  p.ks = choose_ksplit(p.tiles, C, num_sms());
  p.cps = (int)(((C + p.ks - 1) / p.ks + 31) / 32 * 32);
  p.ks = (int)((C + p.cps - 1) / p.cps);
  int mks = p.ks;
  p.uks = 0; p.ucps = 0; p.utiles = 0;
  size_t uphi = 0;
  if (N <= 4 && C % 4 == 0) {
    p.utiles = (B + 127) / 128;
    const int ks = choose_proj_splits(p.utiles, C, 2 * num_sms());
    p.ucps = (int)(((C + ks - 1) / ks + 31) / 32 * 32);
    p.uks = (int)((C + p.ucps - 1) / p.ucps);
    // the fallback projections (misaligned x) reuse this split plan, so the
    // partial buffers are sized for the plan that actually runs
    p.ks = p.uks;
    p.cps = p.ucps;
    mks = p.uks;
    uphi = (size_t)2 * PumCfg<(N <= 4 ? N : 4)>::NB * N * C;
  }
  p.ppart = (size_t)mks * B * L<N>::NHP;
  p.gpart = (size_t)mks * B * L<N>::NG;
  p.rec_tmp = (size_t)B * L<N>::REC;
  p.phiT = N <= 4 ? (size_t)C * PjtCfg<(N <= 4 ? N : 4)>::PROW : 0;
  if (uphi > p.phiT) p.phiT = uphi;
  return p;
}

constexpr int kTokPartBlocks = 64;

struct BwdPlan {
  int ntiles, nsplit;
  int64_t nblk6;  // token blocks of the warp-specialised grad_x (n = 4, dynamic H)
  int nsplit6;
  size_t img;
  size_t stats, tokb, tokr, dphi, gw, tot;
};

template <int N, bool DYN>
BwdPlan plan_bwd(int64_t B, int64_t C) {
  BwdPlan p;
  p.ntiles = (int)((C + GX_CW - 1) / GX_CW);
  p.nsplit = choose_gx_splits(p.ntiles, B, num_sms(), N <= 4 ? 2 : 1);
  p.nblk6 = (N == 4 && DYN) ? (B + Gx6Cfg::TOK - 1) / Gx6Cfg::TOK : 0;
  p.nsplit6 = (N == 4 && DYN && p.nblk6 > 0) ? choose_gx_splits((C + 31) / 32, p.nblk6, num_sms(), 1) : 0;
  p.img = (size_t)p.nblk6 * Gx6Cfg::IMG_FLOATS;
  int64_t msplit = p.nsplit;
  if (p.nsplit6 > msplit) msplit = p.nsplit6;
  p.stats = (size_t)B * (DYN ? L<N>::NSD : L<N>::NS1) * 2;  // fp64
  p.tokb = (size_t)B * L<N>::TB;
  p.tokr = (size_t)B * (DYN ? L<N>::NR : L<N>::NRS) * 2;  // fp64
  p.dphi = DYN ? (size_t)msplit * L<N>::NH * N * C : 0;
  p.gw = (size_t)msplit * C;
  // dynamic: per-block token partials of finish_dyn_bwd + its arrival counter
  p.tot = DYN ? (size_t)kTokPartBlocks * L<N>::NR * 2 + 4 : (size_t)L<N>::NRS * 2;  // fp64
  return p;
}

template <int N>
size_t fwd_ws_bytes(int64_t B, int64_t C, bool need_rec) {
  FwdPlan p = plan_fwd<N>(B, C);
  Carve cv(nullptr);
  cv.take(p.ppart);
  cv.take(p.gpart);
  cv.take(p.phiT);
  if (need_rec) cv.take(p.rec_tmp);
  return cv.off;
}

template <int N, bool DYN>
size_t bwd_ws_bytes(int64_t B, int64_t C) {
  BwdPlan p = plan_bwd<N, DYN>(B, C);
  Carve cv(nullptr);
  cv.take(p.stats); cv.take(p.tokb); cv.take(p.tokr); cv.take(p.dphi); cv.take(p.gw);
  cv.take(p.tot);
  cv.take(p.img);
  if (!DYN) cv.take(L<N>::REC);
  return cv.off;
}

// Per-token kernels run one thread per token with long dependent fp64
// chains; one-warp blocks spread a few thousand tokens over every SM.
constexpr int kTokThreads = 32;

inline unsigned grid_1d(int64_t n, int threads, int64_t cap = 1 << 30) {
  int64_t g = (n + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (unsigned)g;
}

// Launch the TMA-pipelined grad_x when the layout allows it; false -> caller
// uses the generic kernel.
template <int N, bool DYN>
bool launch_grad_x_tma(const float* g, const float* x, const float* w, const float* pp,
                       const float* pq, const float* pr, const float* tokb, float* gx,
                       float* dphi, float* gwp, int64_t B, int64_t C, const BwdPlan& p,
                       int* nsplit_used, cudaStream_t s) {
  *nsplit_used = p.nsplit;
  if constexpr (N > 4) {
    return false;
  } else {
    if constexpr (N == 4) {
      using F = Gx4Cfg;
      CUtensorMap gm, xm, tm, om;
      if (C % 64 == 0 && aligned16(g) && aligned16(x) && aligned16(tokb) && aligned16(gx) &&
          (!DYN || aligned16(dphi)) &&
          make_tmap_2d_f32(&gm, g, (uint64_t)B * N, C, C, F::TOK * N, F::CW) &&
          make_tmap_2d_f32(&om, gx, (uint64_t)B * N, C, C, F::TOK * N, F::CW) &&
          make_tmap_2d_f32(&xm, x, (uint64_t)B * N, C, C, F::TOK * N, F::CW) &&
          make_tmap_2d_f32(&tm, tokb, B, L<N>::TB, L<N>::TB, F::TOK, L<N>::TB)) {
        cudaFuncSetAttribute(grad_x4_kernel<DYN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)F::SMEM);
        { ProfScope _ps("grad_x", s); grad_x4_kernel<DYN><<<(unsigned)(p.ntiles * p.nsplit), 256, F::SMEM, s>>>(
            gm, xm, tm, om, w, pp, pq, pr, gx, dphi, gwp, B, C, p.ntiles, p.nsplit); }
        return true;
      }
    }
    using Cf = GxtCfg<N>;
    CUtensorMap gmap, xmap, tmap;
    if (C % 4 != 0 || !aligned16(g) || !aligned16(x) || !aligned16(tokb)) return false;
    if (!make_tmap_2d_f32(&gmap, g, (uint64_t)B * N, C, C, Cf::ROWS, GX_CW) ||
        !make_tmap_2d_f32(&xmap, x, (uint64_t)B * N, C, C, Cf::ROWS, GX_CW) ||
        !make_tmap_2d_f32(&tmap, tokb, B, L<N>::TB, L<N>::TB, GXT_TB, L<N>::TB))
      return false;
    cudaFuncSetAttribute(grad_x_tma_kernel<N, DYN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)Cf::SMEM);
    { ProfScope _ps("grad_x", s); grad_x_tma_kernel<N, DYN><<<(unsigned)(p.ntiles * p.nsplit), GX_CW * N, Cf::SMEM, s>>>(
        gmap, xmap, tmap, w, pp, pq, pr, gx, dphi, gwp, B, C, p.ntiles, p.nsplit); }
    return true;
  }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
template <typename T> constexpr CUtensorMapDataType tmap_dtype() {
  return sizeof(T) == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
}

// T = float, or __nv_bfloat16 for bf16 streams (x, out; fp32 arithmetic), which
// needs the tensor-core projection (n <= 4, C % 64 == 0, 16-byte aligned).
template <int N, typename T = float>
int run_fwd_dynamic(const T* x, const float* w, const float* pp, const float* pq,
                    const float* pr, const float* ap, const float* aq, const float* ar,
                    const float* bp, const float* bq, const float* br, T* out,
                    float* token_state, int64_t B, int64_t C, int iters, float s_eps,
                    float r_eps, void* ws, size_t ws_bytes, cudaStream_t s) {
  const bool need_rec = token_state == nullptr;
  const size_t need = fwd_ws_bytes<N>(B, C, need_rec);
  MHC_REQUIRE(ws != nullptr && ws_bytes >= need, MHC_ERR_WORKSPACE,
              "mhc_layer_fwd_dynamic: workspace of %zu bytes required, got %zu", need, ws_bytes);
  FwdPlan p = plan_fwd<N>(B, C);
  Carve cv(ws);
  float* ppart = cv.take(p.ppart);
  float* gpart = cv.take(p.gpart);
  float* phiT = cv.take(p.phiT);
  float* rec = need_rec ? cv.take(p.rec_tmp) : token_state;

  int rc = MHC_OK;
  bool done = false;
  int ks = p.ks;
  if constexpr (N <= 4) {
    // tcgen05 projection: phi split once into tf32 hi/lo rows, x streamed by TMA.
    using PU = PumCfg<N, T>;
    const int64_t nC = (int64_t)N * C;
    float* ph = phiT;
    float* pl = phiT + (size_t)PU::NB * nC;
    CUtensorMap xmap, hmap, lmap;
    const uint64_t cs = (uint64_t)C * 4, rs = (uint64_t)nC * 4;
    const uint64_t xcs = (uint64_t)C * sizeof(T), xrs = (uint64_t)nC * sizeof(T);
    // channels per split: a multiple of the stage width
    const int ucps = (p.ucps + PU::CH - 1) / PU::CH * PU::CH;
    const int uks = p.ucps > 0 ? (int)((C + ucps - 1) / ucps) : 0;
    if (p.uks > 0 && B > 0 && C % PU::CH == 0 && aligned16(x) && aligned16(ph) && aligned16(pl) &&
        make_tmap_3d(&xmap, tmap_dtype<T>(), x, C, N, B, xcs, xrs, PU::CH, 1, PU::TOK, CU_TENSOR_MAP_SWIZZLE_128B) &&
        make_tmap_3d_f32(&hmap, ph, C, N, PU::NB, cs, rs, 32, 1, PU::NB, CU_TENSOR_MAP_SWIZZLE_128B) &&
        make_tmap_3d_f32(&lmap, pl, C, N, PU::NB, cs, rs, 32, 1, PU::NB, CU_TENSOR_MAP_SWIZZLE_128B)) {
      {
        const bool pvec = nC % 4 == 0 && aligned16(pp) && aligned16(pq) && aligned16(pr);
        ProfScope _ps("phi_split", s);
        phi_split_kernel<N><<<dim3(grid_1d(pvec ? nC / 4 : nC, 256, 64), PU::NB), 256, 0, s>>>(pp, pq, pr, ph, pl, C, pvec);
      }
      cudaFuncSetAttribute(proj_umma_kernel<N, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PU::SMEM);
      { ProfScope _ps("proj_stats", s); proj_umma_kernel<N, T><<<dim3((unsigned)p.utiles, (unsigned)uks), PU::THREADS, PU::SMEM, s>>>(
          xmap, hmap, lmap, ppart, gpart, B, C, ucps); }
      ks = uks;
      done = true;
    }
  }
  if constexpr (sizeof(T) == 2) {
    MHC_REQUIRE(done, MHC_ERR_UNSUPPORTED,
                "mhc_layer_fwd_dynamic_bf16: needs n <= 4, hidden %% 64 == 0 and 16-byte aligned x");
  }
  if constexpr (N <= 4 && sizeof(T) == 4) if (!done) {
    // TMA-pipelined projection when the layout allows it.
    using PT = PjtCfg<N>;
    CUtensorMap xmap, pmap;
    if (C % 4 == 0 && aligned16(x) && aligned16(phiT) &&
        make_tmap_2d_f32(&xmap, x, (uint64_t)B * N, C, C, PT::TT * N, 32) &&
        make_tmap_2d_f32(&pmap, phiT, C, PT::PROW, PT::PROW, 32, PT::PROW)) {
      { ProfScope _ps("phi_transpose", s); phi_transpose_kernel<N><<<grid_1d(C * PT::PROW, 256, 2048), 256, 0, s>>>(pp, pq, pr, phiT, C); }
      cudaFuncSetAttribute(proj_stats_tma_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)PT::SMEM);
      { ProfScope _ps("proj_stats", s); proj_stats_tma_kernel<N><<<dim3((unsigned)p.tiles, (unsigned)p.ks), PJT_THREADS, PT::SMEM, s>>>(
          xmap, pmap, ppart, gpart, B, C, p.cps); }
      done = true;
    }
  }
  if constexpr (sizeof(T) == 4) if (!done) {
    using P = ProjCfg<N>;
    const size_t smem = (size_t)P::SMEM_FLOATS * sizeof(float);
    // Opt in to > 48 KB of dynamic shared memory (cheap, idempotent, per device).
    cudaFuncSetAttribute(proj_stats_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    { ProfScope _ps("proj_stats", s); proj_stats_kernel<N><<<dim3((unsigned)p.tiles, (unsigned)p.ks), 256, smem, s>>>(
        x, pp, pq, pr, ppart, gpart, B, C, p.cps); }
  }
  rc = check_launch("mhc_layer_fwd_dynamic/proj_stats");
  if (rc) return rc;
  { constexpr int TG = N <= 2 ? 2 : (N <= 4 ? 4 : 8); ProfScope _ps("token_fwd", s); if (B > 0) token_fwd_lanes_kernel<N><<<grid_1d(B * TG, 128), 128, 0, s>>>(ppart, gpart, ks, ap, aq, ar, bp, bq, br,
                                                     rec, B, C, iters, s_eps, r_eps); }
  rc = check_launch("mhc_layer_fwd_dynamic/token_fwd");
  if (rc) return rc;
  const bool vec = (C % 4 == 0) && aligned16(x) && aligned16(out) && aligned16(w);
  const unsigned grid = (unsigned)(B < (1 << 30) ? B : (1 << 30));
  // the fp64 Gram matrix is only needed when the record is kept for a backward
  if (vec && !need_rec)
    { ProfScope _ps("stream_fwd", s); stream_fwd_kernel<N, true, true, T><<<grid, 256, 0, s>>>(x, w, rec, L<N>::REC, nullptr, out, B, C, rec); }
  else if (vec)
    { ProfScope _ps("stream_fwd", s); stream_fwd_kernel<N, true, false, T><<<grid, 256, 0, s>>>(x, w, rec, L<N>::REC, nullptr, out, B, C, rec); }
  else if constexpr (sizeof(T) == 2)
    return fail(MHC_ERR_ALIGNMENT, "mhc_layer_fwd_dynamic_bf16: out and weight must be 16-byte aligned");
  else if (!need_rec)
    { ProfScope _ps("stream_fwd", s); stream_fwd_kernel<N, false, true><<<grid, 256, 0, s>>>(x, w, rec, L<N>::REC, nullptr, out, B, C, rec); }
  else
    { ProfScope _ps("stream_fwd", s); stream_fwd_kernel<N, false, false><<<grid, 256, 0, s>>>(x, w, rec, L<N>::REC, nullptr, out, B, C, rec); }
  return check_launch("mhc_layer_fwd_dynamic/stream_fwd");
}

// T = float, or __nv_bfloat16 for bf16 streams (grad_out, x, grad_x; fp32
// arithmetic), which needs the tensor-core grad_x (n = 4, C % 32 == 0, aligned).
template <int N, typename T = float>
int run_bwd_dynamic(const T* g, const T* x, const float* w, const float* pp,
                    const float* pq, const float* pr, const float* ap, const float* aq,
                    const float* ar, const float* bp, const float* bq, const float* br,
                    const float* rec, T* gx, float* gw, float* gpp, float* gpq, float* gpr,
                    float* gap, float* gaq, float* gar, float* gbp, float* gbq, float* gbr,
                    int64_t B, int64_t C, int iters, float s_eps, float r_eps, void* ws,
                    size_t ws_bytes, cudaStream_t s) {
  const size_t need = bwd_ws_bytes<N, true>(B, C);
  MHC_REQUIRE(ws != nullptr && ws_bytes >= need, MHC_ERR_WORKSPACE,
              "mhc_layer_bwd_dynamic: workspace of %zu bytes required, got %zu", need, ws_bytes);
  BwdPlan p = plan_bwd<N, true>(B, C);
  Carve cv(ws);
  double* stats = (double*)cv.take(p.stats);
  float* tokb = cv.take(p.tokb);
  double* tokr = (double*)cv.take(p.tokr);
  float* dphi = cv.take(p.dphi);
  float* gwp = cv.take(p.gw);
  double* tot = (double*)cv.take(p.tot);
  unsigned int* counter = reinterpret_cast<unsigned int*>(tot + (size_t)kTokPartBlocks * L<N>::NR);
  float* img = cv.take(p.img);
  const bool vec = (C % 4 == 0) && aligned16(x) && aligned16(g) && aligned16(w);
  const unsigned grid = (unsigned)(B < (1 << 30) ? B : (1 << 30));
  if constexpr (sizeof(T) == 2) {
    MHC_REQUIRE(N == 4 && vec && C % Gx6Cfg::CW == 0 && p.nsplit6 > 0 && aligned16(gx),
                MHC_ERR_UNSUPPORTED,
                "mhc_layer_bwd_dynamic_bf16: needs n == 4, hidden %% 32 == 0 and 16-byte aligned tensors");
  }
  if (vec) { ProfScope _ps("bwd_stats", s); bwd_stats_kernel<N, true, false, T><<<grid, 128, 0, s>>>(g, x, w, stats, B, C); }
  else if constexpr (sizeof(T) == 4) { ProfScope _ps("bwd_stats", s); bwd_stats_kernel<N, false, false><<<grid, 128, 0, s>>>(g, x, w, stats, B, C); }
  int rc = check_launch("mhc_layer_bwd_dynamic/bwd_stats");
  if (rc) return rc;
  constexpr int TG = N <= 2 ? 2 : (N <= 4 ? 4 : 8);
  // the warp-specialised grad_x (n = 4) reads the operand image token_bwd writes
  const bool use6 = N == 4 && p.nsplit6 > 0 && C % Gx6Cfg::CW == 0 && aligned16(g) && aligned16(x) &&
                    aligned16(img) && aligned16(gx);
  const int64_t img_tokens = use6 ? p.nblk6 * Gx6Cfg::TOK : 0;
  const int64_t tb_tokens = B > img_tokens ? B : img_tokens;
  if (B > 0) { ProfScope _ps("token_bwd", s); token_bwd_lanes_kernel<N><<<grid_1d(tb_tokens * TG, 128), 128, 0, s>>>(stats, rec, ap, aq, ar, bp, bq, br, tokb,
                                                     tokr, B, C, iters, s_eps, r_eps, counter,
                                                     use6 ? img : nullptr, img_tokens); }
  else cudaMemsetAsync(counter, 0, sizeof(unsigned int), s);
  rc = check_launch("mhc_layer_bwd_dynamic/token_bwd");
  if (rc) return rc;
  int nsplit = p.nsplit;
  bool gx_done = false;
  if constexpr (N == 4) {
    // warp-specialised tensor-core grad_x
    using F6 = Gx6Cfg;
    using S6 = Gx6S<T>;
    constexpr CUtensorMapDataType dt = tmap_dtype<T>();
    CUtensorMap gm, xm, om;
    if (use6 &&
        make_tmap_2d(&gm, dt, sizeof(T), g, (uint64_t)B * N, C, C, F6::TOK * N, F6::CW) &&
        make_tmap_2d(&xm, dt, sizeof(T), x, (uint64_t)B * N, C, C, F6::TOK * N, F6::CW) &&
        make_tmap_2d(&om, dt, sizeof(T), gx, (uint64_t)B * N, C, C, F6::TOK * N, F6::CW)) {
      cudaFuncSetAttribute(grad_x6_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S6::SMEM);
      const int nt6 = (int)(C / F6::CW);
      { ProfScope _ps("grad_x", s); grad_x6_kernel<T><<<(unsigned)(nt6 * p.nsplit6), F6::THREADS, S6::SMEM, s>>>(
          gm, xm, om, img, w, pp, pq, pr, gx, dphi, gwp, B, C, nt6, p.nsplit6, p.nblk6); }
      nsplit = p.nsplit6;
      gx_done = true;
    }
  }
  if constexpr (sizeof(T) == 2) {
    MHC_REQUIRE(gx_done, MHC_ERR_UNSUPPORTED, "mhc_layer_bwd_dynamic_bf16: tensor map creation failed");
  } else {
    if (!gx_done && !launch_grad_x_tma<N, true>(g, x, w, pp, pq, pr, tokb, gx, dphi, gwp, B, C, p, &nsplit, s))
      { ProfScope _ps("grad_x", s); grad_x_kernel<N, true><<<(unsigned)(p.ntiles * p.nsplit), GX_CW * N, 0, s>>>(
          g, x, w, pp, pq, pr, tokb, gx, dphi, gwp, B, C, p.ntiles, p.nsplit); }
  }
  rc = check_launch("mhc_layer_bwd_dynamic/grad_x");
  if (rc) return rc;
  const int64_t nC = (int64_t)N * C;
  {
    const int nb_dphi = (int)grid_1d((int64_t)L<N>::NH * nC, 256, 4 * (int64_t)num_sms());
    const int nb_gw = (int)grid_1d(C, 256, 64);
    const int nb_tok = (int)(B / 128 < 1 ? 1 : (B / 128 < kTokPartBlocks ? B / 128 : kTokPartBlocks));
    ProfScope _ps("finish", s);
    finish_dyn_bwd_kernel<N><<<(unsigned)(nb_dphi + nb_gw + nb_tok), 256, 0, s>>>(
        dphi, gwp, nsplit, C, gpp, gpq, gpr, gw, tokr, B, tot, counter, nb_dphi, nb_gw, nb_tok,
        gbp, gbq, gbr, gap, gaq, gar);
  }
  return check_launch("mhc_layer_bwd_dynamic/reduce");
}

template <int N, typename T>
int run_fwd_static(const T* x, const float* w, const float* Hp, const float* Hq, const float* Hr,
                   T* out, float* rms, int64_t B, int64_t C, int iters, float s_eps, float r_eps,
                   void* ws, size_t ws_bytes, cudaStream_t s) {
  MHC_REQUIRE(ws != nullptr && ws_bytes >= align_up(L<N>::REC * sizeof(float)),
              MHC_ERR_WORKSPACE, "mhc_layer_fwd_static: workspace too small");
  float* rec = (float*)ws;
  { ProfScope _ps("static_prep", s); static_prep_kernel<N><<<1, 32, 0, s>>>(Hp, Hq, Hr, rec, iters, s_eps); }
  int rc = check_launch("mhc_layer_fwd_static/prep");
  if (rc) return rc;
  const bool vec = (C % 4 == 0) && aligned16(x) && aligned16(out) && aligned16(w);
  const int64_t q = (C / 4 + 255) / 256;  // quads per thread
  const unsigned grid = (unsigned)(B < (1 << 30) ? B : (1 << 30));
  if (B == 0) return MHC_OK;
  if (vec && q <= 1) { ProfScope _ps("static_fwd", s); static_fwd_kernel<N, 1, T><<<grid, 256, 0, s>>>(x, w, rec, rms, out, B, C, r_eps); }
  else if (vec && q <= 2) { ProfScope _ps("static_fwd", s); static_fwd_kernel<N, 2, T><<<grid, 256, 0, s>>>(x, w, rec, rms, out, B, C, r_eps); }
  else if (vec && q <= 4) { ProfScope _ps("static_fwd", s); static_fwd_kernel<N, 4, T><<<grid, 256, 0, s>>>(x, w, rec, rms, out, B, C, r_eps); }
  else if (vec && q <= 8 && N <= 4) { ProfScope _ps("static_fwd", s); static_fwd_kernel<N, (N <= 4 ? 8 : 4), T><<<grid, 256, 0, s>>>(x, w, rec, rms, out, B, C, r_eps); }
  else { ProfScope _ps("static_fwd_generic", s); static_fwd_generic_kernel<N, T><<<grid, 256, 0, s>>>(x, w, rec, rms, out, B, C, r_eps); }
  return check_launch("mhc_layer_fwd_static");
}

template <int N>
int run_bwd_static(const float* g, const float* x, const float* w, const float* Hp,
                   const float* Hq, const float* Hr, const float* rms, float* gx, float* gw,
                   float* gHp, float* gHq, float* gHr, int64_t B, int64_t C, int iters,
                   float s_eps, float r_eps, void* ws, size_t ws_bytes, cudaStream_t s) {
  const size_t need = bwd_ws_bytes<N, false>(B, C);
  MHC_REQUIRE(ws != nullptr && ws_bytes >= need, MHC_ERR_WORKSPACE,
              "mhc_layer_bwd_static: workspace of %zu bytes required, got %zu", need, ws_bytes);
  BwdPlan p = plan_bwd<N, false>(B, C);
  Carve cv(ws);
  double* stats = (double*)cv.take(p.stats);
  float* tokb = cv.take(p.tokb);
  double* tokr = (double*)cv.take(p.tokr);
  cv.take(p.dphi);
  float* gwp = cv.take(p.gw);
  double* tot = (double*)cv.take(p.tot);
  float* rec = cv.take(L<N>::REC);
  { ProfScope _ps("static_prep", s); static_prep_kernel<N><<<1, 32, 0, s>>>(Hp, Hq, Hr, rec, iters, s_eps); }
  const bool vec = (C % 4 == 0) && aligned16(x) && aligned16(g) && aligned16(w);
  const unsigned grid = (unsigned)(B < (1 << 30) ? B : (1 << 30));
  if (vec) { ProfScope _ps("bwd_stats", s); bwd_stats_kernel<N, true, true><<<grid, 128, 0, s>>>(g, x, w, stats, B, C); }
  else { ProfScope _ps("bwd_stats", s); bwd_stats_kernel<N, false, true><<<grid, 128, 0, s>>>(g, x, w, stats, B, C); }
  int rc = check_launch("mhc_layer_bwd_static/bwd_stats");
  if (rc) return rc;
  { ProfScope _ps("token_bwd_static", s); token_bwd_static_kernel<N><<<grid_1d(B, kTokThreads), kTokThreads, 0, s>>>(stats, Hp, Hq, rec, tokb, tokr, B, C, r_eps); }
  int nsplit = p.nsplit;
  if (!launch_grad_x_tma<N, false>(g, x, w, nullptr, nullptr, nullptr, tokb, gx, nullptr, gwp, B,
                                   C, p, &nsplit, s))
    { ProfScope _ps("grad_x", s); grad_x_kernel<N, false><<<(unsigned)(p.ntiles * p.nsplit), GX_CW * N, 0, s>>>(
        g, x, w, nullptr, nullptr, nullptr, tokb, gx, nullptr, gwp, B, C, p.ntiles, p.nsplit); }
  rc = check_launch("mhc_layer_bwd_static/grad_x");
  if (rc) return rc;
  { ProfScope _ps("reduce_splits", s); reduce_splits_kernel<<<grid_1d(C, 256, 4096), 256, 0, s>>>(gwp, p.nsplit, C, gw); }
  { ProfScope _ps("reduce_tokens", s); reduce_tokens_kernel<<<L<N>::NRS, 256, 0, s>>>(tokr, B, L<N>::NRS, tot); }
  { ProfScope _ps("static_param_grads", s); static_param_grads_kernel<N><<<1, 32, 0, s>>>(tot, Hr, gHp, gHq, gHr, iters, s_eps); }
  return check_launch("mhc_layer_bwd_static/reduce");
}

int check_layer_args(const char* what, int64_t B, int n, int64_t C, int iters, float s_eps,
                     float r_eps) {
  MHC_REQUIRE(B >= 0, MHC_ERR_INVALID_ARG, "%s: batch must be >= 0", what);
  MHC_REQUIRE(C >= 1, MHC_ERR_INVALID_ARG, "%s: hidden_dim must be >= 1", what);
  MHC_REQUIRE(n >= 1 && n <= 8, MHC_ERR_UNSUPPORTED, "%s: expansion_rate n must be in [1, 8], got %d",
              what, n);
  MHC_REQUIRE(iters >= 0, MHC_ERR_INVALID_ARG, "%s: sinkhorn_iters must be >= 0", what);
  MHC_REQUIRE(s_eps >= 0.f && r_eps >= 0.f, MHC_ERR_INVALID_ARG, "%s: eps must be >= 0", what);
  MHC_REQUIRE((int64_t)n * C < (1LL << 31), MHC_ERR_UNSUPPORTED, "%s: n*C too large", what);
  return MHC_OK;
}

}  // namespace
}  // namespace mhc

using namespace mhc;

#define MHC_DISPATCH_N(n, CALL)          \
  switch (n) {                           \
    case 1: { constexpr int NN = 1; return CALL; } \
    case 2: { constexpr int NN = 2; return CALL; } \
    case 3: { constexpr int NN = 3; return CALL; } \
    case 4: { constexpr int NN = 4; return CALL; } \
    case 5: { constexpr int NN = 5; return CALL; } \
    case 6: { constexpr int NN = 6; return CALL; } \
    case 7: { constexpr int NN = 7; return CALL; } \
    case 8: { constexpr int NN = 8; return CALL; } \
    default: return fail(MHC_ERR_UNSUPPORTED, "expansion_rate %d unsupported", n); \
  }

extern "C" int32_t mhc_token_state_stride(int32_t n) { return rec_stride(n); }

extern "C" size_t mhc_layer_fwd_dynamic_workspace_bytes(int64_t batch, int32_t n,
                                                        int64_t hidden) {
  if (batch <= 0 || hidden <= 0 || n < 1 || n > 8) return 0;
  switch (n) {
    case 1: return fwd_ws_bytes<1>(batch, hidden, true);
    case 2: return fwd_ws_bytes<2>(batch, hidden, true);
    case 3: return fwd_ws_bytes<3>(batch, hidden, true);
    case 4: return fwd_ws_bytes<4>(batch, hidden, true);
    case 5: return fwd_ws_bytes<5>(batch, hidden, true);
    case 6: return fwd_ws_bytes<6>(batch, hidden, true);
    case 7: return fwd_ws_bytes<7>(batch, hidden, true);
    default: return fwd_ws_bytes<8>(batch, hidden, true);
  }
}

template <typename T>
static int fwd_dynamic_entry(const char* what, const T* x, const float* rmsnorm_weight,
                             const float* phi_pre, const float* phi_post, const float* phi_res,
                             const float* alpha_pre, const float* alpha_post,
                             const float* alpha_res, const float* b_pre, const float* b_post,
                             const float* b_res, T* out, float* token_state, int64_t batch,
                             int32_t n, int64_t hidden, int32_t sinkhorn_iters,
                             float sinkhorn_eps, float rmsnorm_eps, void* workspace,
                             size_t workspace_bytes, void* stream) {
  int rc = check_layer_args(what, batch, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps);
  if (rc) return rc;
  MHC_REQUIRE_PTR(x); MHC_REQUIRE_PTR(rmsnorm_weight); MHC_REQUIRE_PTR(phi_pre);
  MHC_REQUIRE_PTR(phi_post); MHC_REQUIRE_PTR(phi_res); MHC_REQUIRE_PTR(alpha_pre);
  MHC_REQUIRE_PTR(alpha_post); MHC_REQUIRE_PTR(alpha_res); MHC_REQUIRE_PTR(b_pre);
  MHC_REQUIRE_PTR(b_post); MHC_REQUIRE_PTR(b_res); MHC_REQUIRE_PTR(out);
  if (batch == 0) return MHC_OK;
  cudaStream_t s = (cudaStream_t)stream;
  MHC_DISPATCH_N(n, (run_fwd_dynamic<NN, T>(x, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
                                            alpha_post, alpha_res, b_pre, b_post, b_res, out,
                                            token_state, batch, hidden, sinkhorn_iters,
                                            sinkhorn_eps, rmsnorm_eps, workspace, workspace_bytes, s)));
}

extern "C" int mhc_layer_fwd_dynamic(const float* x, const float* rmsnorm_weight,
                                     const float* phi_pre, const float* phi_post,
                                     const float* phi_res, const float* alpha_pre,
                                     const float* alpha_post, const float* alpha_res,
                                     const float* b_pre, const float* b_post, const float* b_res,
                                     float* out, float* token_state, int64_t batch, int32_t n,
                                     int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps,
                                     float rmsnorm_eps, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  return fwd_dynamic_entry<float>("mhc_layer_fwd_dynamic", x, rmsnorm_weight, phi_pre, phi_post,
                                  phi_res, alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res,
                                  out, token_state, batch, n, hidden, sinkhorn_iters, sinkhorn_eps,
                                  rmsnorm_eps, workspace, workspace_bytes, stream);
}

extern "C" int mhc_layer_fwd_dynamic_bf16(const void* x, const float* rmsnorm_weight,
                                          const float* phi_pre, const float* phi_post,
                                          const float* phi_res, const float* alpha_pre,
                                          const float* alpha_post, const float* alpha_res,
                                          const float* b_pre, const float* b_post,
                                          const float* b_res, void* out, float* token_state,
                                          int64_t batch, int32_t n, int64_t hidden,
                                          int32_t sinkhorn_iters, float sinkhorn_eps,
                                          float rmsnorm_eps, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  return fwd_dynamic_entry<__nv_bfloat16>(
      "mhc_layer_fwd_dynamic_bf16", (const __nv_bfloat16*)x, rmsnorm_weight, phi_pre, phi_post,
      phi_res, alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res, (__nv_bfloat16*)out,
      token_state, batch, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps, workspace,
      workspace_bytes, stream);
}

extern "C" size_t mhc_layer_bwd_dynamic_workspace_bytes(int64_t batch, int32_t n,
                                                        int64_t hidden) {
  if (batch <= 0 || hidden <= 0 || n < 1 || n > 8) return 0;
  switch (n) {
    case 1: return bwd_ws_bytes<1, true>(batch, hidden);
    case 2: return bwd_ws_bytes<2, true>(batch, hidden);
    case 3: return bwd_ws_bytes<3, true>(batch, hidden);
    case 4: return bwd_ws_bytes<4, true>(batch, hidden);
    case 5: return bwd_ws_bytes<5, true>(batch, hidden);
    case 6: return bwd_ws_bytes<6, true>(batch, hidden);
    case 7: return bwd_ws_bytes<7, true>(batch, hidden);
    default: return bwd_ws_bytes<8, true>(batch, hidden);
  }
}

template <typename T>
static int bwd_dynamic_entry(
    const char* what, const T* grad_out, const T* x, const float* rmsnorm_weight,
    const float* phi_pre, const float* phi_post, const float* phi_res, const float* alpha_pre,
    const float* alpha_post, const float* alpha_res, const float* b_pre, const float* b_post,
    const float* b_res, const float* token_state, T* grad_x, float* grad_rmsnorm_weight,
    float* grad_phi_pre, float* grad_phi_post, float* grad_phi_res, float* grad_alpha_pre,
    float* grad_alpha_post, float* grad_alpha_res, float* grad_b_pre, float* grad_b_post,
    float* grad_b_res, int64_t batch, int32_t n, int64_t hidden, int32_t sinkhorn_iters,
    float sinkhorn_eps, float rmsnorm_eps, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_layer_args(what, batch, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps);
  if (rc) return rc;
  MHC_REQUIRE_PTR(grad_out); MHC_REQUIRE_PTR(x); MHC_REQUIRE_PTR(rmsnorm_weight);
  MHC_REQUIRE_PTR(phi_pre); MHC_REQUIRE_PTR(phi_post); MHC_REQUIRE_PTR(phi_res);
  MHC_REQUIRE_PTR(alpha_pre); MHC_REQUIRE_PTR(alpha_post); MHC_REQUIRE_PTR(alpha_res);
  MHC_REQUIRE_PTR(b_pre); MHC_REQUIRE_PTR(b_post); MHC_REQUIRE_PTR(b_res);
  MHC_REQUIRE_PTR(token_state); MHC_REQUIRE_PTR(grad_x);
  MHC_REQUIRE_PTR(grad_rmsnorm_weight); MHC_REQUIRE_PTR(grad_phi_pre);
  MHC_REQUIRE_PTR(grad_phi_post); MHC_REQUIRE_PTR(grad_phi_res); MHC_REQUIRE_PTR(grad_alpha_pre);
  MHC_REQUIRE_PTR(grad_alpha_post); MHC_REQUIRE_PTR(grad_alpha_res);
  MHC_REQUIRE_PTR(grad_b_pre); MHC_REQUIRE_PTR(grad_b_post); MHC_REQUIRE_PTR(grad_b_res);
  MHC_REQUIRE(batch > 0, MHC_ERR_INVALID_ARG, "%s: batch must be > 0", what);
  cudaStream_t s = (cudaStream_t)stream;
  MHC_DISPATCH_N(n, (run_bwd_dynamic<NN, T>(grad_out, x, rmsnorm_weight, phi_pre, phi_post, phi_res,
                                            alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res,
                                            token_state, grad_x, grad_rmsnorm_weight, grad_phi_pre,
                                            grad_phi_post, grad_phi_res, grad_alpha_pre,
                                            grad_alpha_post, grad_alpha_res, grad_b_pre, grad_b_post,
                                            grad_b_res, batch, hidden, sinkhorn_iters, sinkhorn_eps,
                                            rmsnorm_eps, workspace, workspace_bytes, s)));
}

extern "C" int mhc_layer_bwd_dynamic(
    const float* grad_out, const float* x, const float* rmsnorm_weight, const float* phi_pre,
    const float* phi_post, const float* phi_res, const float* alpha_pre, const float* alpha_post,
    const float* alpha_res, const float* b_pre, const float* b_post, const float* b_res,
    const float* token_state, float* grad_x, float* grad_rmsnorm_weight, float* grad_phi_pre,
    float* grad_phi_post, float* grad_phi_res, float* grad_alpha_pre, float* grad_alpha_post,
    float* grad_alpha_res, float* grad_b_pre, float* grad_b_post, float* grad_b_res,
    int64_t batch, int32_t n, int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps,
    float rmsnorm_eps, void* workspace, size_t workspace_bytes, void* stream) {
  return bwd_dynamic_entry<float>(
      "mhc_layer_bwd_dynamic", grad_out, x, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
      alpha_post, alpha_res, b_pre, b_post, b_res, token_state, grad_x, grad_rmsnorm_weight,
      grad_phi_pre, grad_phi_post, grad_phi_res, grad_alpha_pre, grad_alpha_post, grad_alpha_res,
      grad_b_pre, grad_b_post, grad_b_res, batch, n, hidden, sinkhorn_iters, sinkhorn_eps,
      rmsnorm_eps, workspace, workspace_bytes, stream);
}

extern "C" int mhc_layer_bwd_dynamic_bf16(
    const void* grad_out, const void* x, const float* rmsnorm_weight, const float* phi_pre,
    const float* phi_post, const float* phi_res, const float* alpha_pre, const float* alpha_post,
    const float* alpha_res, const float* b_pre, const float* b_post, const float* b_res,
    const float* token_state, void* grad_x, float* grad_rmsnorm_weight, float* grad_phi_pre,
    float* grad_phi_post, float* grad_phi_res, float* grad_alpha_pre, float* grad_alpha_post,
    float* grad_alpha_res, float* grad_b_pre, float* grad_b_post, float* grad_b_res,
    int64_t batch, int32_t n, int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps,
    float rmsnorm_eps, void* workspace, size_t workspace_bytes, void* stream) {
  return bwd_dynamic_entry<__nv_bfloat16>(
      "mhc_layer_bwd_dynamic_bf16", (const __nv_bfloat16*)grad_out, (const __nv_bfloat16*)x,
      rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre, alpha_post, alpha_res, b_pre, b_post,
      b_res, token_state, (__nv_bfloat16*)grad_x, grad_rmsnorm_weight, grad_phi_pre, grad_phi_post,
      grad_phi_res, grad_alpha_pre, grad_alpha_post, grad_alpha_res, grad_b_pre, grad_b_post,
      grad_b_res, batch, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps, workspace,
      workspace_bytes, stream);
}

extern "C" size_t mhc_layer_static_workspace_bytes(int64_t batch, int32_t n, int64_t hidden) {
  if (hidden <= 0 || n < 1 || n > 8) return 0;
  if (batch < 1) batch = 1;
  switch (n) {
    case 1: return bwd_ws_bytes<1, false>(batch, hidden);
    case 2: return bwd_ws_bytes<2, false>(batch, hidden);
    case 3: return bwd_ws_bytes<3, false>(batch, hidden);
    case 4: return bwd_ws_bytes<4, false>(batch, hidden);
    case 5: return bwd_ws_bytes<5, false>(batch, hidden);
    case 6: return bwd_ws_bytes<6, false>(batch, hidden);
    case 7: return bwd_ws_bytes<7, false>(batch, hidden);
    default: return bwd_ws_bytes<8, false>(batch, hidden);
  }
}

template <typename T>
static int fwd_static_entry(const T* x, const float* w, const float* Hp, const float* Hq,
                            const float* Hr, T* out, float* rms, int64_t batch, int32_t n,
                            int64_t hidden, int32_t iters, float s_eps, float r_eps, void* ws,
                            size_t ws_bytes, void* stream) {
  int rc = check_layer_args("mhc_layer_fwd_static", batch, n, hidden, iters, s_eps, r_eps);
  if (rc) return rc;
  MHC_REQUIRE_PTR(x); MHC_REQUIRE_PTR(w); MHC_REQUIRE_PTR(Hp); MHC_REQUIRE_PTR(Hq);
  MHC_REQUIRE_PTR(Hr); MHC_REQUIRE_PTR(out);
  cudaStream_t s = (cudaStream_t)stream;
  MHC_DISPATCH_N(n, (run_fwd_static<NN, T>(x, w, Hp, Hq, Hr, out, rms, batch, hidden, iters,
                                           s_eps, r_eps, ws, ws_bytes, s)));
}

extern "C" int mhc_layer_fwd_static_f32(const float* x, const float* rmsnorm_weight,
                                        const float* H_pre, const float* H_post,
                                        const float* H_res, float* out, float* rms,
                                        int64_t batch, int32_t n, int64_t hidden,
                                        int32_t sinkhorn_iters, float sinkhorn_eps,
                                        float rmsnorm_eps, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  return fwd_static_entry<float>(x, rmsnorm_weight, H_pre, H_post, H_res, out, rms, batch, n,
                                 hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps, workspace,
                                 workspace_bytes, stream);
}

extern "C" int mhc_layer_fwd_static_bf16(const void* x, const float* rmsnorm_weight,
                                         const float* H_pre, const float* H_post,
                                         const float* H_res, void* out, float* rms,
                                         int64_t batch, int32_t n, int64_t hidden,
                                         int32_t sinkhorn_iters, float sinkhorn_eps,
                                         float rmsnorm_eps, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  return fwd_static_entry<__nv_bfloat16>((const __nv_bfloat16*)x, rmsnorm_weight, H_pre, H_post,
                                         H_res, (__nv_bfloat16*)out, rms, batch, n, hidden,
                                         sinkhorn_iters, sinkhorn_eps, rmsnorm_eps, workspace,
                                         workspace_bytes, stream);
}

extern "C" int mhc_layer_bwd_static(const float* grad_out, const float* x,
                                    const float* rmsnorm_weight, const float* H_pre,
                                    const float* H_post, const float* H_res, const float* rms,
                                    float* grad_x, float* grad_rmsnorm_weight, float* grad_H_pre,
                                    float* grad_H_post, float* grad_H_res, int64_t batch,
                                    int32_t n, int64_t hidden, int32_t sinkhorn_iters,
                                    float sinkhorn_eps, float rmsnorm_eps, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  int rc = check_layer_args("mhc_layer_bwd_static", batch, n, hidden, sinkhorn_iters,
                            sinkhorn_eps, rmsnorm_eps);
  if (rc) return rc;
  MHC_REQUIRE_PTR(grad_out); MHC_REQUIRE_PTR(x); MHC_REQUIRE_PTR(rmsnorm_weight);
  MHC_REQUIRE_PTR(H_pre); MHC_REQUIRE_PTR(H_post); MHC_REQUIRE_PTR(H_res); MHC_REQUIRE_PTR(rms);
  MHC_REQUIRE_PTR(grad_x); MHC_REQUIRE_PTR(grad_rmsnorm_weight); MHC_REQUIRE_PTR(grad_H_pre);
  MHC_REQUIRE_PTR(grad_H_post); MHC_REQUIRE_PTR(grad_H_res);
  MHC_REQUIRE(batch > 0, MHC_ERR_INVALID_ARG, "mhc_layer_bwd_static: batch must be > 0");
  cudaStream_t s = (cudaStream_t)stream;
  MHC_DISPATCH_N(n, (run_bwd_static<NN>(grad_out, x, rmsnorm_weight, H_pre, H_post, H_res, rms,
                                        grad_x, grad_rmsnorm_weight, grad_H_pre, grad_H_post,
                                        grad_H_res, batch, hidden, sinkhorn_iters, sinkhorn_eps,
                                        rmsnorm_eps, workspace, workspace_bytes, s)));
}

extern "C" int mhc_device_error_word(int32_t* value, int32_t reset) {
  MHC_REQUIRE_PTR(value);
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_mhc_device_error, sizeof(int));
  if (e != cudaSuccess)
    return fail(MHC_ERR_CUDA, "mhc_device_error_word: %s", cudaGetErrorString(e));
  *value = v;
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_mhc_device_error, &zero, sizeof(int));
    if (e != cudaSuccess)
      return fail(MHC_ERR_CUDA, "mhc_device_error_word: %s", cudaGetErrorString(e));
  }
  return MHC_OK;
}
