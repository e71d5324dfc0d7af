// Layout constants and device helpers shared by the fused layer kernels.
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

// Per-stream scales of MHCResidualWrapper's packing (reference layer.py:
// 299-310): stream i is s[i] * residual, stream 1 the branch output (s[1] = 1:
// kernels that scale every stream leave the branch as is); "decay" 1, 1, 0.1,
// 0.01, "zero" 1, 1, 0, 0.
struct WrapScales {
  float s[4];
};

__host__ __device__ inline int rec_stride(int n) {
  const int raw = 2 + 2 * n + n * n + (n * n + 2 * n);
  if (n > 8) return (raw + 3) / 4 * 4;  // wide rates keep no Gram block
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
  // D2 (the dphi contraction over tokens) alternates between two accumulators
  // every DR2 blocks; the epilogue warps add each finished one into fp32 sums
  // in shared memory LAG2 blocks later, so no tensor-memory accumulation chain
  // spans more than DR2 blocks (12 MMAs each).  Tensor-memory accumulation
  // rounds toward zero -- a uniform relative shrink of ~2e-8 per MMA, which
  // over the 1024 blocks of a 32768-token split reached 5e-3 on dphi
  static constexpr int DR2 = 8, LAG2 = 4;
  // local-term / grad_x tile buffers: three, so the E warps fill block j + 2
  // while block j's store drains and block j + 1's epilogue runs
  static constexpr int NL = 3;
  static constexpr int NBAR = 2 * SG + 2 * SI + 4 * ND + 2 * NL + 2 + 4;
  // tensor memory: D1[b] [TOK b, +TOK); D2 [64, 96) and [160, 192); Phi^T hi
  // [96, 120), lo [128, 152); X^T[b] [256 + 2 TOK b, +2 TOK) hi|lo
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t D2_COL = 64, D2B_COL = 160, A1_COL = 96, A1L_COL = 128, XT_COL = 256;
  static_assert(LAG2 >= 1 && LAG2 <= DR2, "drain schedule");
  static_assert(ND * TOK <= 64 && XT_COL + 2 * TOK * ND <= TMEM_COLS && TOK % 16 == 0, "tensor-memory plan");
};

// Shared-memory plan of grad_x6 for stream element type T (fp32 or bf16 I/O).
// WRAP (MHCResidualWrapper, fp32): a stage holds the block's mean gradient,
// residual and branch rows ([TOK][CW] each) instead of g and x of the four
// streams, and the epilogue stages the residual / branch gradient tiles.
template <typename T, bool WRAP = false>
struct Gx6S {
  using F = Gx6Cfg;
  static constexpr bool BF16 = sizeof(T) == 2;
  static constexpr uint32_t GB = WRAP ? F::TOK * F::CW * 4                 // one [TOK][CW] row tile
                                      : F::TOK * 4 * F::CW * sizeof(T);    // g (or x) tile bytes
  static constexpr uint32_t STAGE = (WRAP ? 3 : 2) * GB;          // g, x  /  gmean, residual, branch
  static constexpr uint32_t OFF_IMG = F::SG * STAGE;               // g/x ring, then the image ring
  static constexpr uint32_t OFF_LOC = OFF_IMG + F::SI * F::IMG;    // [NL buffers]
  static constexpr uint32_t STGB = BF16 ? F::TOK * F::COLS * 2     // bf16 grad_x staging tile
                                        : (WRAP ? 2 * F::TOK * F::CW * 4 : 0);  // residual | branch gradient tiles
  static constexpr uint32_t OFF_STG = OFF_LOC + F::NL * F::LOCB;   // [NL buffers]
  static constexpr uint32_t OFF_GW = OFF_STG + F::NL * STGB;       // grad-w partials [E warps][32]
  static constexpr uint32_t OFF_D2S = OFF_GW + F::E_WARPS * F::CW * 4;  // drained D2 sums [NH][128]
  static constexpr uint32_t OFF_BAR = OFF_D2S + F::NH * F::COLS * 4;
  static constexpr size_t SMEM = OFF_BAR + F::NBAR * 8 + 16 + 128;
  static_assert(SMEM <= 227 * 1024, "shared-memory plan");
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

}  // namespace
}  // namespace mhc
