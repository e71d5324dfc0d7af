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
//             (sum(xf^2) = trace G, sum_c x_agg^2 = h^T G h); the streaming
//             pass also accumulates G exactly in fp64 for the backward;
//   backward: gM = g x^T and W = g diag(w) x^T; with the forward's G every
//             per-token scalar of the backward follows in closed form (see
//             token_bwd_lanes_kernel).
// So the forward reads x twice and writes out once; the backward reads g and
// x twice and writes grad_x once; parameter gradients are fixed-order
// reductions (no atomics: bitwise reproducible).
//
// Kernels (launch order; fallbacks for other shapes / layouts in brackets):
//   fwd : phi_split -> proj_umma (tcgen05) [proj_stats_tma, proj_stats]
//         -> token_fwd (gates, Sinkhorn, r) -> stream_fwd (out, fp64 Gram)
//   bwd : bwd_stats (gM, W) -> token_bwd (Sinkhorn reverse, d_p, operand
//         image) -> grad_x6 (tcgen05) [grad_x4, grad_x_tma, grad_x]
//         -> finish (fixed-order sums over splits / tokens)
// Files: layer/common.cuh (layout), layer/fwd.cuh, layer/bwd_token.cuh,
// layer/grad_x_legacy.cuh, layer/tcgen05.cuh, layer/reduce.cuh (kernels);
// this file: workspace planning, launchers and the C-ABI entry points.

#include "common.cuh"
#include "sinkhorn.cuh"
#include "sinkhorn_lanes.cuh"
#include "tma.cuh"
#include <cuda_bf16.h>
#include <type_traits>

#include "layer/common.cuh"
#include "layer/fwd.cuh"
#include "layer/bwd_token.cuh"
#include "layer/grad_x_legacy.cuh"
#include "layer/tcgen05.cuh"
#include "layer/reduce.cuh"
#include "layer/wide.cuh"

namespace mhc {
namespace {

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

// Token splits of the tensor-core grad_x (grad_x6_kernel, one CTA per SM):
// minimise waves x (blocks per CTA x t_block + t_ramp), with t_block the
// steady time of a 32-token block and t_ramp a CTA's start-up and drain,
// fitted from measured launches over split counts 1..8 on a B200 at
// n = 4, C = 4096 (fp32 streams 1.24 / 8.7 us, bf16 1.54 / 4.9 us).  Pure
// wave balance ignores the ramp: at 8192 fp32 tokens it picked 8 splits
// (0.339 ms) where one split takes 0.327 ms.
int choose_gx6_splits(int64_t tiles, int64_t nblk, int sms, double t_block, double t_ramp) {
  int best = 1;
  double best_cost = 1e300;
  const int64_t max_s = nblk < 1024 ? nblk : 1024;
  for (int64_t s = 1; s <= max_s; ++s) {
    const int64_t waves = (tiles * s + sms - 1) / sms;
    const double cost = (double)waves * ((double)((nblk + s - 1) / s) * t_block + t_ramp);
    if (cost < best_cost - 1e-9) { best_cost = cost; best = (int)s; }
  }
  return best;
}

struct BwdPlan {
  int ntiles, nsplit;
  int64_t nblk6;  // token blocks of the warp-specialised grad_x (n = 4, dynamic H)
  int nsplit6, nsplit6b;  // fp32 streams, bf16 streams
  size_t img;
  size_t stats, tokb, tokr, dphi, gw, tot;
};

template <int N, bool DYN>
BwdPlan plan_bwd(int64_t B, int64_t C) {
  BwdPlan p;
  p.ntiles = (int)((C + GX_CW - 1) / GX_CW);
  p.nsplit = choose_gx_splits(p.ntiles, B, num_sms(), N <= 4 ? 2 : 1);
  p.nblk6 = (N == 4 && DYN) ? (B + Gx6Cfg::TOK - 1) / Gx6Cfg::TOK : 0;
  const bool six = N == 4 && DYN && p.nblk6 > 0;
  p.nsplit6 = six ? choose_gx6_splits((C + 31) / 32, p.nblk6, num_sms(), 1.24, 8.7) : 0;
  p.nsplit6b = six ? choose_gx6_splits((C + 31) / 32, p.nblk6, num_sms(), 1.54, 4.9) : 0;
  p.img = (size_t)p.nblk6 * Gx6Cfg::IMG_FLOATS;
  int64_t msplit = p.nsplit;
  if (p.nsplit6 > msplit) msplit = p.nsplit6;
  if (p.nsplit6b > msplit) msplit = p.nsplit6b;
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

// Shared-memory staged forward 3 (token_stream_fwd_kernel): launched when a
// ring of at least two token buffers fits in shared memory and the rows are
// 16-byte aligned; returns false otherwise (the caller uses another kernel).
template <int N, typename T, bool DYN, bool GRAM>
bool launch_token_stream(const T* x, const float* w, float* rec, float* rms, T* out, int64_t B,
                         int64_t C, float r_eps, cudaStream_t s) {
  if (B <= 0 || (C * (int64_t)sizeof(T)) % 16 != 0 || !aligned16(x) || !aligned16(out) ||
      !aligned16(w))
    return false;
  const size_t tok = ((size_t)N * C * sizeof(T) + (DYN ? L<N>::REC * 4 : 0) + 127) & ~(size_t)127;
  // dynamic shared memory left next to the kernel's static arrays (227 KB opt-in)
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, token_stream_fwd_kernel<N, T, DYN, GRAM>) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  const size_t avail = (size_t)227 * 1024 - fa.sharedSizeBytes;
  int nbuf = (int)((avail - 4 * 8) / tok);
  if (nbuf > 4) nbuf = 4;
  if (nbuf < 2) return false;
  const size_t smem = (size_t)nbuf * tok + (size_t)nbuf * 8;
  cudaFuncSetAttribute(token_stream_fwd_kernel<N, T, DYN, GRAM>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t g = B < num_sms() ? B : num_sms();
  token_stream_fwd_kernel<N, T, DYN, GRAM><<<(unsigned)g, kTsThreads, smem, s>>>(
      x, w, rec, rms, out, B, C, r_eps, nbuf);
  return true;
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
  bool sumsq = false;  // the tensor-core projection: sum of squares only, r in stream_fwd_r
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
    // channels per split: a multiple of the x stage width
    constexpr int SW = PU::CH * PU::XW;
    const int ucps = (p.ucps + SW - 1) / SW * SW;
    const int uks = p.ucps > 0 ? (int)((C + ucps - 1) / ucps) : 0;
    if (p.uks > 0 && B > 0 && C % PU::CH == 0 && aligned16(x) && aligned16(ph) && aligned16(pl) &&
        aligned16(out) && aligned16(w) &&
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
          xmap, hmap, lmap, xmap, WrapScales{}, ppart, gpart, B, C, ucps); }
      ks = uks;
      done = true;
      sumsq = true;
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
  {
    constexpr int TG = N <= 2 ? 2 : (N <= 4 ? 4 : 8);
    ProfScope _ps("token_fwd", s);
    if (B > 0 && sumsq && N <= 4)
      token_fwd_lanes_kernel<N, N <= 4><<<grid_1d(B * TG, 128), 128, 0, s>>>(
          ppart, gpart, ks, ap, aq, ar, bp, bq, br, rec, B, C, iters, s_eps, r_eps);
    else if (B > 0)
      token_fwd_lanes_kernel<N, false><<<grid_1d(B * TG, 128), 128, 0, s>>>(
          ppart, gpart, ks, ap, aq, ar, bp, bq, br, rec, B, C, iters, s_eps, r_eps);
  }
  rc = check_launch("mhc_layer_fwd_dynamic/token_fwd");
  if (rc) return rc;
  if constexpr (N <= 4) if (sumsq) {
    // r and out from the token, register-resident when it fits
    const unsigned grid = (unsigned)(B < (1 << 30) ? B : (1 << 30));
    const int64_t quads = C / 4;
    ProfScope _ps("stream_fwd", s);
    auto go = [&](auto gram) {
      constexpr bool G = decltype(gram)::value;
      // tokens that fit two CTAs' registers per SM stream best from registers;
      // larger ones from the shared-memory ring
      if (quads > 1024 && launch_token_stream<N, T, true, G>(x, w, rec, nullptr, out, B, C, r_eps, s))
        return;
      if (quads <= 256)
        stream_fwd_r_kernel<N, 1, G, T><<<grid, 256, 0, s>>>(x, w, rec, out, B, C, r_eps);
      else if (quads <= 512)
        stream_fwd_r_kernel<N, 2, G, T><<<grid, 256, 0, s>>>(x, w, rec, out, B, C, r_eps);
      else if (quads <= 1024)
        stream_fwd_r_kernel<N, 4, G, T><<<grid, 256, 0, s>>>(x, w, rec, out, B, C, r_eps);
      else if (quads <= 2048)
        stream_fwd_r_kernel<N, 4, G, T, 512><<<grid, 512, 0, s>>>(x, w, rec, out, B, C, r_eps);
      else
        stream_fwd_r_kernel<N, 0, G, T><<<grid, 256, 0, s>>>(x, w, rec, out, B, C, r_eps);
    };
    // the fp64 Gram matrix is only needed when the record is kept for a backward
    if (need_rec) go(std::false_type{});
    else go(std::true_type{});
    return check_launch("mhc_layer_fwd_dynamic/stream_fwd");
  }
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
      const int ns6 = sizeof(T) == 2 ? p.nsplit6b : p.nsplit6;
      { ProfScope _ps("grad_x", s); grad_x6_kernel<T><<<(unsigned)(nt6 * ns6), F6::THREADS, S6::SMEM, s>>>(
          gm, xm, om, xm, om, WrapScales{}, img, w, pp, pq, pr, gx, dphi, gwp, B, C, nt6, ns6, p.nblk6); }
      nsplit = ns6;
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

// ---------------------------------------------------------------------------
// MHCResidualWrapper with the streams built inside the kernels (n = 4, fp32):
// the [T, n, C] packed input, the layer output and their gradients never
// reach HBM.  Same split plans and workspaces as the bare layer.
// ---------------------------------------------------------------------------
int run_fwd_wrap(const float* res, const float* br, WrapScales sc, const float* w, const float* pp,
                 const float* pq, const float* pr, const float* ap, const float* aq,
                 const float* ar, const float* bp, const float* bq, const float* brs,
                 float* mean, float* token_state, int64_t B, int64_t C, int iters, float s_eps,
                 float r_eps, void* ws, size_t ws_bytes, cudaStream_t s, PreNorm pn = PreNorm{}) {
  constexpr int N = 4;
  using PU = PumCfg<N, float>;
  const bool need_rec = token_state == nullptr;
  const size_t need = fwd_ws_bytes<N>(B, C, need_rec);
  MHC_REQUIRE(ws != nullptr && ws_bytes >= need, MHC_ERR_WORKSPACE,
              "mhc_wrapper_fwd_dynamic: workspace of %zu bytes required, got %zu", need, ws_bytes);
  MHC_REQUIRE(C % Gx6Cfg::CW == 0 && aligned16(res) && aligned16(br) && aligned16(mean) &&
                  aligned16(w),
              MHC_ERR_UNSUPPORTED,
              "mhc_wrapper_fwd_dynamic: needs hidden %% 32 == 0 and 16-byte aligned tensors");
  FwdPlan p = plan_fwd<N>(B, C);
  Carve cv(ws);
  float* ppart = cv.take(p.ppart);
  float* gpart = cv.take(p.gpart);
  float* phiT = cv.take(p.phiT);
  float* rec = need_rec ? cv.take(p.rec_tmp) : token_state;
  const int64_t nC = (int64_t)N * C;
  float* ph = phiT;
  float* pl = phiT + (size_t)PU::NB * nC;
  constexpr int SW = PU::CH * PU::XW;
  const int ucps = (p.ucps + SW - 1) / SW * SW;
  const int uks = (int)((C + ucps - 1) / ucps);
  CUtensorMap rmap, bmap, hmap, lmap;
  const uint64_t cs = (uint64_t)C * 4, rs = (uint64_t)nC * 4;
  MHC_REQUIRE(p.uks > 0 && aligned16(ph) && aligned16(pl) &&
                  make_tmap_2d(&rmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, res, B, C, C, PU::TOK,
                               PU::CH, CU_TENSOR_MAP_SWIZZLE_128B) &&
                  make_tmap_2d(&bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, br, B, C, C, PU::TOK,
                               PU::CH, CU_TENSOR_MAP_SWIZZLE_128B) &&
                  make_tmap_3d_f32(&hmap, ph, C, N, PU::NB, cs, rs, 32, 1, PU::NB, CU_TENSOR_MAP_SWIZZLE_128B) &&
                  make_tmap_3d_f32(&lmap, pl, C, N, PU::NB, cs, rs, 32, 1, PU::NB, CU_TENSOR_MAP_SWIZZLE_128B),
              MHC_ERR_UNSUPPORTED, "mhc_wrapper_fwd_dynamic: tensor map creation failed");
  {
    const bool pvec = nC % 4 == 0 && aligned16(pp) && aligned16(pq) && aligned16(pr);
    ProfScope _ps("phi_split", s);
    phi_split_kernel<N><<<dim3(grid_1d(pvec ? nC / 4 : nC, 256, 64), PU::NB), 256, 0, s>>>(pp, pq, pr, ph, pl, C, pvec);
  }
  cudaFuncSetAttribute(proj_umma_kernel<N, float, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PU::SMEM);
  { ProfScope _ps("proj_stats", s); proj_umma_kernel<N, float, true><<<dim3((unsigned)p.utiles, (unsigned)uks), PU::THREADS, PU::SMEM, s>>>(
      rmap, hmap, lmap, bmap, sc, ppart, gpart, B, C, ucps); }
  int rc = check_launch("mhc_wrapper_fwd_dynamic/proj_stats");
  if (rc) return rc;
  { ProfScope _ps("token_fwd", s); token_fwd_lanes_kernel<N, true><<<grid_1d(B * 4, 128), 128, 0, s>>>(
      ppart, gpart, uks, ap, aq, ar, bp, bq, brs, rec, B, C, iters, s_eps, r_eps); }
  rc = check_launch("mhc_wrapper_fwd_dynamic/token_fwd");
  if (rc) return rc;
  const unsigned grid = (unsigned)(B < (1 << 30) ? B : (1 << 30));
  const int64_t quads = C / 4;
  ProfScope _ps("stream_fwd", s);
  auto go = [&](auto gram, auto pre) {
    constexpr bool G = decltype(gram)::value, P = decltype(pre)::value;
    if (quads <= 256) wrap_fwd_r_kernel<N, 1, G, 256, P><<<grid, 256, 0, s>>>(res, br, sc, w, rec, mean, B, C, r_eps, pn);
    else if (quads <= 512) wrap_fwd_r_kernel<N, 2, G, 256, P><<<grid, 256, 0, s>>>(res, br, sc, w, rec, mean, B, C, r_eps, pn);
    else if (quads <= 1024) wrap_fwd_r_kernel<N, 4, G, 256, P><<<grid, 256, 0, s>>>(res, br, sc, w, rec, mean, B, C, r_eps, pn);
    else if (quads <= 2048) wrap_fwd_r_kernel<N, 4, G, 512, P><<<grid, 512, 0, s>>>(res, br, sc, w, rec, mean, B, C, r_eps, pn);
    else wrap_fwd_r_kernel<N, 0, G, 256, P><<<grid, 256, 0, s>>>(res, br, sc, w, rec, mean, B, C, r_eps, pn);
  };
  const bool pre = pn.normed != nullptr;
  if (need_rec && pre) go(std::false_type{}, std::true_type{});
  else if (need_rec) go(std::false_type{}, std::false_type{});
  else if (pre) go(std::true_type{}, std::true_type{});
  else go(std::true_type{}, std::false_type{});
  return check_launch("mhc_wrapper_fwd_dynamic/stream_fwd");
}

int run_bwd_wrap(const float* gmean, const float* res, const float* br, WrapScales sc,
                 const float* w, const float* pp, const float* pq, const float* pr,
                 const float* ap, const float* aq, const float* ar, const float* bp,
                 const float* bq, const float* brs, const float* rec, float* gres, float* gbr,
                 float* gw, float* gpp, float* gpq, float* gpr, float* gap, float* gaq,
                 float* gar, float* gbp, float* gbq, float* gbr_b, int64_t B, int64_t C,
                 int iters, float s_eps, float r_eps, void* ws, size_t ws_bytes, cudaStream_t s) {
  constexpr int N = 4;
  const size_t need = bwd_ws_bytes<N, true>(B, C);
  MHC_REQUIRE(ws != nullptr && ws_bytes >= need, MHC_ERR_WORKSPACE,
              "mhc_wrapper_bwd_dynamic: workspace of %zu bytes required, got %zu", need, ws_bytes);
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
  using F6 = Gx6Cfg;
  using S6 = Gx6S<float, true>;
  MHC_REQUIRE(p.nsplit6 > 0 && C % F6::CW == 0 && aligned16(gmean) && aligned16(res) &&
                  aligned16(br) && aligned16(gres) && aligned16(gbr) && aligned16(w) &&
                  aligned16(img),
              MHC_ERR_UNSUPPORTED,
              "mhc_wrapper_bwd_dynamic: needs hidden %% 32 == 0 and 16-byte aligned tensors");
  CUtensorMap gm, rm, bm, om, om2;
  constexpr CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  MHC_REQUIRE(make_tmap_2d(&gm, dt, 4, gmean, B, C, C, F6::TOK, F6::CW) &&
                  make_tmap_2d(&rm, dt, 4, res, B, C, C, F6::TOK, F6::CW) &&
                  make_tmap_2d(&bm, dt, 4, br, B, C, C, F6::TOK, F6::CW) &&
                  make_tmap_2d(&om, dt, 4, gres, B, C, C, F6::TOK, F6::CW) &&
                  make_tmap_2d(&om2, dt, 4, gbr, B, C, C, F6::TOK, F6::CW),
              MHC_ERR_UNSUPPORTED, "mhc_wrapper_bwd_dynamic: tensor map creation failed");
  const unsigned grid = (unsigned)(B < (1 << 30) ? B : (1 << 30));
  { ProfScope _ps("bwd_stats", s); wrap_bwd_stats_kernel<N><<<grid, 128, 0, s>>>(gmean, res, br, sc, w, stats, B, C); }
  int rc = check_launch("mhc_wrapper_bwd_dynamic/bwd_stats");
  if (rc) return rc;
  const int64_t img_tokens = p.nblk6 * F6::TOK;
  const int64_t tb_tokens = B > img_tokens ? B : img_tokens;
  { ProfScope _ps("token_bwd", s); token_bwd_lanes_kernel<N><<<grid_1d(tb_tokens * 4, 128), 128, 0, s>>>(
      stats, rec, ap, aq, ar, bp, bq, brs, tokb, tokr, B, C, iters, s_eps, r_eps, counter, img,
      img_tokens); }
  rc = check_launch("mhc_wrapper_bwd_dynamic/token_bwd");
  if (rc) return rc;
  cudaFuncSetAttribute(grad_x6_kernel<float, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S6::SMEM);
  const int nt6 = (int)(C / F6::CW);
  { ProfScope _ps("grad_x", s); grad_x6_kernel<float, true><<<(unsigned)(nt6 * p.nsplit6), F6::THREADS, S6::SMEM, s>>>(
      gm, rm, om, bm, om2, sc, img, w, pp, pq, pr, gres, dphi, gwp, B, C, nt6, p.nsplit6, p.nblk6); }
  rc = check_launch("mhc_wrapper_bwd_dynamic/grad_x");
  if (rc) return rc;
  const int64_t nC = (int64_t)N * C;
  const int nb_dphi = (int)grid_1d((int64_t)L<N>::NH * nC, 256, 4 * (int64_t)num_sms());
  const int nb_gw = (int)grid_1d(C, 256, 64);
  const int nb_tok = (int)(B / 128 < 1 ? 1 : (B / 128 < kTokPartBlocks ? B / 128 : kTokPartBlocks));
  { ProfScope _ps("finish", s);
    finish_dyn_bwd_kernel<N><<<(unsigned)(nb_dphi + nb_gw + nb_tok), 256, 0, s>>>(
        dphi, gwp, p.nsplit6, C, gpp, gpq, gpr, gw, tokr, B, tot, counter, nb_dphi, nb_gw, nb_tok,
        gbp, gbq, gbr_b, gap, gaq, gar); }
  return check_launch("mhc_wrapper_bwd_dynamic/reduce");
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
  {
    bool staged;
    {
      ProfScope _ps("static_fwd", s);
      staged = launch_token_stream<N, T, false, false>(x, w, rec, rms, out, B, C, r_eps, s);
    }
    if (staged) return check_launch("mhc_layer_fwd_static");
  }
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

// ---------------------------------------------------------------------------
// Wide expansion rates (8 < n <= 32): kernels in layer/wide.cuh
// ---------------------------------------------------------------------------
constexpr size_t kWidePartCap = size_t(256) << 20;  // split-K partials, bytes per GEMM
constexpr int kColsumChunks = 64;                   // row chunks of the column sums

struct WideSplit {
  int S;
  int64_t kchunk;
};

// Split K for the tcgen05 GEMM (one CTA per SM): waves times the k each CTA
// runs (~16 ns per k: 12 MMAs per 32-k stage, issue-bound), plus the split
// partials at HBM speed; K ranges are whole 32-k stages.
WideSplit wide_split_umma(int64_t M, int64_t N, int64_t K) {
  const int64_t tiles = ((M + WuCfg::BM - 1) / WuCfg::BM) * ((N + WuCfg::BN - 1) / WuCfg::BN);
  const int64_t slots = num_sms();
  int best = 1;
  double best_ns = -1.0;
  for (int S = 1; S <= 64; ++S) {
    if (S > 1 && (K / S < 2 * WuCfg::BK || (size_t)S * M * N * sizeof(float) > kWidePartCap)) break;
    const int64_t kc = ((K + S - 1) / S + WuCfg::BK - 1) / WuCfg::BK * WuCfg::BK;
    const int64_t waves = (tiles * S + slots - 1) / slots;
    const double ns = (double)waves * ((double)kc * 16.0 + 2000.0) +
                      (S > 1 ? 2.0 * S * (double)M * N * sizeof(float) / 6500.0 : 0.0);
    if (best_ns < 0 || ns < best_ns * 0.98) { best_ns = ns; best = S; }
  }
  int64_t kchunk = ((K + best - 1) / best + WuCfg::BK - 1) / WuCfg::BK * WuCfg::BK;
  if (kchunk < WuCfg::BK) kchunk = WuCfg::BK;
  int S = (int)((K + kchunk - 1) / kchunk);
  if (S < 1) S = 1;
  return WideSplit{S, kchunk};
}

size_t wide_fwd_ws_bytes(int64_t B, int n, int64_t C, bool need_rec) {
  const int64_t NH = (int64_t)n * n + 2 * n;
  const WideSplit sp = wide_split_umma(B, NH, (int64_t)n * C);
  Carve cv(nullptr);
  if (need_rec) cv.take((size_t)B * rec_stride(n));
  cv.take((size_t)sp.S * B * NH);
  cv.take((size_t)B * n * n);
  cv.take((size_t)B * n * n);
  return cv.off;
}

size_t wide_bwd_ws_bytes(int64_t B, int n, int64_t C) {
  const int64_t NH = (int64_t)n * n + 2 * n, nC = (int64_t)n * C;
  const WideSplit s1 = wide_split_umma(B, nC, NH), s2 = wide_split_umma(NH, nC, B);
  Carve cv(nullptr);
  for (int q = 0; q < 3; ++q) cv.take((size_t)B * n * n);  // E, gE, gM
  cv.take((size_t)B * 2 * n);                                // gh | ghp
  cv.take((size_t)B * NH);                                   // d_p
  cv.take((size_t)B * (NH + 3));                             // bias / alpha rows
  cv.take((size_t)B);                                        // rms_h coefficient
  cv.take((size_t)B * C);                                    // weight-gradient rows
  cv.take((size_t)NH + 3);                                   // their sums
  cv.take((size_t)2 * kColsumChunks * (C + NH + 3));         // fp64 column-sum partials
  if (s1.S > 1) cv.take((size_t)s1.S * B * nC);
  if (s2.S > 1) cv.take((size_t)s2.S * NH * nC);
  return cv.off;
}

// dynamic shared memory of the per-token stream kernels
inline size_t wide_fwd_smem(int NM, int64_t C) { return (size_t)(NM * NM + 2 * NM + C) * sizeof(float); }
inline size_t wide_bwd_smem(int NM, int64_t C) {
  return (size_t)(NM * NM + 2 * NM + 2 * NM * 33 + 2 * C) * sizeof(float);
}
constexpr size_t kWideSmemMax = 200 * 1024;

// Column sums of a [R][W] matrix in fixed order (chunks of rows, then the
// chunk partials in order); part holds kColsumChunks * W doubles.
void wide_colsum(const float* src, int64_t R, int64_t W, int64_t ld, double* part, float* out,
                 cudaStream_t s) {
  int64_t chunk = (R + kColsumChunks - 1) / kColsumChunks;
  if (chunk < 64) chunk = 64;
  const int RB = (int)((R + chunk - 1) / chunk);
  wide_colsum_part_kernel<<<dim3((unsigned)((W + 31) / 32), (unsigned)RB), 256, 0, s>>>(src, R, W, ld, chunk, part);
  wide_colsum_final_kernel<<<grid_1d(W, 256, 1024), 256, 0, s>>>(part, RB, W, out);
}

int run_fwd_wide(const float* x, const float* w, const float* pp, const float* pq, const float* pr,
                 const float* ap, const float* aq, const float* ar, const float* bp,
                 const float* bq, const float* br, float* out, float* token_state, int64_t B,
                 int n, int64_t C, int iters, float s_eps, float r_eps, void* ws, size_t ws_bytes,
                 cudaStream_t s) {
  const int NM = n <= 8 ? 8 : (n <= 16 ? 16 : 32);
  const int64_t NH = (int64_t)n * n + 2 * n, nC = (int64_t)n * C;
  const int RS = rec_stride(n);
  const size_t smem = wide_fwd_smem(NM, C);
  MHC_REQUIRE(smem <= kWideSmemMax, MHC_ERR_UNSUPPORTED,
              "mhc_layer_fwd_dynamic: hidden_dim %lld too large for n = %d", (long long)C, n);
  const size_t need = wide_fwd_ws_bytes(B, n, C, token_state == nullptr);
  MHC_REQUIRE(ws != nullptr && ws_bytes >= need, MHC_ERR_WORKSPACE,
              "mhc_layer_fwd_dynamic: workspace of %zu bytes required, got %zu", need, ws_bytes);
  const WideSplit sp = wide_split_umma(B, NH, nC);
  Carve cv(ws);
  float* rec = token_state ? token_state : cv.take((size_t)B * RS);
  float* part = cv.take((size_t)sp.S * B * NH);
  float* E = cv.take((size_t)B * n * n);
  float* Mb = cv.take((size_t)B * n * n);
  { ProfScope _ps("wide_rms", s); wide_rms_kernel<<<(unsigned)B, 256, 0, s>>>(x, nC, rec, RS, r_eps); }
  {
    ProfScope _ps("wide_gemm_proj", s);
    const dim3 grid((unsigned)((NH + WuCfg::BN - 1) / WuCfg::BN), (unsigned)((B + WuCfg::BM - 1) / WuCfg::BM), (unsigned)sp.S);
    const bool xv = nC % 4 == 0 && aligned16(x);
    const bool pv = nC % 4 == 0 && aligned16(pp) && aligned16(pq) && aligned16(pr);
    cudaFuncSetAttribute(wide_umma_gemm_kernel<true, true, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WuCfg::SMEM);
    wide_umma_gemm_kernel<true, true, 0><<<grid, WuCfg::THREADS, WuCfg::SMEM, s>>>(
        rows1(x, nC), rows3(pp, pq, pr, n, 2 * n, nC), B, NH, nC, sp.kchunk, xv, pv, part, Rows3{}, nullptr, Rows3{});
  }
  { ProfScope _ps("wide_gates", s); wide_gates_kernel<<<(unsigned)B, 256, 0, s>>>(part, sp.S, B, n, ap, aq, ar, bp, bq, br, rec, RS, E); }
  int rc = check_launch("mhc_layer_fwd_dynamic/wide_proj");
  if (rc) return rc;
  rc = mhc_sinkhorn_knopp_fwd(E, Mb, B, n, iters, s_eps, s);
  if (rc) return rc;
  {
    ProfScope _ps("wide_stream_fwd", s);
    if (NM == 8) {
      cudaFuncSetAttribute(wide_stream_fwd_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      wide_stream_fwd_kernel<8><<<(unsigned)B, 256, smem, s>>>(x, w, Mb, rec, RS, out, n, C, r_eps);
    } else if (NM == 16) {
      cudaFuncSetAttribute(wide_stream_fwd_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      wide_stream_fwd_kernel<16><<<(unsigned)B, 256, smem, s>>>(x, w, Mb, rec, RS, out, n, C, r_eps);
    } else {
      cudaFuncSetAttribute(wide_stream_fwd_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      wide_stream_fwd_kernel<32><<<(unsigned)B, 256, smem, s>>>(x, w, Mb, rec, RS, out, n, C, r_eps);
    }
  }
  return check_launch("mhc_layer_fwd_dynamic/wide_stream_fwd");
}

int run_bwd_wide(const float* g, const float* x, const float* w, const float* pp, const float* pq,
                 const float* pr, const float* ap, const float* aq, const float* ar,
                 const float* br, const float* rec, float* gx, float* gw, float* gpp, float* gpq,
                 float* gpr, float* gap, float* gaq, float* gar, float* gbp, float* gbq,
                 float* gbr, int64_t B, int n, int64_t C, int iters, float s_eps, void* ws,
                 size_t ws_bytes, cudaStream_t s) {
  const int NM = n <= 8 ? 8 : (n <= 16 ? 16 : 32);
  const int64_t NH = (int64_t)n * n + 2 * n, nC = (int64_t)n * C;
  const int RS = rec_stride(n);
  const size_t smem = wide_bwd_smem(NM, C);
  MHC_REQUIRE(smem <= kWideSmemMax, MHC_ERR_UNSUPPORTED,
              "mhc_layer_bwd_dynamic: hidden_dim %lld too large for n = %d", (long long)C, n);
  const size_t need = wide_bwd_ws_bytes(B, n, C);
  MHC_REQUIRE(ws != nullptr && ws_bytes >= need, MHC_ERR_WORKSPACE,
              "mhc_layer_bwd_dynamic: workspace of %zu bytes required, got %zu", need, ws_bytes);
  const WideSplit s1 = wide_split_umma(B, nC, NH), s2 = wide_split_umma(NH, nC, B);
  Carve cv(ws);
  float* E = cv.take((size_t)B * n * n);
  float* gE = cv.take((size_t)B * n * n);
  float* gM = cv.take((size_t)B * n * n);
  float* ghh = cv.take((size_t)B * 2 * n);
  float* GP = cv.take((size_t)B * NH);
  float* rows = cv.take((size_t)B * (NH + 3));
  float* coef = cv.take((size_t)B);
  float* gwt = cv.take((size_t)B * C);
  float* tot = cv.take((size_t)NH + 3);
  double* csp = reinterpret_cast<double*>(cv.take((size_t)2 * kColsumChunks * (C + NH + 3)));
  float* part1 = s1.S > 1 ? cv.take((size_t)s1.S * B * nC) : nullptr;
  float* part2 = s2.S > 1 ? cv.take((size_t)s2.S * NH * nC) : nullptr;
  {
    ProfScope _ps("wide_bwd_stream", s);
    if (NM == 8) {
      cudaFuncSetAttribute(wide_bwd_stream_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      wide_bwd_stream_kernel<8><<<(unsigned)B, 256, smem, s>>>(g, x, w, rec, RS, ar, br, n, C, gx, gwt, ghh, gM, E);
    } else if (NM == 16) {
      cudaFuncSetAttribute(wide_bwd_stream_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      wide_bwd_stream_kernel<16><<<(unsigned)B, 256, smem, s>>>(g, x, w, rec, RS, ar, br, n, C, gx, gwt, ghh, gM, E);
    } else {
      cudaFuncSetAttribute(wide_bwd_stream_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      wide_bwd_stream_kernel<32><<<(unsigned)B, 256, smem, s>>>(g, x, w, rec, RS, ar, br, n, C, gx, gwt, ghh, gM, E);
    }
  }
  int rc = check_launch("mhc_layer_bwd_dynamic/wide_bwd_stream");
  if (rc) return rc;
  rc = mhc_sinkhorn_knopp_bwd(gM, E, E, gE, B, n, iters, s_eps, s);
  if (rc) return rc;
  { ProfScope _ps("wide_bwd_token", s); wide_bwd_token_kernel<<<(unsigned)B, 128, 0, s>>>(rec, RS, ghh, gE, E, ap, aq, ar, n, nC, GP, rows, coef); }
  const Rows3 phi = rows3(pp, pq, pr, n, 2 * n, nC);
  const Rows3 xr = rows1(x, nC), gxr = rows1(gx, nC), gpr_ = rows1(GP, NH);
  {
    // grad_x += d_p phi + coef x   (M = tokens, N = nC, K = NH) on tcgen05;
    // phi is an N-contiguous operand here (staged as such, no transposed copy)
    ProfScope _ps("wide_gemm_gx", s);
    const dim3 grid((unsigned)((nC + WuCfg::BN - 1) / WuCfg::BN), (unsigned)((B + WuCfg::BM - 1) / WuCfg::BM), (unsigned)s1.S);
    const bool gv = NH % 4 == 0 && aligned16(GP), tv = nC % 4 == 0 && aligned16(pp) && aligned16(pq) && aligned16(pr);
    if (s1.S == 1) {
      cudaFuncSetAttribute(wide_umma_gemm_kernel<true, false, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WuCfg::SMEM);
      wide_umma_gemm_kernel<true, false, 2><<<grid, WuCfg::THREADS, WuCfg::SMEM, s>>>(gpr_, phi, B, nC, NH, s1.kchunk, gv, tv, nullptr, gxr, coef, xr);
    } else {
      cudaFuncSetAttribute(wide_umma_gemm_kernel<true, false, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WuCfg::SMEM);
      wide_umma_gemm_kernel<true, false, 0><<<grid, WuCfg::THREADS, WuCfg::SMEM, s>>>(gpr_, phi, B, nC, NH, s1.kchunk, gv, tv, part1, Rows3{}, nullptr, Rows3{});
      wide_split_reduce_kernel<2><<<grid_1d(B * nC, 256, 4096), 256, 0, s>>>(part1, s1.S, B, nC, gxr, coef, xr);
    }
  }
  {
    // d_phi = d_p^T X   (M = NH, N = nC, K = tokens) on tcgen05, both
    // operands M/N-contiguous
    ProfScope _ps("wide_gemm_dphi", s);
    const Rows3 gphi = rows3(gpp, gpq, gpr, n, 2 * n, nC);
    const bool gv2 = NH % 4 == 0 && aligned16(GP), xv = nC % 4 == 0 && aligned16(x);
    const dim3 grid((unsigned)((nC + WuCfg::BN - 1) / WuCfg::BN), (unsigned)((NH + WuCfg::BM - 1) / WuCfg::BM), (unsigned)s2.S);
    if (s2.S == 1) {
      cudaFuncSetAttribute(wide_umma_gemm_kernel<false, false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WuCfg::SMEM);
      wide_umma_gemm_kernel<false, false, 1><<<grid, WuCfg::THREADS, WuCfg::SMEM, s>>>(gpr_, xr, NH, nC, B, s2.kchunk, gv2, xv, nullptr, gphi, nullptr, Rows3{});
    } else {
      cudaFuncSetAttribute(wide_umma_gemm_kernel<false, false, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WuCfg::SMEM);
      wide_umma_gemm_kernel<false, false, 0><<<grid, WuCfg::THREADS, WuCfg::SMEM, s>>>(gpr_, xr, NH, nC, B, s2.kchunk, gv2, xv, part2, Rows3{}, nullptr, Rows3{});
      wide_split_reduce_kernel<1><<<grid_1d(NH * nC, 256, 4096), 256, 0, s>>>(part2, s2.S, NH, nC, gphi, nullptr, Rows3{});
    }
  }
  {
    ProfScope _ps("wide_colsum", s);
    wide_colsum(gwt, B, C, C, csp, gw, s);
    wide_colsum(rows, B, NH + 3, NH + 3, csp + kColsumChunks * C, tot, s);
    wide_param_finalize_kernel<<<1, 256, 0, s>>>(tot, n, gbp, gbq, gbr, gap, gaq, gar);
  }
  return check_launch("mhc_layer_bwd_dynamic/wide");
}

// Which kernels run the dynamic layer: the wide-rate set (GEMM projection,
// warp Sinkhorn, block-per-token mixes) for n >= 8, and for n = 6, 7 from
// 1024 tokens; the fused n <= 8 kernels otherwise.  Measured on B200 (fwd +
// bwd, C = 1280): n = 8, 8192 tokens 12.1 -> 3.7 ms; n = 7, 4096 tokens
// 4.8 -> 1.8 ms; n = 5 and small batches favour the fused kernels.  The
// token record keeps rec_stride(n) either way (the wide kernels take the
// stride and ignore the Gram block).
inline bool use_wide(int n, int64_t B) { return n >= 8 || (n >= 6 && B >= 1024); }

int check_layer_args(const char* what, int64_t B, int n, int64_t C, int iters, float s_eps,
                     float r_eps, int max_n = 8) {
  MHC_REQUIRE(B >= 0, MHC_ERR_INVALID_ARG, "%s: batch must be >= 0", what);
  MHC_REQUIRE(C >= 1, MHC_ERR_INVALID_ARG, "%s: hidden_dim must be >= 1", what);
  MHC_REQUIRE(n >= 1 && n <= max_n, MHC_ERR_UNSUPPORTED,
              "%s: expansion_rate n must be in [1, %d], got %d", what, max_n, n);
  MHC_REQUIRE(iters >= 0, MHC_ERR_INVALID_ARG, "%s: sinkhorn_iters must be >= 0", what);
  MHC_REQUIRE(s_eps >= 0.f && r_eps >= 0.f, MHC_ERR_INVALID_ARG, "%s: eps must be >= 0", what);
  MHC_REQUIRE((int64_t)n * C < (1LL << 31), MHC_ERR_UNSUPPORTED, "%s: n*C too large", what);
  return MHC_OK;
}

}  // namespace

// Shared with the allocation-free entry point (noalloc.cu): argument checks of
// the fp32 dynamic forward, and its exact scratch need, which leaves out the
// token record when the caller keeps it (token_state != NULL).
int fwd_dynamic_check_args(const char* what, int64_t B, int n, int64_t C, int iters,
                           float s_eps, float r_eps) {
  return check_layer_args(what, B, n, C, iters, s_eps, r_eps, WIDE_MAX_N);
}

size_t fwd_dynamic_scratch_bytes(int64_t B, int n, int64_t C, bool need_rec) {
  if (B <= 0 || C <= 0 || n < 1 || n > WIDE_MAX_N) return 0;
  if (use_wide(n, B)) return wide_fwd_ws_bytes(B, n, C, need_rec);
  switch (n) {
    case 1: return fwd_ws_bytes<1>(B, C, need_rec);
    case 2: return fwd_ws_bytes<2>(B, C, need_rec);
    case 3: return fwd_ws_bytes<3>(B, C, need_rec);
    case 4: return fwd_ws_bytes<4>(B, C, need_rec);
    case 5: return fwd_ws_bytes<5>(B, C, need_rec);
    case 6: return fwd_ws_bytes<6>(B, C, need_rec);
    case 7: return fwd_ws_bytes<7>(B, C, need_rec);
    default: return fwd_ws_bytes<8>(B, C, need_rec);
  }
}

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
  return fwd_dynamic_scratch_bytes(batch, n, hidden, true);
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
  int rc = check_layer_args(what, batch, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps,
                            sizeof(T) == 4 ? WIDE_MAX_N : 8);
  if (rc) return rc;
  MHC_REQUIRE_PTR(x); MHC_REQUIRE_PTR(rmsnorm_weight); MHC_REQUIRE_PTR(phi_pre);
  MHC_REQUIRE_PTR(phi_post); MHC_REQUIRE_PTR(phi_res); MHC_REQUIRE_PTR(alpha_pre);
  MHC_REQUIRE_PTR(alpha_post); MHC_REQUIRE_PTR(alpha_res); MHC_REQUIRE_PTR(b_pre);
  MHC_REQUIRE_PTR(b_post); MHC_REQUIRE_PTR(b_res); MHC_REQUIRE_PTR(out);
  if (batch == 0) return MHC_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if constexpr (sizeof(T) == 4) {
    if (use_wide(n, batch))
      return run_fwd_wide(x, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre, alpha_post,
                          alpha_res, b_pre, b_post, b_res, out, token_state, batch, n, hidden,
                          sinkhorn_iters, sinkhorn_eps, rmsnorm_eps, workspace, workspace_bytes, s);
  }
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
  if (batch <= 0 || hidden <= 0 || n < 1 || n > WIDE_MAX_N) return 0;
  if (use_wide(n, batch)) return wide_bwd_ws_bytes(batch, n, hidden);
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
  int rc = check_layer_args(what, batch, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps,
                            sizeof(T) == 4 ? WIDE_MAX_N : 8);
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
  if constexpr (sizeof(T) == 4) {
    if (use_wide(n, batch))
      return run_bwd_wide(grad_out, x, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
                          alpha_post, alpha_res, b_res, token_state, grad_x, grad_rmsnorm_weight,
                          grad_phi_pre, grad_phi_post, grad_phi_res, grad_alpha_pre,
                          grad_alpha_post, grad_alpha_res, grad_b_pre, grad_b_post, grad_b_res,
                          batch, n, hidden, sinkhorn_iters, sinkhorn_eps, workspace,
                          workspace_bytes, s);
  }
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

static int wrap_scales(const char* what, const float* scales, int32_t n, WrapScales* sc) {
  MHC_REQUIRE_PTR(scales);
  MHC_REQUIRE(n == 4, MHC_ERR_UNSUPPORTED, "%s: the fused wrapper path needs expansion_rate 4, got %d",
              what, n);
  for (int i = 0; i < 4; ++i) sc->s[i] = scales[i];
  sc->s[0] = 1.0f;
  sc->s[1] = 1.0f;  // the branch stream is taken as is (the projection scales every stream)
  return MHC_OK;
}

extern "C" int mhc_wrapper_fwd_dynamic(
    const float* residual, const float* branch, const float* scales, const float* rmsnorm_weight,
    const float* phi_pre, const float* phi_post, const float* phi_res, const float* alpha_pre,
    const float* alpha_post, const float* alpha_res, const float* b_pre, const float* b_post,
    const float* b_res, float* out_mean, float* token_state, int64_t tokens, int32_t n,
    int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps, float rmsnorm_eps,
    void* workspace, size_t workspace_bytes, void* stream) {
  const char* what = "mhc_wrapper_fwd_dynamic";
  int rc = check_layer_args(what, tokens, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps);
  if (rc) return rc;
  WrapScales sc;
  rc = wrap_scales(what, scales, n, &sc);
  if (rc) return rc;
  MHC_REQUIRE_PTR(residual); MHC_REQUIRE_PTR(branch); MHC_REQUIRE_PTR(rmsnorm_weight);
  MHC_REQUIRE_PTR(phi_pre); MHC_REQUIRE_PTR(phi_post); MHC_REQUIRE_PTR(phi_res);
  MHC_REQUIRE_PTR(alpha_pre); MHC_REQUIRE_PTR(alpha_post); MHC_REQUIRE_PTR(alpha_res);
  MHC_REQUIRE_PTR(b_pre); MHC_REQUIRE_PTR(b_post); MHC_REQUIRE_PTR(b_res); MHC_REQUIRE_PTR(out_mean);
  if (tokens == 0) return MHC_OK;
  return run_fwd_wrap(residual, branch, sc, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
                      alpha_post, alpha_res, b_pre, b_post, b_res, out_mean, token_state, tokens,
                      hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps, workspace,
                      workspace_bytes, (cudaStream_t)stream);
}

extern "C" int mhc_wrapper_fwd_dynamic_prenorm(
    const float* residual, const float* branch, const float* scales, const float* rmsnorm_weight,
    const float* phi_pre, const float* phi_post, const float* phi_res, const float* alpha_pre,
    const float* alpha_post, const float* alpha_res, const float* b_pre, const float* b_post,
    const float* b_res, const float* norm_weight, float norm_eps, float* out_mean,
    float* out_normed, float* out_norm_rms, float* token_state, int64_t tokens, int32_t n,
    int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps, float rmsnorm_eps,
    void* workspace, size_t workspace_bytes, void* stream) {
  const char* what = "mhc_wrapper_fwd_dynamic_prenorm";
  int rc = check_layer_args(what, tokens, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps);
  if (rc) return rc;
  MHC_REQUIRE(norm_eps >= 0.f, MHC_ERR_INVALID_ARG, "%s: norm_eps must be >= 0", what);
  WrapScales sc;
  rc = wrap_scales(what, scales, n, &sc);
  if (rc) return rc;
  MHC_REQUIRE_PTR(residual); MHC_REQUIRE_PTR(branch); MHC_REQUIRE_PTR(rmsnorm_weight);
  MHC_REQUIRE_PTR(phi_pre); MHC_REQUIRE_PTR(phi_post); MHC_REQUIRE_PTR(phi_res);
  MHC_REQUIRE_PTR(alpha_pre); MHC_REQUIRE_PTR(alpha_post); MHC_REQUIRE_PTR(alpha_res);
  MHC_REQUIRE_PTR(b_pre); MHC_REQUIRE_PTR(b_post); MHC_REQUIRE_PTR(b_res); MHC_REQUIRE_PTR(out_mean);
  MHC_REQUIRE_PTR(norm_weight); MHC_REQUIRE_PTR(out_normed); MHC_REQUIRE_PTR(out_norm_rms);
  MHC_REQUIRE(aligned16(norm_weight) && aligned16(out_normed), MHC_ERR_ALIGNMENT,
              "%s: norm_weight and out_normed must be 16-byte aligned", what);
  if (tokens == 0) return MHC_OK;
  PreNorm pn;
  pn.w2 = norm_weight;
  pn.eps2 = norm_eps;
  pn.normed = out_normed;
  pn.rms2 = out_norm_rms;
  return run_fwd_wrap(residual, branch, sc, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
                      alpha_post, alpha_res, b_pre, b_post, b_res, out_mean, token_state, tokens,
                      hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps, workspace,
                      workspace_bytes, (cudaStream_t)stream, pn);
}

extern "C" int mhc_wrapper_bwd_dynamic(
    const float* grad_mean, const float* residual, const float* branch, const float* scales,
    const float* rmsnorm_weight, const float* phi_pre, const float* phi_post, const float* phi_res,
    const float* alpha_pre, const float* alpha_post, const float* alpha_res, const float* b_pre,
    const float* b_post, const float* b_res, const float* token_state, float* grad_residual,
    float* grad_branch, float* grad_rmsnorm_weight, float* grad_phi_pre, float* grad_phi_post,
    float* grad_phi_res, float* grad_alpha_pre, float* grad_alpha_post, float* grad_alpha_res,
    float* grad_b_pre, float* grad_b_post, float* grad_b_res, int64_t tokens, int32_t n,
    int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps, float rmsnorm_eps,
    void* workspace, size_t workspace_bytes, void* stream) {
  const char* what = "mhc_wrapper_bwd_dynamic";
  int rc = check_layer_args(what, tokens, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps);
  if (rc) return rc;
  WrapScales sc;
  rc = wrap_scales(what, scales, n, &sc);
  if (rc) return rc;
  MHC_REQUIRE_PTR(grad_mean); MHC_REQUIRE_PTR(residual); MHC_REQUIRE_PTR(branch);
  MHC_REQUIRE_PTR(rmsnorm_weight); MHC_REQUIRE_PTR(phi_pre); MHC_REQUIRE_PTR(phi_post);
  MHC_REQUIRE_PTR(phi_res); MHC_REQUIRE_PTR(alpha_pre); MHC_REQUIRE_PTR(alpha_post);
  MHC_REQUIRE_PTR(alpha_res); MHC_REQUIRE_PTR(b_pre); MHC_REQUIRE_PTR(b_post);
  MHC_REQUIRE_PTR(b_res); MHC_REQUIRE_PTR(token_state); MHC_REQUIRE_PTR(grad_residual);
  MHC_REQUIRE_PTR(grad_branch); MHC_REQUIRE_PTR(grad_rmsnorm_weight);
  MHC_REQUIRE_PTR(grad_phi_pre); MHC_REQUIRE_PTR(grad_phi_post); MHC_REQUIRE_PTR(grad_phi_res);
  MHC_REQUIRE_PTR(grad_alpha_pre); MHC_REQUIRE_PTR(grad_alpha_post);
  MHC_REQUIRE_PTR(grad_alpha_res); MHC_REQUIRE_PTR(grad_b_pre); MHC_REQUIRE_PTR(grad_b_post);
  MHC_REQUIRE_PTR(grad_b_res);
  MHC_REQUIRE(tokens > 0, MHC_ERR_INVALID_ARG, "%s: tokens must be > 0", what);
  return run_bwd_wrap(grad_mean, residual, branch, sc, rmsnorm_weight, phi_pre, phi_post, phi_res,
                      alpha_pre, alpha_post, alpha_res, b_pre, b_post, b_res, token_state,
                      grad_residual, grad_branch, grad_rmsnorm_weight, grad_phi_pre,
                      grad_phi_post, grad_phi_res, grad_alpha_pre, grad_alpha_post,
                      grad_alpha_res, grad_b_pre, grad_b_post, grad_b_res, tokens, hidden,
                      sinkhorn_iters, sinkhorn_eps, rmsnorm_eps, workspace, workspace_bytes,
                      (cudaStream_t)stream);
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
