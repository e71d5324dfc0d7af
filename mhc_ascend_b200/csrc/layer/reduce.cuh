// Fixed-order reductions over splits and tokens, the one-launch tail of the
// dynamic backward and the static-H parameter gradients.
// Part of the fused layer translation unit (included by layer.cu, in order).
#pragma once

#include <cuda_bf16.h>

#include "../common.cuh"
#include "../sinkhorn.cuh"
#include "../sinkhorn_lanes.cuh"
#include "../tma.cuh"

namespace mhc {
namespace {

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

}  // namespace
}  // namespace mhc
