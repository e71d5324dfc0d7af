// Wide expansion rates of the dynamic-H layer (n <= 32; used for n >= 8 and,
// from 1024 tokens, for n = 6, 7 -- use_wide() in layer.cu).
//
// At these rates the projection has n^2 + 2n = 99..1088 outputs over nC
// channels (a real GEMM, not a skinny dot-product pass) and the per-token
// mixes are n x n mat-vecs over C, so the layer is built from different
// pieces than the n <= 8 kernels:
//   fwd : wide_rms (rms_h) -> wide_umma_gemm (P = X phi^T, split-K partials)
//         -> wide_gates (fixed-order split sum, gates, E = exp(t_res))
//         -> Sinkhorn (sinkhorn.cu, warp per matrix) -> wide_stream_fwd
//   bwd : wide_bwd_stream (gy, ghp, RMSNorm reverse, gh, gM, grad_x of the
//         mix / aggregate, gw terms, E) -> Sinkhorn reverse (sinkhorn.cu)
//         -> wide_bwd_token (gate derivatives, d_p, per-token rows of the
//         bias / alpha sums, rms_h coefficient)
//         -> wide_umma_gemm (grad_x += d_p phi + coef x)
//         -> wide_umma_gemm (d_phi = d_p^T X) -> wide_colsum (gw, gb, galpha)
// Every reduction over tokens or splits runs in a fixed order: results are
// bitwise reproducible.  Token-state record: the prefix of the n <= 8 layout
// (rec_stride; no Gram block is written), addressed with the stride passed in.
#pragma once

namespace mhc {

constexpr int WIDE_MAX_N = 32;

// Row-addressed fp32 matrix whose rows may live in up to three tensors (the
// phi_pre | phi_post | phi_res stack): row r < r1 -> p0, r < r2 -> p1, else p2.
struct Rows3 {
  float* p0;
  float* p1;
  float* p2;
  int64_t r1, r2, ld;
  __device__ __forceinline__ float* row(int64_t r) const {
    return r < r1 ? p0 + r * ld : (r < r2 ? p1 + (r - r1) * ld : p2 + (r - r2) * ld);
  }
};
inline Rows3 rows1(const float* p, int64_t ld) {
  return Rows3{const_cast<float*>(p), const_cast<float*>(p), const_cast<float*>(p), INT64_MAX,
               INT64_MAX, ld};
}
inline Rows3 rows3(const float* a, const float* b, const float* c, int64_t r1, int64_t r2,
                   int64_t ld) {
  return Rows3{const_cast<float*>(a), const_cast<float*>(b), const_cast<float*>(c), r1, r2, ld};
}

// Output modes of the contractions (C(m, n) = sum_k A(m, k) B(n, k)):
//   MODE 0: part[z][m][n] = acc              (split-K partials, row length N)
//   MODE 1: Cw.row(m)[n] = acc
//   MODE 2: Cw.row(m)[n] += acc + coef[m] * X.row(m)[n]

// Fixed-order sum of S split-K partials [S][M][N] into the MODE 1 / MODE 2
// destination.
template <int MODE>
__global__ void __launch_bounds__(256)
    wide_split_reduce_kernel(const float* __restrict__ part, int S, int64_t M, int64_t N, Rows3 Cw,
                             const float* __restrict__ coef, Rows3 X) {
  const int64_t total = M * N;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int z = 0; z < S; ++z) acc += part[z * total + e];
    const int64_t m = e / N, nn = e - m * N;
    float* dst = Cw.row(m);
    if (MODE == 2) dst[nn] = dst[nn] + acc + coef[m] * X.row(m)[nn];
    else dst[nn] = acc;
  }
}

// ---------------------------------------------------------------------------
// The same contractions on tcgen05 (kind::tf32, 3xTF32: a_lo b_hi + a_hi b_lo
// + a_hi b_hi, fp32-class accuracy), accumulator in tensor memory.
//   CTA = one 128 x 128 output tile and one K range; 288 threads: warps 0..7
//   stage the operands (coalesced global loads in either layout, split into
//   tf32 hi/lo, stored in the no-swizzle K-major core-matrix layout; the next
//   stage's loads are issued before this stage's stores) and run the
//   epilogue; warp 8 allocates tensor memory and one lane issues 12 MMAs
//   (M = N = 128, K = 8) per 32-k stage.  Barriers: full (256 staging
//   threads), empty and done (MMA commits).  Every wait is
//   bounded; a wait that runs out raises the CTA's abort word and the device
//   error word, and the CTA drains its MMAs before releasing tensor memory.
//   Output modes as above.
// ---------------------------------------------------------------------------
struct WuCfg {
  static constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3;
  static constexpr int LOADERS = 256, THREADS = LOADERS + 32;  // 8 staging warps + MMA warp
  static constexpr uint32_t OPB = 128 * BK * 4;         // one operand part (16 KB)
  static constexpr uint32_t SLOT = 4 * OPB;             // A hi | A lo | B hi | B lo
  static constexpr uint32_t OFF_BAR = STAGES * SLOT;
  static constexpr size_t SMEM = OFF_BAR + (2 * STAGES + 1) * 8 + 16 + 1024;
  static constexpr uint32_t TCOLS = 128;
};

// One staging thread's share of a 128-row x 32-k operand tile (rows r0..,
// k k0..), 16 values held in registers between the load and the store so
// the next stage's loads are in flight while this stage is stored.
//   KC (element (r, k) at R.row(r)[k]): 4 float4 along k; a quarter-warp
//     covers 8 rows of one 4-k group (conflict-free 16-byte stores);
//   otherwise (at R.row(k)[r]): 4 k-rows x 4 consecutive rows (float4 along
//     the rows; a warp reads 512 contiguous bytes per k-row), transposed in
//     registers to 4-k groups.
template <bool KC>
__device__ __forceinline__ void wu_load(const Rows3& R, int64_t r0, int64_t rows, int64_t k0,
                                        int64_t ke, bool vec, int w, int lane, float (&v)[16]) {
  if (KC) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kq = (lane >> 3) + 4 * (j & 1);
      const int r = (j >> 1) * 64 + w * 8 + (lane & 7);
      const int64_t k = k0 + 4 * kq;
      float* d = v + 4 * j;
      d[0] = d[1] = d[2] = d[3] = 0.f;
      if (r0 + r < rows) {
        const float* src = R.row(r0 + r);
        if (vec && k + 3 < ke) {
          const float4 q = __ldg(reinterpret_cast<const float4*>(src + k));
          d[0] = q.x; d[1] = q.y; d[2] = q.z; d[3] = q.w;
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) d[e] = (k + e < ke) ? __ldg(src + k + e) : 0.f;
        }
      }
    }
  } else {
    // 4 k-rows x 4 consecutive rows (float4 along the rows when aligned)
    const int64_t r = r0 + 4 * lane;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int64_t k = k0 + 4 * w + kk;
      float* d = v + 4 * kk;
      d[0] = d[1] = d[2] = d[3] = 0.f;
      if (k < ke) {
        const float* src = R.row(k);
        if (vec && r + 3 < rows) {
          const float4 q = __ldg(reinterpret_cast<const float4*>(src + r));
          d[0] = q.x; d[1] = q.y; d[2] = q.z; d[3] = q.w;
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) d[e] = (r + e < rows) ? __ldg(src + r + e) : 0.f;
        }
      }
    }
  }
}

template <bool KC>
__device__ __forceinline__ void wu_store(const float (&v)[16], unsigned char* hi, unsigned char* lo,
                                         int w, int lane) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t off;
    float a, b, c, d;
    if (KC) {
      const int kq = (lane >> 3) + 4 * (j & 1);
      const int r = (j >> 1) * 64 + w * 8 + (lane & 7);
      off = umma_kmaj_off(r, 4 * kq, 128);
      a = v[4 * j]; b = v[4 * j + 1]; c = v[4 * j + 2]; d = v[4 * j + 3];
    } else {
      off = umma_kmaj_off(4 * lane + j, 4 * w, 128);
      a = v[j]; b = v[4 + j]; c = v[8 + j]; d = v[12 + j];
    }
    uint4 h, l;
    split_tf32(a, h.x, l.x); split_tf32(b, h.y, l.y);
    split_tf32(c, h.z, l.z); split_tf32(d, h.w, l.w);
    *reinterpret_cast<uint4*>(hi + off) = h;
    *reinterpret_cast<uint4*>(lo + off) = l;
  }
}

__device__ __forceinline__ void umma_tf32_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <bool A_KC, bool B_KC, int MODE>
__global__ void __launch_bounds__(WuCfg::THREADS, 1)
    wide_umma_gemm_kernel(Rows3 A, Rows3 Bm, int64_t M, int64_t N, int64_t K, int64_t kchunk,
                          bool a_vec, bool b_vec, float* __restrict__ part, Rows3 Cw,
                          const float* __restrict__ coef, Rows3 X) {
  using W = WuCfg;
  extern __shared__ unsigned char wu_smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(wu_smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + W::OFF_BAR);
  uint64_t* empty = full + W::STAGES;
  uint64_t* done = empty + W::STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t m0 = (int64_t)blockIdx.y * W::BM, n0 = (int64_t)blockIdx.x * W::BN;
  const int64_t kb = (int64_t)blockIdx.z * kchunk;
  const int64_t ke = kb + kchunk < K ? kb + kchunk : K;
  const int nsteps = ke > kb ? (int)((ke - kb + W::BK - 1) / W::BK) : 0;

  if (warp == 8) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(W::TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < W::STAGES; ++s) {
      mbar_init(&full[s], W::LOADERS);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_word = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp < 8) {
    // ---- staging: loads of stage it + 1 in flight while stage it is stored ----
    float va[16], vb[16];
    if (nsteps > 0) {
      wu_load<A_KC>(A, m0, M, kb, ke, a_vec, warp, lane, va);
      wu_load<B_KC>(Bm, n0, N, kb, ke, b_vec, warp, lane, vb);
    }
    for (int it = 0; it < nsteps; ++it) {
      const int s = it % W::STAGES;
      float na[16], nb[16];
      if (it + 1 < nsteps) {
        const int64_t k1 = kb + (int64_t)(it + 1) * W::BK;
        wu_load<A_KC>(A, m0, M, k1, ke, a_vec, warp, lane, na);
        wu_load<B_KC>(Bm, n0, N, k1, ke, b_vec, warp, lane, nb);
      }
      if (it >= W::STAGES && !mbar_wait_or_abort(&empty[s], (uint32_t)((it / W::STAGES - 1) & 1), abort_word)) {
        *abort_word = 1;
        break;
      }
      unsigned char* slot = sm + s * W::SLOT;
      wu_store<A_KC>(va, slot, slot + W::OPB, warp, lane);
      wu_store<B_KC>(vb, slot + 2 * W::OPB, slot + 3 * W::OPB, warp, lane);
      fence_proxy_async_smem();
      mbar_arrive(&full[s]);
      if (it + 1 < nsteps) {
#pragma unroll
        for (int e = 0; e < 16; ++e) { va[e] = na[e]; vb[e] = nb[e]; }
      }
    }
  } else if (lane == 0) {
    // ---- MMA issue ----
    constexpr uint32_t idesc = umma_idesc_tf32(128, 128);
    for (int it = 0; it < nsteps; ++it) {
      const int s = it % W::STAGES;
      if (!mbar_wait_or_abort(&full[s], (uint32_t)((it / W::STAGES) & 1), abort_word)) {
        *abort_word = 1;
        break;
      }
      tc_fence_after();
      const uint32_t base = smem_u32(sm + s * W::SLOT);
#pragma unroll
      for (int ks = 0; ks < W::BK / 8; ++ks) {
        const uint64_t ah = umma_desc_k(base, 128, ks, 0), al = umma_desc_k(base + W::OPB, 128, ks, 0);
        const uint64_t bh = umma_desc_k(base + 2 * W::OPB, 128, ks, 0);
        const uint64_t bl = umma_desc_k(base + 3 * W::OPB, 128, ks, 0);
        umma_tf32_ss(tmem, al, bh, idesc, (it > 0 || ks > 0) ? 1u : 0u);
        umma_tf32_ss(tmem, ah, bl, idesc, 1u);
        umma_tf32_ss(tmem, ah, bh, idesc, 1u);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(done);  // arrives once every MMA issued above has completed
  }

  // ---- epilogue: tensor memory -> shared tile (warp w: lane quadrant w % 4,
  // columns 64 (w / 4) ..) -> global rows, lanes along the columns (float4),
  // so every store instruction writes whole 128-byte lines ----
  if (warp < 8) {
    // plain bounded wait: every MMA issued must have finished before tensor
    // memory is read or released (and before the stage buffers are reused)
    const bool ok = mbar_wait(done, 0u) && !*abort_word;
    tc_fence_after();
    constexpr int TS = 132;  // tile row stride (floats): 16-byte rows, conflict-free
    float* tile = reinterpret_cast<float*>(sm);
    const int q = warp & 3, cbase = 64 * (warp >> 2);
    const int row = 32 * q + lane;
#pragma unroll 1
    for (int c0 = cbase; c0 < cbase + 64; c0 += 16) {
      float v[16];
      if (ok && nsteps > 0) {
        tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 16; e += 4)
        *reinterpret_cast<float4*>(&tile[row * TS + c0 + e]) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(W::LOADERS) : "memory");
    if (ok) {
      const int64_t nc = n0 + 4 * lane;
#pragma unroll 1
      for (int rr = warp; rr < W::BM; rr += 8) {
        const int64_t m = m0 + rr;
        if (m >= M) break;
        float* dst;
        const float* xr = nullptr;
        float cf = 0.f;
        if (MODE == 0) {
          dst = part + ((int64_t)blockIdx.z * M + m) * N;
        } else {
          dst = Cw.row(m);
          if (MODE == 2) { xr = X.row(m); cf = coef[m]; }
        }
        const float4 t = *reinterpret_cast<const float4*>(&tile[rr * TS + 4 * lane]);
        const float tv[4] = {t.x, t.y, t.z, t.w};
        const bool vec4 = (nc + 3 < N) && ((reinterpret_cast<uintptr_t>(dst + nc) & 15) == 0) &&
                          (MODE != 2 || (reinterpret_cast<uintptr_t>(xr + nc) & 15) == 0);
        if (vec4) {
          float4 o = t;
          if (MODE == 2) {
            const float4 d0 = *reinterpret_cast<const float4*>(dst + nc);
            const float4 x0 = __ldg(reinterpret_cast<const float4*>(xr + nc));
            o = make_float4(d0.x + t.x + cf * x0.x, d0.y + t.y + cf * x0.y,
                            d0.z + t.z + cf * x0.z, d0.w + t.w + cf * x0.w);
          }
          *reinterpret_cast<float4*>(dst + nc) = o;
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int64_t nn = nc + e;
            if (nn < N) {
              if (MODE == 2) dst[nn] = dst[nn] + tv[e] + cf * xr[nn];
              else dst[nn] = tv[e];
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(W::TCOLS));
}

// ---------------------------------------------------------------------------
// forward, per token
// ---------------------------------------------------------------------------

// rec[0] = rms_h = sqrt(mean(xf^2) + eps)  (compute_rms, ops_pytorch_backward.py:65-75)
__global__ void __launch_bounds__(256)
    wide_rms_kernel(const float* __restrict__ x, int64_t nC, float* __restrict__ rec, int RS,
                    float eps) {
  __shared__ float red[8];
  __shared__ float out_s[1];
  const int64_t b = blockIdx.x;
  const float* xb = x + b * nC;
  double s = 0.0;
  for (int64_t e = threadIdx.x; e < nC; e += blockDim.x) {
    const float v = xb[e];
    s += (double)(v * v);
  }
  float acc[1] = {(float)s};
  block_sum_array<1>(acc, red, out_s);
  if (threadIdx.x == 0) rec[b * RS] = sqrtf(out_s[0] / (float)nC + eps);
}

// Sums the split-K partials of p in fixed order, stores p and the gates in
// the record and E = exp(t_res) (the Sinkhorn input) in E[b][n*n].
__global__ void __launch_bounds__(256)
    wide_gates_kernel(const float* __restrict__ part, int S, int64_t B, int n,
                      const float* __restrict__ ap, const float* __restrict__ aq,
                      const float* __restrict__ ar, const float* __restrict__ bp,
                      const float* __restrict__ bq, const float* __restrict__ br,
                      float* __restrict__ rec, int RS, float* __restrict__ E) {
  const int64_t b = blockIdx.x;
  const int NH = n * n + 2 * n;
  float* r = rec + b * RS;
  const float inv_rh = 1.0f / r[0];
  const float a0 = *ap, a1 = *aq, a2 = *ar;
  for (int k = threadIdx.x; k < NH; k += blockDim.x) {
    float p = 0.f;
    for (int z = 0; z < S; ++z) p += part[((int64_t)z * B + b) * NH + k];
    r[2 + 2 * n + n * n + k] = p;
    if (k < n) {
      r[2 + k] = sigmoidf_(a0 * p * inv_rh + bp[k]);
    } else if (k < 2 * n) {
      r[2 + k] = 2.0f * sigmoidf_(a1 * p * inv_rh + bq[k - n]);
    } else {
      E[b * n * n + (k - 2 * n)] = expf(a2 * p * inv_rh + br[k - 2 * n]);
    }
  }
}

// Aggregate, RMSNorm and distribute-mix-add of one token per block:
//   a = sum_i h_i x_i ; r = sqrt(mean(a^2) + eps) ; y = a / r * w
//   out_i = hp_i y + sum_j M_ij x_j
// Copies M (from the Sinkhorn output) into the record and stores r.
// Dynamic shared memory: NM*NM + 2*NM + C floats.
template <int NM>
__global__ void __launch_bounds__(256)
    wide_stream_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                           const float* __restrict__ Mbuf, float* __restrict__ rec, int RS,
                           float* __restrict__ out, int n, int64_t C, float eps) {
  extern __shared__ __align__(16) float wsm[];
  float* sM = wsm;                 // [NM][NM]
  float* sh = sM + NM * NM;        // [NM]
  float* shp = sh + NM;            // [NM]
  float* sa = shp + NM;            // [C]
  __shared__ float red[8];
  __shared__ float tot_s[1];
  const int64_t b = blockIdx.x;
  float* r = rec + b * RS;
  const float* xb = x + b * n * C;
  for (int e = threadIdx.x; e < NM * NM; e += blockDim.x) {
    const int i = e / NM, j = e % NM;
    float v = 0.f;
    if (i < n && j < n) {
      v = Mbuf[b * n * n + i * n + j];
      r[2 + 2 * n + i * n + j] = v;
    }
    sM[e] = v;
  }
  for (int i = threadIdx.x; i < NM; i += blockDim.x) {
    sh[i] = i < n ? r[2 + i] : 0.f;
    shp[i] = i < n ? r[2 + n + i] : 0.f;
  }
  __syncthreads();
  float ss[1] = {0.f};
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    float a = 0.f;
    for (int i = 0; i < n; ++i) a += sh[i] * xb[i * C + c];
    sa[c] = a;
    ss[0] += a * a;
  }
  block_sum_array<1>(ss, red, tot_s);
  const float rr = sqrtf(tot_s[0] / (float)C + eps);
  if (threadIdx.x == 0) r[1] = rr;
  float* ob = out + b * n * C;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float y = sa[c] / rr * w[c];
    float xr[NM];
#pragma unroll
    for (int j = 0; j < NM; ++j) xr[j] = j < n ? xb[j * C + c] : 0.f;
    for (int i = 0; i < n; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < NM; j += 4) {
        const float4 m4 = *reinterpret_cast<const float4*>(&sM[i * NM + j]);
        acc = fmaf(m4.x, xr[j], acc);
        acc = fmaf(m4.y, xr[j + 1], acc);
        acc = fmaf(m4.z, xr[j + 2], acc);
        acc = fmaf(m4.w, xr[j + 3], acc);
      }
      ob[i * C + c] = shp[i] * y + acc;
    }
  }
}

// ---------------------------------------------------------------------------
// backward, per token
// ---------------------------------------------------------------------------

// One token per block.  Writes
//   grad_x[i,c] = sum_k M_ki g_k[c] + h_i ga[c]    (mix and aggregate paths)
//   gwt[b][c]   = gy[c] a[c] / r                    (rows of the weight gradient)
//   ghh[b]      = [gh (n) | ghp (n)]
//   gM[b]       = g x^T  (n x n)
//   E[b]        = exp(t_res) (the Sinkhorn input, from the saved projections)
// with a = sum h_i x_i, y = a w / r, gy = sum hp_i g_i, ghp_i = <g_i, y>,
// ga = w gy / r - a S / (C r^3), S = sum gy w a, gh_i = <ga, x_i>.
// Dynamic shared memory: NM*NM + 2*NM + 2*NM*33 + 2*C floats.
// (NM <= 8: capped at 128 registers for two blocks per SM, no spills; the
// uncapped 178-register build ran one block per SM, 1.16 vs 0.67 ms at
// n = 8 and 8192 tokens.)
template <int NM>
__global__ void __launch_bounds__(256, NM <= 8 ? 2 : 1)
    wide_bwd_stream_kernel(const float* __restrict__ g, const float* __restrict__ x,
                           const float* __restrict__ w, const float* __restrict__ rec, int RS,
                           const float* __restrict__ ar, const float* __restrict__ br, int n,
                           int64_t C, float* __restrict__ gx, float* __restrict__ gwt,
                           float* __restrict__ ghh, float* __restrict__ gM,
                           float* __restrict__ E) {
  extern __shared__ __align__(16) float wsm[];
  float* sM = wsm;                 // [NM][NM]
  float* sh = sM + NM * NM;
  float* shp = sh + NM;
  float* sg = shp + NM;            // [NM][33] chunk of g
  float* sx = sg + NM * 33;        // [NM][33] chunk of x
  float* sa = sx + NM * 33;        // [C]
  float* sgy = sa + C;             // [C]
  // NM <= 8: gM = g x^T is accumulated in pass 1 (NM^2 registers) and pass 3 is skipped
  constexpr bool FUSE_GM = NM <= 8;
  constexpr int V1 = NM + 1 + (FUSE_GM ? NM * NM : 0);
  __shared__ float red[8 * V1];
  __shared__ float tot_s[V1];
  const int64_t b = blockIdx.x;
  const float* r = rec + b * RS;
  const float* xb = x + b * n * C;
  const float* gb = g + b * n * C;
  const int nn = n * n;
  for (int e = threadIdx.x; e < NM * NM; e += blockDim.x) {
    const int i = e / NM, j = e % NM;
    sM[e] = (i < n && j < n) ? r[2 + 2 * n + i * n + j] : 0.f;
  }
  for (int i = threadIdx.x; i < NM; i += blockDim.x) {
    sh[i] = i < n ? r[2 + i] : 0.f;
    shp[i] = i < n ? r[2 + n + i] : 0.f;
  }
  {
    const float inv_rh = 1.0f / r[0], a2 = *ar;
    for (int e = threadIdx.x; e < nn; e += blockDim.x)
      E[b * nn + e] = expf(a2 * r[2 + 2 * n + nn + 2 * n + e] * inv_rh + br[e]);
  }
  __syncthreads();
  const float rr = r[1];
  const float inv_r = 1.0f / rr;

  // pass 1: a, gy, S, ghp, gw rows (and gM when FUSE_GM)
  float acc1[V1];
#pragma unroll
  for (int i = 0; i < V1; ++i) acc1[i] = 0.f;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    float a = 0.f, gy = 0.f;
    float gr[NM], xr[NM];
#pragma unroll
    for (int i = 0; i < NM; ++i) {
      gr[i] = i < n ? gb[i * C + c] : 0.f;
      xr[i] = i < n ? xb[i * C + c] : 0.f;
      if (i < n) {
        a += sh[i] * xr[i];
        gy += shp[i] * gr[i];
      }
    }
    if (FUSE_GM) {
#pragma unroll
      for (int i = 0; i < NM; ++i)
#pragma unroll
        for (int j = 0; j < NM; ++j) acc1[NM + 1 + i * NM + j] = fmaf(gr[i], xr[j], acc1[NM + 1 + i * NM + j]);
    }
    const float wc = w[c];
    const float y = a * inv_r * wc;
    sa[c] = a;
    sgy[c] = gy;
    gwt[b * C + c] = gy * a * inv_r;
    acc1[NM] += gy * wc * a;
#pragma unroll
    for (int i = 0; i < NM; ++i) acc1[i] += gr[i] * y;
  }
  block_sum_array<V1>(acc1, red, tot_s);
  const float S = tot_s[NM];
  if (threadIdx.x < n) ghh[b * 2 * n + n + threadIdx.x] = tot_s[threadIdx.x];
  if (FUSE_GM) {
    for (int e = threadIdx.x; e < nn; e += blockDim.x)
      gM[b * nn + e] = tot_s[NM + 1 + (e / n) * NM + (e % n)];
  }
  const float sc = S / ((float)C * rr * rr * rr);
  __syncthreads();  // tot_s is reused below

  // pass 2: ga, gh, grad_x
  float acc2[NM];
#pragma unroll
  for (int i = 0; i < NM; ++i) acc2[i] = 0.f;
  float* gxb = gx + b * n * C;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float ga = w[c] * sgy[c] * inv_r - sa[c] * sc;
    float gr[NM];
#pragma unroll
    for (int k = 0; k < NM; ++k) gr[k] = k < n ? gb[k * C + c] : 0.f;
#pragma unroll
    for (int i = 0; i < NM; ++i) {
      if (i < n) {
        acc2[i] = fmaf(ga, xb[i * C + c], acc2[i]);
        float mix = 0.f;
#pragma unroll
        for (int k = 0; k < NM; ++k) mix = fmaf(sM[k * NM + i], gr[k], mix);
        gxb[i * C + c] = mix + sh[i] * ga;
      }
    }
  }
  block_sum_array<NM>(acc2, red, tot_s);
  if (threadIdx.x < n) ghh[b * 2 * n + threadIdx.x] = tot_s[threadIdx.x];

  if (FUSE_GM) return;

  // pass 3: gM = g x^T over 32-channel chunks
  constexpr int PAIRS = (NM * NM + 255) / 256;
  float accm[PAIRS];
#pragma unroll
  for (int q = 0; q < PAIRS; ++q) accm[q] = 0.f;
  for (int64_t c0 = 0; c0 < C; c0 += 32) {
    __syncthreads();
    for (int e = threadIdx.x; e < NM * 32; e += blockDim.x) {
      const int i = e >> 5, cc = e & 31;
      const bool ok = i < n && c0 + cc < C;
      sg[i * 33 + cc] = ok ? gb[i * C + c0 + cc] : 0.f;
      sx[i * 33 + cc] = ok ? xb[i * C + c0 + cc] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < PAIRS; ++q) {
      const int pr = threadIdx.x + 256 * q;
      if (pr < NM * NM) {
        const int i = pr / NM, j = pr % NM;
        float s = accm[q];
#pragma unroll 8
        for (int cc = 0; cc < 32; ++cc) s = fmaf(sg[i * 33 + cc], sx[j * 33 + cc], s);
        accm[q] = s;
      }
    }
  }
#pragma unroll
  for (int q = 0; q < PAIRS; ++q) {
    const int pr = threadIdx.x + 256 * q;
    if (pr < NM * NM) {
      const int i = pr / NM, j = pr % NM;
      if (i < n && j < n) gM[b * nn + i * n + j] = accm[q];
    }
  }
}

// Gate derivatives and projection gradient of one token per block:
//   gt = gh h (1 - h) | ghp hp (1 - hp/2) | gE E ;  d_p = alpha gt / rms_h
//   GP[b][k] = d_p ; rows[b] = [gt (NH) | sum gt p / rms_h per group (3)]
//   coef[b] = d rms_h / (nC rms_h), d rms_h = -sum gt alpha p / rms_h^2
__global__ void __launch_bounds__(128)
    wide_bwd_token_kernel(const float* __restrict__ rec, int RS, const float* __restrict__ ghh,
                          const float* __restrict__ gE, const float* __restrict__ E,
                          const float* __restrict__ ap, const float* __restrict__ aq,
                          const float* __restrict__ ar, int n, int64_t nC,
                          float* __restrict__ GP, float* __restrict__ rows,
                          float* __restrict__ coef) {
  __shared__ float red[4 * 4];
  __shared__ float tot_s[4];
  const int64_t b = blockIdx.x;
  const int NH = n * n + 2 * n, nn = n * n;
  const float* r = rec + b * RS;
  const float rh = r[0], inv_rh = 1.0f / rh;
  const float al[3] = {*ap, *aq, *ar};
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k = threadIdx.x; k < NH; k += blockDim.x) {
    const float p = r[2 + 2 * n + nn + k];
    float gt;
    int grp;
    if (k < n) {
      const float h = r[2 + k];
      gt = ghh[b * 2 * n + k] * h * (1.0f - h);
      grp = 0;
    } else if (k < 2 * n) {
      const float hp = r[2 + k];
      gt = ghh[b * 2 * n + k] * hp * (1.0f - 0.5f * hp);
      grp = 1;
    } else {
      gt = gE[b * nn + k - 2 * n] * E[b * nn + k - 2 * n];
      grp = 2;
    }
    GP[b * NH + k] = al[grp] * gt * inv_rh;
    rows[b * (NH + 3) + k] = gt;
    const float tp = gt * p * inv_rh;
    acc[grp] += tp;
    acc[3] -= al[grp] * tp * inv_rh;
  }
  block_sum_array<4>(acc, red, tot_s);
  if (threadIdx.x < 3) rows[b * (NH + 3) + NH + threadIdx.x] = tot_s[threadIdx.x];
  if (threadIdx.x == 0) coef[b] = tot_s[3] / ((float)nC * rh);
}

// Fixed-order column sums of src [R][W] (row stride ld) in two launches:
// block (x, y) owns 32 columns of row chunk y (8 row groups accumulate in
// fp64, combined in group order) and writes part[y][col]; the second kernel
// sums the RB chunk partials in chunk order into out[W].
__global__ void __launch_bounds__(256)
    wide_colsum_part_kernel(const float* __restrict__ src, int64_t R, int64_t W, int64_t ld,
                            int64_t rows_per_chunk, double* __restrict__ part) {
  __shared__ double acc[8][32];
  const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.x * 32 + lane;
  const int64_t r_begin = (int64_t)blockIdx.y * rows_per_chunk;
  const int64_t r_end = r_begin + rows_per_chunk < R ? r_begin + rows_per_chunk : R;
  double s = 0.0;
  if (col < W)
    for (int64_t rr = r_begin + grp; rr < r_end; rr += 8) s += (double)src[rr * ld + col];
  acc[grp][lane] = s;
  __syncthreads();
  if (grp == 0 && col < W) {
    double t = 0.0;
    for (int q = 0; q < 8; ++q) t += acc[q][lane];
    part[(int64_t)blockIdx.y * W + col] = t;
  }
}

__global__ void __launch_bounds__(256)
    wide_colsum_final_kernel(const double* __restrict__ part, int RB, int64_t W,
                             float* __restrict__ out) {
  for (int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; col < W;
       col += (int64_t)gridDim.x * blockDim.x) {
    double t = 0.0;
    for (int y = 0; y < RB; ++y) t += part[(int64_t)y * W + col];
    out[col] = (float)t;
  }
}

// tot = [gb_pre (n) | gb_post (n) | gb_res (n^2) | galpha (3)] -> parameter gradients
__global__ void wide_param_finalize_kernel(const float* __restrict__ tot, int n,
                                           float* __restrict__ gbp, float* __restrict__ gbq,
                                           float* __restrict__ gbr, float* __restrict__ gap,
                                           float* __restrict__ gaq, float* __restrict__ gar) {
  const int NH = n * n + 2 * n;
  for (int k = threadIdx.x; k < NH + 3; k += blockDim.x) {
    const float v = tot[k];
    if (k < n) gbp[k] = v;
    else if (k < 2 * n) gbq[k - n] = v;
    else if (k < NH) gbr[k - 2 * n] = v;
    else if (k == NH) *gap = v;
    else if (k == NH + 1) *gaq = v;
    else *gar = v;
  }
}

}  // namespace mhc
