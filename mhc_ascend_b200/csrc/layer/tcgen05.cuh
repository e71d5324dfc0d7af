// tcgen05 kernels: helpers (shared-memory descriptors, tensor-memory loads and
// stores, MMA issue), the warp-specialised projection and grad_x.
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
// Forward 1 on tcgen05: projection p = x_flat . phi^T and the per-token sum of
// squares, for n <= 4 (C % 32 == 0 fp32 / % 64 bf16, x 16-byte aligned).
//   CTA = 128 tokens (one M=128 MMA tile) x one split of the channels, two
//   CTAs per SM, warp-specialised: warp 0 issues TMA, warp 1 issues MMAs,
//   warps 2..9 (two threads per token, one per half of a 128-byte row)
//   prepare the A operand.  x arrives stream by stream in stages of XW
//   128-byte boxes per token row (256 contiguous bytes per row: 128-byte row
//   pieces cap DRAM at ~73% of its bandwidth, 256-byte ones reach ~90%); each
//   box is one sub-chunk: x[128 tokens x 32 fp32 / 64 bf16 channels] and
//   phi[hi rows | lo rows][those channels] (phi split once per call into tf32
//   hi + lo, both 128-byte-swizzled as TMA writes them).  The operand threads
//   read their token's row, add its squares, and store it split into tf32
//   hi/lo into tensor memory with tcgen05.st (lane = token, column = channel:
//   the A operand, no proxy fence).  3xTF32 in two MMAs per K-step:
//   x_hi . [phi_hi | phi_lo] (N = 2 NB: the hi.hi and hi.lo products land in
//   separate accumulator columns) and x_lo . phi_hi (added to the hi.hi
//   columns).  Every DR sub-chunks the MMA warp switches between two
//   accumulator sets and the operand warps add the finished set into fp32
//   registers, so no accumulation chain in tensor memory is longer than DR
//   sub-chunks.
//   Barriers: xfull / xempty per x stage, pfull / pempty per phi stage,
//   aready / afree per tensor-memory A buffer, dready / dfree per
//   accumulator set.
// ---------------------------------------------------------------------------
template <int N, typename T = float>
struct PumCfg {
  static constexpr int NH = L<N>::NH, NHP = L<N>::NHP;
  static constexpr int NB = (NH + 7) / 8 * 8;              // phi rows per tile (8-row swizzle atoms)
  static constexpr int NC = 2 * NB;                        // MMA N of x_hi . [phi_hi | phi_lo]
  static constexpr int NLO = (NB + 15) / 16 * 16;          // MMA N of x_lo . phi_hi (<= NC)
  // a sub-chunk is one 128-byte box per token row: 32 fp32 or 64 bf16 channels
  static constexpr int TOK = 128, CH = 128 / (int)sizeof(T), THREADS = 320;
  static constexpr int PSUB = CH / 32;                     // 32-channel phi sub-tiles per sub-chunk
  static constexpr bool BF16 = sizeof(T) == 2;             // bf16 x is exact in tf32: no lo part
  static constexpr int XW = 2;                             // boxes per x stage
  static constexpr uint32_t XB = TOK * 128;                // one box of x
  static constexpr uint32_t XS = XW * XB;                  // one x stage
  static constexpr uint32_t PT = NB * 128;                 // one phi_hi (or phi_lo) sub-tile
  static constexpr uint32_t PB = 2 * PT * PSUB;            // phi of one sub-chunk: [hi | lo] per sub-tile
  // two rings, each refilled by its own producer thread: x (released once the
  // operand warps hold it in registers) and phi (released when the
  // sub-chunk's MMAs are done; deep, to hide the L2 latency between a
  // sub-chunk's MMAs and the load of the phi tile SP sub-chunks later)
  static constexpr int SX = 2, SP = BF16 ? 3 : 6, NA = 2;  // x stages, phi stages, tensor-memory A buffers
  static constexpr uint32_t OFF_PR = SX * XS;              // phi ring after the x ring
  // tensor memory: accumulator sets D[s] = [64 s, 64 s + NC); A[a] = [128 + 64 a, +64): fp32 hi|lo, bf16 hi
  static constexpr uint32_t TCOLS = 256, ACOL = 128;
  // sub-chunks accumulated into one set before the operand warps add it into
  // fp32 registers.  Accumulation in tensor memory rounds toward
  // zero (measured: a relative shrink of ~2e-8 per accumulating MMA, uniform
  // over all outputs), so chains stay at DR x 8 MMAs: 32 at DR = 4, ~6e-7.
  static constexpr int DR = 4;
  static constexpr uint32_t OFF_BAR = OFF_PR + SP * PB;
  // after the last MMA the x ring holds the exchange: sum of squares [128],
  // phi_lo sums [NB][128]
  static_assert(TOK * 4 + NB * TOK * 4 <= SX * XS, "exchange fits the x ring");
  static constexpr size_t SMEM = OFF_BAR + (2 * SX + 2 * SP + 2 * NA + 4 + 1) * 8 + 16 + 1024;
  static_assert(NC <= 64 && NB % 8 == 0, "one 64-column accumulator set");
  static_assert(XB % 1024 == 0 && PT % 1024 == 0 && OFF_PR % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
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
  if (mbar_poll(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    if (mbar_poll(addr, parity)) return true;
    if (*abort_word) return false;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  atomicExch(&g_mhc_device_error, 1);
  return false;
}

// WRAP (MHCResidualWrapper, fp32): the streams are not in memory; stream i
// is sc.s[i] * residual (xmap, 2D [tokens, C]) or, for i = 1, the branch
// output (bmap), built in registers as the reference's packing computes them.
template <int N, typename T = float, bool WRAP = false>
__global__ void __launch_bounds__(320, 2)
    proj_umma_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap hmap,
                     const __grid_constant__ CUtensorMap lmap, const __grid_constant__ CUtensorMap bmap,
                     WrapScales sc, float* __restrict__ ppart, float* __restrict__ sqpart, int64_t B,
                     int64_t C, int cps) {
  static_assert(!WRAP || sizeof(T) == 4, "wrapper streams are fp32");
  using P = PumCfg<N, T>;
  constexpr int NHP = P::NHP, NB = P::NB, SX = P::SX, SP = P::SP, NA = P::NA, DR = P::DR, XW = P::XW;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* xfull = reinterpret_cast<uint64_t*>(sm + P::OFF_BAR);
  uint64_t* xempty = xfull + SX;
  uint64_t* pfull = xempty + SX;
  uint64_t* pempty = pfull + SP;
  uint64_t* aready = pempty + SP;
  uint64_t* afree = aready + NA;
  uint64_t* dready = afree + NA;
  uint64_t* dfree = dready + 2;
  uint64_t* done = dfree + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t sbase = smem_u32(sm);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t t0 = (int64_t)blockIdx.x * P::TOK;
  const int split = blockIdx.y;
  const int64_t c_begin = (int64_t)split * cps;
  const int64_t c_end = c_begin + cps < C ? c_begin + cps : C;
  // boxes per stream, x stages per stream (the last one may hold fewer boxes)
  const int nbox = c_begin < c_end ? (int)((c_end - c_begin + P::CH - 1) / P::CH) : 0;
  const int nst = (nbox + XW - 1) / XW;
  const int nstages = nst * N;
  const int nchunks = nbox * N;            // sub-chunks, stream-major

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(P::TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 32) {
    prefetch_tmap(&xmap);
    prefetch_tmap(&hmap);
    prefetch_tmap(&lmap);
    for (int st = 0; st < SX; ++st) {
      mbar_init(&xfull[st], 1);
      mbar_init(&xempty[st], 8);
    }
    for (int st = 0; st < SP; ++st) {
      mbar_init(&pfull[st], 1);
      mbar_init(&pempty[st], 1);
    }
    for (int a = 0; a < NA; ++a) {
      mbar_init(&aready[a], 8);
      mbar_init(&afree[a], 1);
    }
    for (int d = 0; d < 2; ++d) {
      mbar_init(&dready[d], 1);
      mbar_init(&dfree[d], 8);
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
    // ---------------- TMA producers: lane 0 x, lane 1 phi ----------------
    // (separate threads, so neither ring's refill waits on the other's)
    if (lane == 0) {
      int kx = 0;
      for (; kx < nstages; ++kx) {
        if (kx >= SX && !mbar_wait_or_abort(&xempty[kx % SX], (uint32_t)(((kx / SX) - 1) & 1), abort_word)) {
          *abort_word = 1;
          break;
        }
        const int i = kx / nst, sb = kx % nst;
        const int boxes = nbox - sb * XW < XW ? nbox - sb * XW : XW;
        const int c = (int)(c_begin + (int64_t)sb * XW * P::CH);
        unsigned char* xb = sm + (kx % SX) * P::XS;
        mbar_expect_tx(&xfull[kx % SX], (uint32_t)boxes * P::XB);
        for (int bb = 0; bb < boxes; ++bb) {
          if constexpr (WRAP)
            tma_load_2d(xb + bb * P::XB, i == 1 ? &bmap : &xmap, c + bb * P::CH, (int)t0, &xfull[kx % SX]);
          else
            tma_load_3d(xb + bb * P::XB, &xmap, c + bb * P::CH, i, (int)t0, &xfull[kx % SX]);
        }
      }
      // no copy may still be landing when the CTA exits (bounded)
      for (int q = kx > SX ? kx - SX : 0; q < kx; ++q) mbar_wait(&xfull[q % SX], (uint32_t)((q / SX) & 1));
    } else if (lane == 1) {
      int kp = 0;
      for (; kp < nchunks; ++kp) {
        if (kp >= SP && !mbar_wait_or_abort(&pempty[kp % SP], (uint32_t)(((kp / SP) - 1) & 1), abort_word)) {
          *abort_word = 1;
          break;
        }
        const int i = kp / nbox, bx = kp % nbox;
        const int c = (int)(c_begin + (int64_t)bx * P::CH);
        unsigned char* pb = sm + P::OFF_PR + (kp % SP) * P::PB;
        mbar_expect_tx(&pfull[kp % SP], P::PB);
#pragma unroll
        for (int ps = 0; ps < P::PSUB; ++ps) {
          tma_load_3d(pb + ps * 2 * P::PT, &hmap, c + 32 * ps, i, 0, &pfull[kp % SP]);
          tma_load_3d(pb + ps * 2 * P::PT + P::PT, &lmap, c + 32 * ps, i, 0, &pfull[kp % SP]);
        }
      }
      for (int q = kp > SP ? kp - SP : 0; q < kp; ++q) mbar_wait(&pfull[q % SP], (uint32_t)((q / SP) & 1));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t IDC = umma_idesc_tf32(128, P::NC);
      constexpr uint32_t IDL = umma_idesc_tf32(128, P::NLO);
      for (int k = 0; k < nchunks; ++k) {
        const int slot = k % SP, a = k % NA;
        const int run = k / DR, ds = run & 1;
        const bool first = k % DR == 0;
        if ((first && run >= 2 &&
             !mbar_wait_or_abort(&dfree[ds], (uint32_t)(((run - 2) >> 1) & 1), abort_word)) ||
            !mbar_wait_or_abort(&pfull[slot], (uint32_t)((k / SP) & 1), abort_word) ||
            !mbar_wait_or_abort(&aready[a], (uint32_t)((k / NA) & 1), abort_word)) {
          *abort_word = 1;
          break;
        }
        tc_fence_after();
        const uint32_t sb = sbase + P::OFF_PR + slot * P::PB;
        const uint32_t at = tmem + P::ACOL + 64 * a;
        const uint32_t dt = tmem + 64 * ds;
#pragma unroll
        for (int st = 0; st < P::CH / 8; ++st) {
          const uint32_t boff = (st / 4) * 2 * P::PT + 32 * (st % 4);
          const uint64_t bd = umma_desc_sw128(sb + boff);
          umma_tf32_at(dt, at + 8 * st, bd, IDC, (first && st == 0) ? 0u : 1u);
          if constexpr (!P::BF16) umma_tf32_at(dt, at + 32 + 8 * st, bd, IDL, 1u);
        }
        umma_commit(&pempty[slot]);
        umma_commit(&afree[a]);
        if (k % DR == DR - 1 || k == nchunks - 1) umma_commit(&dready[ds]);
      }
      umma_commit(done);
    }
  } else {
    // ---------------- A operand (tensor memory) + sum of squares ----------------
    const int cw = warp - 2;               // 0..7
    const int h = cw >> 2;                 // half of the 128-byte row; accumulator half
    const int qd = warp & 3;               // tensor-memory lane quadrant
    const int r = 32 * qd + lane;          // token row = tensor-memory lane
    const uint32_t rowoff = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
    const uint32_t dlane = (uint32_t)(32 * qd) << 16;
    uint32_t choff[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) choff[j] = rowoff + (uint32_t)((((4 * h + j) ^ (r & 7))) * 16);
    float sq = 0.f;
    // this thread's accumulator columns -- phi_hi terms (h = 0) or phi_lo terms
    // (h = 1) -- summed in fp32 registers
    float pacc[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) pacc[j] = 0.f;
    auto drain = [&](int ds) {
#pragma unroll
      for (int j = 0; j < NB; j += 8) {
        uint32_t d[8];
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]),
                       "=r"(d[6]), "=r"(d[7])
                     : "r"(tmem + dlane + 64 * ds + NB * h + j));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int e = 0; e < 8; ++e) pacc[j + e] += __uint_as_float(d[e]);
      }
    };
    int drained = 0;  // accumulator runs already added into acc_s
    bool ok = true;
    int k = 0;        // sub-chunk
    for (int ks = 0; ks < nstages && ok; ++ks) {
      const int sb = ks % nst;
      const int boxes = nbox - sb * XW < XW ? nbox - sb * XW : XW;
      const int xslot = ks % SX;
      const float scl = WRAP ? sc.s[ks / nst] : 1.f;  // this stage's stream scale
      if (!mbar_wait_or_abort(&xfull[xslot], (uint32_t)((ks / SX) & 1), abort_word)) { ok = false; break; }
      for (int bb = 0; bb < boxes; ++bb, ++k) {
        const int a = k % NA;
        // run `drained` ended one sub-chunk ago: its MMAs are done or nearly
        if (k == (drained + 1) * DR + 1) {
          const int ds = drained & 1;
          if (!mbar_wait_or_abort(&dready[ds], (uint32_t)((drained >> 1) & 1), abort_word)) { ok = false; break; }
          tc_fence_after();
          drain(ds);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dfree[ds]);
          ++drained;
        }
        // this thread's 16 (fp32) or 32 (bf16) channels, as stored
        const unsigned char* base = sm + xslot * P::XS + bb * P::XB;
        uint4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = *reinterpret_cast<const uint4*>(base + choff[j]);
        if (bb == boxes - 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&xempty[xslot]);  // the stage now lives in registers
        }
        if (k >= NA && !mbar_wait_or_abort(&afree[a], (uint32_t)(((k / NA) - 1) & 1), abort_word)) { ok = false; break; }
        tc_fence_after();
        if constexpr (P::BF16) {
          // bf16 -> fp32 is exact and already a tf32 value: hi only
          const uint32_t ta = tmem + dlane + P::ACOL + 64 * a + 32 * h;
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            uint32_t hi[16];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const uint32_t w2 = (&v[2 * hf].x)[e];   // channels 2e, 2e+1 of chunks 2hf, 2hf+1
              hi[2 * e] = w2 << 16;
              hi[2 * e + 1] = w2 & 0xFFFF0000u;
              sq = fmaf(__uint_as_float(hi[2 * e]), __uint_as_float(hi[2 * e]), sq);
              sq = fmaf(__uint_as_float(hi[2 * e + 1]), __uint_as_float(hi[2 * e + 1]), sq);
            }
            tmem_st16(ta + 16 * hf, hi);
          }
        } else {
          const uint32_t ta = tmem + dlane + P::ACOL + 64 * a + 16 * h;
          float blk = 0.f;
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            uint32_t hi[8], lo[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              float xe = __uint_as_float((&v[2 * hf].x)[e]);
              if constexpr (WRAP) xe = scl * xe;  // the packed stream value, as the reference rounds it
              blk = fmaf(xe, xe, blk);
              split_tf32(xe, hi[e], lo[e]);
            }
            tmem_st8(ta + 8 * hf, hi);
            tmem_st8(ta + 32 + 8 * hf, lo);
          }
          sq += blk;  // per-box partial first: the rounding grows with boxes, not channels
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&aready[a]);
      }
    }
    if (!ok) *abort_word = 1;
    // the runs not drained yet (at most two): every MMA is complete after `done`
    bool have = ok && nchunks > 0 && mbar_wait_or_abort(done, 0u, abort_word);
    have = __all_sync(0xffffffffu, have);
    tc_fence_after();
    if (have) {
      const int runs = (nchunks + DR - 1) / DR;
      for (; drained < runs; ++drained) drain(drained & 1);
    }
    // exchange: h = 1 hands its sum of squares and phi_lo columns to h = 0
    // ([column][token]: conflict-free)
    float* sq_s = reinterpret_cast<float*>(sm);  // the x ring is idle once every MMA is done
    float* px_s = sq_s + P::TOK + r;
    if (h == 1) {
      sq_s[r] = sq;
#pragma unroll
      for (int j = 0; j < NB; ++j) px_s[j * P::TOK] = pacc[j];
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const int64_t tok = t0 + r;
    if (h == 0 && tok < B && (have || nchunks == 0)) {
      float* pd = ppart + ((int64_t)split * B + tok) * NHP;
#pragma unroll
      for (int j = 0; j < NHP; ++j) pd[j] = pacc[j] + px_s[j * P::TOK];
      sqpart[(int64_t)split * B + tok] = sq + sq_s[r];
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


// Two consecutive stream elements as fp32 (bf16 pairs widen exactly).
__device__ __forceinline__ float2 to_f32x2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 to_f32x2(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

// Add one D2 accumulator (this warp's 32 lanes x NH columns) into the fp32
// sums in shared memory ([column][128 lanes], `d2s` already offset to the lane).
__device__ __forceinline__ void gx6_drain_d2(uint32_t taddr, float* d2s) {
  float a[16], b[16];
  tmem_ld16(taddr, a);
  tmem_ld16(taddr + 16, b);
#pragma unroll
  for (int k = 0; k < 16; ++k) d2s[k * Gx6Cfg::COLS] += a[k];
#pragma unroll
  for (int k = 16; k < Gx6Cfg::NH; ++k) d2s[k * Gx6Cfg::COLS] += b[k - 16];
}

// WRAP (MHCResidualWrapper, fp32): gmap / xmap / bmap are 2D [tokens, C] maps
// of the stream mean's gradient, the residual and the branch output; the
// streams and their gradient are built in registers (g = gmean / 4 for every
// stream, stream j = wsc.s[j] * residual, stream 1 = branch) and the epilogue
// folds the four stream gradients into the residual gradient (omap) and the
// branch gradient (omap2), as the packing's reverse does.
template <typename T, bool WRAP = false>
__global__ void __launch_bounds__(Gx6Cfg::THREADS, 1)
    grad_x6_kernel(const __grid_constant__ CUtensorMap gmap, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap omap, const __grid_constant__ CUtensorMap bmap,
                   const __grid_constant__ CUtensorMap omap2, WrapScales wsc,
                   const float* __restrict__ img, const float* __restrict__ w,
                   const float* __restrict__ phi_pre, const float* __restrict__ phi_post,
                   const float* __restrict__ phi_res, T* __restrict__ gx,
                   float* __restrict__ dphi_part, float* __restrict__ gw_part, int64_t B,
                   int64_t C, int ntiles, int nsplit, int64_t nblk) {
  using F = Gx6Cfg;
  using SM = Gx6S<T, WRAP>;
  static_assert(!WRAP || sizeof(T) == 4, "wrapper streams are fp32");
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
  uint64_t* loc_free = loc_ready + F::NL;
  uint64_t* d2_done = loc_free + F::NL;
  uint64_t* phi_ready = d2_done + 1;
  uint64_t* d2_ready = phi_ready + 1;
  uint64_t* d2_free = d2_ready + 2;
  // the allocation slot and the abort word follow the last barrier
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d2_free + 2);
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
    }
    for (int b = 0; b < F::NL; ++b) {
      mbar_init(&loc_ready[b], F::E_WARPS);
      mbar_init(&loc_free[b], 1);
    }
    mbar_init(d2_done, 1);
    mbar_init(phi_ready, 4);
    for (int d = 0; d < 2; ++d) {
      mbar_init(&d2_ready[d], 1);
      mbar_init(&d2_free[d], 4);
    }
    *abort_word = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // g/x (SG-deep) and the operand image (SI-deep) are refilled
    // independently: whichever ring has a free slot is served, so a late
    // image slot does not hold back the g/x stream (bounded: a poll budget)
    if (lane == 0) {
      int gi = 0, ii = 0;
      uint32_t idle = 0;
      while ((gi < nb || ii < nb) && !*abort_word) {
        if (gi < nb && (gi < SG || mbar_try(&gfree[gi % SG], (uint32_t)(((gi / SG) - 1) & 1)))) {
          const int sg = gi % SG;
          unsigned char* gb = sm + sg * SM::STAGE;
          if constexpr (WRAP) {
            const int trow = (int)((blk0 + gi) * TOK);
            mbar_expect_tx(&gfull[sg], 3 * SM::GB);
            tma_load_2d(gb, &gmap, (int)c0, trow, &gfull[sg]);
            tma_load_2d(gb + SM::GB, &xmap, (int)c0, trow, &gfull[sg]);
            tma_load_2d(gb + 2 * SM::GB, &bmap, (int)c0, trow, &gfull[sg]);
          } else {
            const int row = (int)((blk0 + gi) * TOK * 4);
            mbar_expect_tx(&gfull[sg], 2 * SM::GB);
            tma_load_2d(gb, &gmap, (int)c0, row, &gfull[sg]);
            tma_load_2d(gb + SM::GB, &xmap, (int)c0, row, &gfull[sg]);
          }
          ++gi;
          idle = 0;
        } else if (ii < nb && (ii < SI || mbar_try(&ifree[ii % SI], (uint32_t)(((ii / SI) - 1) & 1)))) {
          const int si = ii % SI;
          mbar_expect_tx(&ifull[si], F::IMG);
          bulk_load(sm + SM::OFF_IMG + si * F::IMG, img + (blk0 + ii) * F::IMG_FLOATS, F::IMG, &ifull[si]);
          ++ii;
          idle = 0;
        } else {
          __nanosleep(64);
          if (++idle >= kSpinLimit) {
            atomicExch(&g_mhc_device_error, 1);
            *abort_word = 1;
          }
        }
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
        const int run = j / F::DR2, ds = run & 1;
        const bool first = j % F::DR2 == 0;
        if (first && run >= 2 &&
            !mbar_wait_or_abort(&d2_free[ds], (uint32_t)(((run - 2) >> 1) & 1), abort_word)) { *abort_word = 1; break; }
        if (!mbar_wait_or_abort(&ifull[si], (uint32_t)((j / SI) & 1), abort_word)) { *abort_word = 1; break; }
        if (!mbar_wait_or_abort(&a2_ready[b], (uint32_t)((j / ND) & 1), abort_word)) { *abort_word = 1; break; }
        tc_fence_after();
        const uint32_t im = sbase + SM::OFF_IMG + si * F::IMG;
        const uint32_t a2 = tmem + F::XT_COL + 2 * TOK * b;
        const uint32_t d2 = tmem + (ds ? F::D2B_COL : F::D2_COL);
#pragma unroll
        for (int ks = 0; ks < TOK / 8; ++ks) {
          const uint32_t ah = a2 + 8 * ks, al = a2 + TOK + 8 * ks;
          const uint64_t bh = umma_desc_k(im + F::IMG_B2H * 4, F::KP, ks, 0);
          const uint64_t bl = umma_desc_k(im + F::IMG_B2L * 4, F::KP, ks, 0);
          if constexpr (SM::BF16) {
            umma_tf32_at(d2, ah, bl, ID2, (!first || ks > 0) ? 1u : 0u);
            umma_tf32_at(d2, ah, bh, ID2, 1u);
          } else {
            umma_tf32_at(d2, al, bh, ID2, (!first || ks > 0) ? 1u : 0u);
            umma_tf32_at(d2, ah, bl, ID2, 1u);
            umma_tf32_at(d2, ah, bh, ID2, 1u);
          }
        }
        umma_commit(&a2_free[b]);
        umma_commit(&ifree[si]);
        if (j % F::DR2 == F::DR2 - 1 || j == nb - 1) umma_commit(&d2_ready[ds]);
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
      float xv[TOK];
      if constexpr (WRAP) {
        const float* rs = reinterpret_cast<const float*>(sm + sg * SM::STAGE + SM::GB);
        const float* bs = rs + TOK * CW;
        const float sq = wsc.s[q];
#pragma unroll
        for (int t = 0; t < TOK; ++t) xv[t] = q == 1 ? bs[t * CW + lane] : sq * rs[t * CW + lane];
      } else {
        const T* xs = reinterpret_cast<const T*>(sm + sg * SM::STAGE) + SM::GB / sizeof(T);
#pragma unroll
        for (int t = 0; t < TOK; ++t) xv[t] = to_f32(xs[(t * 4 + q) * CW + lane]);
      }
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
      // ---------------- E: local terms ----------------
      // warp e takes tokens 2e (lanes 0-15) and 2e + 1 (lanes 16-31); each
      // lane a channel pair (2 cp, 2 cp + 1), computed with packed fp32
      // (f32x2) FMAs: half the instructions of a channel per lane
      static_assert(TPE == 2 && CW == 32, "E-warp lane map");
      const int e = warp - 2;
      const int half = lane >> 4, cp = lane & 15;
      const int t = TPE * e + half;          // this lane's token in the block
      const float2 wc2 = __ldg(reinterpret_cast<const float2*>(w + c0) + cp);
      float2 gwacc = make_float2(0.f, 0.f);
      auto bc = [](float v) { return make_float2(v, v); };
      for (int j = 0; j < nb; ++j) {
        const int sg = j % SG, si = j % SI;
        if (!mbar_wait_or_abort(&gfull[sg], (uint32_t)((j / SG) & 1), abort_word)) { ok = false; break; }
        float2 gv[4], xv[4];                 // [stream], channel pair
        if constexpr (WRAP) {
          const float2* gs = reinterpret_cast<const float2*>(sm + sg * SM::STAGE);
          const float2* rs = gs + TOK * CW / 2;
          const float2* bs = rs + TOK * CW / 2;
          const float2 gq = gs[t * (CW / 2) + cp], rq = rs[t * (CW / 2) + cp], bq = bs[t * (CW / 2) + cp];
          const float2 gq4 = make_float2(gq.x / 4.f, gq.y / 4.f);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            gv[jj] = gq4;
            xv[jj] = jj == 1 ? bq : make_float2(wsc.s[jj] * rq.x, wsc.s[jj] * rq.y);
          }
        } else {
          const T* gs = reinterpret_cast<const T*>(sm + sg * SM::STAGE);
          const T* xs = gs + SM::GB / sizeof(T);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            gv[jj] = to_f32x2(gs + (t * 4 + jj) * CW + 2 * cp);
            xv[jj] = to_f32x2(xs + (t * 4 + jj) * CW + 2 * cp);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&gfree[sg]);   // g, x now live in registers
        if (!mbar_wait_or_abort(&ifull[si], (uint32_t)((j / SI) & 1), abort_word)) { ok = false; break; }
        const float* sc = reinterpret_cast<const float*>(sm + SM::OFF_IMG + si * F::IMG) + F::IMG_SC;
        // local terms of the four streams
        const int lbuf = j % F::NL;
        if (j >= F::NL && !mbar_wait_or_abort(&loc_free[lbuf], (uint32_t)(((j / F::NL) - 1) & 1), abort_word)) { ok = false; break; }
        float* lb = locs + lbuf * (F::LOCB / 4);
        {
          const float* st = sc + t * 32;
          const float4 s0 = *reinterpret_cast<const float4*>(st);
          const float4 h4 = *reinterpret_cast<const float4*>(st + 4);
          const float4 q4 = *reinterpret_cast<const float4*>(st + 8);
          float2 gy = __fmul2_rn(bc(q4.x), gv[0]);
          gy = __ffma2_rn(bc(q4.y), gv[1], gy);
          gy = __ffma2_rn(bc(q4.z), gv[2], gy);
          gy = __ffma2_rn(bc(q4.w), gv[3], gy);
          float2 xa = __fmul2_rn(bc(h4.x), xv[0]);
          xa = __ffma2_rn(bc(h4.y), xv[1], xa);
          xa = __ffma2_rn(bc(h4.z), xv[2], xa);
          xa = __ffma2_rn(bc(h4.w), xv[3], xa);
          // agg = gy w s0.y - xa s0.x
          const float2 agg = __ffma2_rn(__fmul2_rn(gy, wc2), bc(s0.y), __fmul2_rn(xa, bc(-s0.x)));
          const float hh[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 m4 = *reinterpret_cast<const float4*>(st + 12 + 4 * i);
            float2 o = __fmul2_rn(bc(m4.x), gv[0]);
            o = __ffma2_rn(bc(m4.y), gv[1], o);
            o = __ffma2_rn(bc(m4.z), gv[2], o);
            o = __ffma2_rn(bc(m4.w), gv[3], o);
            o = __ffma2_rn(bc(hh[i]), agg, o);
            o = __ffma2_rn(bc(s0.z), xv[i], o);
            *reinterpret_cast<float2*>(lb + t * COLS + i * CW + 2 * cp) = o;
          }
          gwacc = __ffma2_rn(__fmul2_rn(gy, xa), bc(s0.y), gwacc);
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&loc_ready[lbuf]);
          mbar_arrive(&ifree[si]);
        }
      }
      // this warp's two tokens per channel pair, summed: lanes 0-15 hold the result
      gwacc.x += __shfl_xor_sync(0xffffffffu, gwacc.x, 16);
      gwacc.y += __shfl_xor_sync(0xffffffffu, gwacc.y, 16);
      if (half == 0) *reinterpret_cast<float2*>(gws + e * CW + 2 * cp) = gwacc;
    } else {
      // ---------------- epilogue: grad_x = D1 + local term ----------------
      const int i = warp & 3;                // stream = tensor-memory lane quadrant
      const bool leader = warp == 2 + F::E_WARPS && lane == 0;
      float* d2s = reinterpret_cast<float*>(sm + SM::OFF_D2S) + 32 * i + lane;
#pragma unroll
      for (int k = 0; k < F::NH; ++k) d2s[k * COLS] = 0.f;
      int drained = 0;                       // D2 runs already added into d2s
      for (int j = 0; j < nb; ++j) {
        const int b = j % ND;
        if (j == (drained + 1) * F::DR2 - 1 + F::LAG2) {
          const int ds = drained & 1;
          if (!mbar_wait_or_abort(&d2_ready[ds], (uint32_t)((drained >> 1) & 1), abort_word)) { ok = false; break; }
          tc_fence_after();
          gx6_drain_d2(tmem + ((uint32_t)(32 * i) << 16) + (ds ? F::D2B_COL : F::D2_COL), d2s);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&d2_free[ds]);
          ++drained;
        }
        if (!mbar_wait_or_abort(&d1_full[b], (uint32_t)((j / ND) & 1), abort_word)) { ok = false; break; }
        const int lbuf = j % F::NL;
        if (!mbar_wait_or_abort(&loc_ready[lbuf], (uint32_t)((j / F::NL) & 1), abort_word)) { ok = false; break; }
        tc_fence_after();
        float* lb = locs + lbuf * (F::LOCB / 4) + i * CW + lane;
        __nv_bfloat16* sb16 = reinterpret_cast<__nv_bfloat16*>(sm + SM::OFF_STG + lbuf * SM::STGB) + i * CW + lane;
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
        if constexpr (WRAP) {
          // fold the stream gradients: residual = sum_{j != 1, s_j != 0} s_j
          // g_j (stream 0 first), branch = g_1; warp i takes tokens 8i .. 8i + 7
          asm volatile("bar.sync 2, 128;" ::: "memory");
          const float* lt = locs + lbuf * (F::LOCB / 4);
          float* stg = reinterpret_cast<float*>(sm + SM::OFF_STG + lbuf * SM::STGB);
#pragma unroll
          for (int u = 0; u < TOK / 4; ++u) {
            const int t = (TOK / 4) * i + u;
            const float* row = lt + t * COLS + lane;
            float acc = row[0];
#pragma unroll
            for (int jj = 2; jj < 4; ++jj)
              if (wsc.s[jj] != 0.f) acc += wsc.s[jj] * row[jj * CW];
            stg[t * CW + lane] = acc;
            stg[TOK * CW + t * CW + lane] = row[CW];
          }
        }
        fence_proxy_async_smem();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (leader) {
          if constexpr (WRAP) {
            const float* stg = reinterpret_cast<const float*>(sm + SM::OFF_STG + lbuf * SM::STGB);
            tma_store_2d(&omap, stg, (int)c0, (int)((blk0 + j) * TOK));
            tma_store_2d(&omap2, stg + TOK * CW, (int)c0, (int)((blk0 + j) * TOK));
          } else {
            tma_store_2d(&omap, SM::BF16 ? static_cast<const void*>(sm + SM::OFF_STG + lbuf * SM::STGB)
                                         : static_cast<const void*>(locs + lbuf * (F::LOCB / 4)),
                         (int)c0, (int)((blk0 + j) * TOK * 4));
          }
          bulk_commit();
          // the previous block's buffer is free once its store has read it
          // (NL = 3 buffers: the E warps work two blocks ahead)
          if (j > 0) {
            asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
            mbar_arrive(&loc_free[(j - 1) % F::NL]);
          }
        }
      }
      if (leader) {
        bulk_wait0();
        if (ok && nb > 0) mbar_arrive(&loc_free[(nb - 1) % F::NL]);
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
      float* d2s = reinterpret_cast<float*>(sm + SM::OFF_D2S) + 32 * i + lane;
      if (have) {
        // the runs not drained yet (at most two): every MMA is done after d2_done
        const int runs = (nb + F::DR2 - 1) / F::DR2;
        // the block loop drained run d at block (d + 1) DR2 - 1 + LAG2
        int drained = nb >= F::LAG2 ? (nb - F::LAG2) / F::DR2 : 0;
        for (; drained < runs; ++drained)
          gx6_drain_d2(tmem + ((uint32_t)(32 * i) << 16) + ((drained & 1) ? F::D2B_COL : F::D2_COL), d2s);
      }
      if (write) {
        float* dd = dphi_part + (int64_t)split * F::NH * nC + (int64_t)i * C + c;
#pragma unroll
        for (int k = 0; k < F::NH; ++k) dd[(int64_t)k * nC] = d2s[k * COLS];
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

}  // namespace
}  // namespace mhc
