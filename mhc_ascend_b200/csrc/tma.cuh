// TMA (cp.async.bulk.tensor) and mbarrier helpers for the streaming kernels.
//
// Tensor maps are encoded on the host with cuTensorMapEncodeTiled, reached
// through cudaGetDriverEntryPoint (no link-time dependency on libcuda).  Loads
// are plain tiled 2D loads into this CTA's own shared memory: no cluster
// multicast anywhere in this library.
//
// Every wait on an mbarrier is bounded: the waiting thread sleeps in hardware
// between polls, and after ~4 s (globaltimer) it records the failure in the
// translation unit's device error word and the kernel abandons its work
// instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace mhc {

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// nullptr if the driver entry point is unavailable
inline EncodeTiledFn encode_tiled_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Encoding needs the device's context current on the calling thread.  A
// thread that has only set the device (an autograd worker running a backward,
// say) may not have it yet: make it current and retry once.
inline CUresult encode_retry(EncodeTiledFn fn, CUtensorMap* map, CUtensorMapDataType dt,
                             cuuint32_t rank, void* base, const cuuint64_t* dims,
                             const cuuint64_t* strides, const cuuint32_t* box,
                             const cuuint32_t* estr, CUtensorMapSwizzle swizzle) {
  CUresult r = fn(map, dt, rank, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_ERROR_INVALID_CONTEXT) {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess)
      r = fn(map, dt, rank, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  return r;
}

// 2D tensor map (element type dt of esize bytes) over a row-major matrix rows x
// cols (row stride in elements; stride x esize a multiple of 16), box
// box_rows x box_cols, optional shared-memory swizzle; elements outside the
// matrix read as zero.  Returns false on failure.
inline bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, uint32_t esize, const void* base,
                         uint64_t rows, uint64_t cols, uint64_t row_stride_elems, uint32_t box_rows,
                         uint32_t box_cols, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride_elems * esize};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_retry(fn, map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, swizzle);
  return r == CUDA_SUCCESS;
}
inline bool make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                             uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols,
                             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
  return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, rows, cols, row_stride_elems,
                      box_rows, box_cols, swizzle);
}

// 3D tensor map: dims (d0 innermost, d1, d2), byte strides of d1 and d2
// (multiples of 16), box (b0, b1, b2), optional swizzle; out-of-range
// elements read as zero.  Returns false on failure.
inline bool make_tmap_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0,
                         uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                         uint32_t b0, uint32_t b1, uint32_t b2,
                         CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_retry(fn, map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, swizzle);
  return r == CUDA_SUCCESS;
}
inline bool make_tmap_3d_f32(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1,
                             uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                             uint32_t b0, uint32_t b1, uint32_t b2,
                             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
  return make_tmap_3d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, d0, d1, d2, stride1_bytes,
                      stride2_bytes, b0, b1, b2, swizzle);
}

// ---------------------------------------------------------------------------
// device side
// ---------------------------------------------------------------------------
constexpr uint32_t kSpinLimit = 1u << 26;  // ~seconds of polling, then give up

// Error word set by bounded waits that timed out (one per translation unit
// that includes this header; layer.cu exposes its copy through the C-ABI).
static __device__ int g_mhc_device_error = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// One suspending poll: the thread sleeps in hardware until the phase
// completes or about kSuspendNs pass, so waiting warps take no issue slots.
constexpr uint32_t kSuspendNs = 20000;
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // a wait that runs past ~4 s gives up

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_poll(uint32_t addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(addr), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return done != 0;
}

// Bounded wait for completion of the phase with the given parity; returns
// false (and records the error) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_poll(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    if (mbar_poll(addr, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  atomicExch(&g_mhc_device_error, 1);
  return false;
}

// Non-blocking test of the phase with the given parity.
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// plain arrive (no transaction bytes)
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 3D tiled TMA load: box at (c0, c1, c2) of the map into dst (this CTA's smem).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// 1D bulk copy global -> this CTA's smem (addresses 16-byte aligned, bytes a
// multiple of 16), completion counted on the mbarrier.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2D tiled TMA load: box at (col, row) of the map into dst (this CTA's smem).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int col, int row,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(col), "r"(row), "r"(smem_u32(bar))
      : "memory");
}

// 2D tiled TMA store: this CTA's smem tile -> box at (col, row) of the map.
// Completion is tracked with the bulk async-group of the issuing thread.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int col,
                                             int row) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(col), "r"(row)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until the issuing thread's bulk stores have finished reading smem
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// wait until the issuing thread's bulk stores are complete
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// make this thread's generic-proxy smem writes visible to the async proxy
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace mhc
