// si_tma.cuh -- mbarrier, TMA and bounded-wait helpers shared by the
// tcgen05 GEMM and the GEMV (sm_100a), and host-side tensor-map encoding
// through the driver entry point (no link dependency on libcuda).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace si {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
// Aligns a pointer into dynamic shared memory by pointer arithmetic on the
// __shared__ array itself, so the compiler keeps every access derived from it
// in the shared window (an integer round trip turns them into generic loads
// and stores with 64-bit address arithmetic).
template <unsigned ALIGN>
__device__ __forceinline__ uint8_t *smem_align(uint8_t *p) {
  const uint32_t a = smem_u32(p);
  return p + ((ALIGN - (a & (ALIGN - 1))) & (ALIGN - 1));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes (or the hint, 0.5 ms, runs out) instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(500000u)
      : "memory");
  return ok != 0;
}
// Bounded wait: false if the 2 s deadline passes or another role aborted.
// The common case -- the phase completes within one suspended try_wait --
// never reads the global timer.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort) {
  if (mbar_try(bar, parity)) return true;
  if (mbar_try_sleep(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_sleep(bar, parity)) {
    if (*abort) return false;
    if (globaltimer() - t0 > 2000000000ull) return false;
  }
  return true;
}
// The same for a whole warp: every lane polls (each observes the phase itself),
// and all lanes leave together.  A dependent mbarrier wait costs a few hundred
// cycles on B200 even when the phase is already complete, so the kernel keeps
// them to one or two per 4-block stage and issues independent ones together.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile int *abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok) != 0;
}
__device__ __forceinline__ bool mbar_wait2_warp(uint32_t b1, uint32_t p1, uint32_t b2, uint32_t p2,
                                                volatile int *abort) {
  const bool t1 = mbar_try(b1, p1), t2 = mbar_try(b2, p2);  // both in flight at once
  bool ok = true;
  if (!t1) ok = mbar_wait(b1, p1, abort);
  if (ok && !t2) ok = mbar_wait(b2, p2, abort);
  return __all_sync(0xffffffffu, ok) != 0;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- host ---------------------------------------------------------------
inline PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

inline bool tma_encode(CUtensorMap *m, CUtensorMapDataType dt, int rank, const void *base,
                   const cuuint64_t *dims, const cuuint64_t *strides, const cuuint32_t *box,
                   CUtensorMapSwizzle swz) {
  cuuint32_t es[4] = {1, 1, 1, 1};
  return tma_encode_fn()(m, dt, rank, const_cast<void *>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace si
