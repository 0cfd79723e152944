// tc_peak.cu -- int8 tensor-core throughput probe (tcgen05.mma kind::i8).
//
// The roofline denominator for the prefill GEMM: the dense int8 rate this
// device's tensor cores sustain, measured rather than taken from the data
// sheet.  One persistent CTA per SM stages one A tile (128 rows x 128 bytes)
// and one B tile (BN rows x 128 bytes) of pseudo-random int8 in shared memory,
// in the 128-byte-swizzled K-major layout the GEMM uses, then one thread
// issues `iters` x 4 MMAs of 128 x BN x 32 (one K block each) into a TMEM
// accumulator.  Nothing else runs, so the launch's duration is the tensor
// pipe's time for 2*128*BN*32 int8 operations per MMA.  The final commit is
// waited for with the usual bounded wait (about 2 s; SI_ERR_TIMEOUT on
// expiry) and TMEM is freed on every path.
#include "si_common.cuh"
#include "si_kernels.cuh"
#include "si_tc.cuh"
#include "si_tma.cuh"

namespace si {
namespace tc {

template <int BN>
__global__ void __launch_bounds__(128, 1) k_tc_i8_peak(int iters, int *err, int *sink) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<1024>(smem_raw);
  constexpr int A_BYTES = 128 * 128, B_BYTES = BN * 128;
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + A_BYTES + B_BYTES);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bar + 2);
  const int warp = threadIdx.x >> 5;

  // Pseudo-random operands (xorshift of the word index and the CTA).
  for (int i = threadIdx.x; i < (A_BYTES + B_BYTES) / 4; i += blockDim.x) {
    uint32_t v = (uint32_t)i * 0x9E3779B9u ^ (uint32_t)blockIdx.x * 0x85EBCA6Bu;
    v ^= v << 13; v ^= v >> 17; v ^= v << 5;
    reinterpret_cast<uint32_t *>(smem)[i] = v;
  }
  fence_proxy_async();  // generic-proxy stores -> visible to the tensor core
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(bar), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"((uint32_t)BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (threadIdx.x == 0) {
    const uint32_t a0 = smem_u32(smem), b0 = smem_u32(smem + A_BYTES);
    const uint32_t idesc = idesc_i8(128, BN);
    for (int i = 0; i < iters; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        mma_i8(tmem, smem_desc(a0 + 32 * j), smem_desc(b0 + 32 * j), idesc, (i | j) != 0);
    }
    mma_commit(smem_u32(bar));
  }
  __syncwarp();
  if (warp == 0) {
    const bool ok = mbar_wait_warp(smem_u32(bar), 0, abort_flag);
    if (!ok && threadIdx.x == 0) raise_error(err, 6 /* SI_ERR_TIMEOUT */);
    if (ok) {
      tc_fence_after();
      uint32_t r[8];
      tmem_ld8(tmem, r);
      tmem_wait_ld();
      if (threadIdx.x == 0) sink[blockIdx.x] = (int)(r[0] ^ r[7]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)BN));
}

}  // namespace tc

cudaError_t launch_tc_i8_peak(int n, int iters, int *err, int *sink, int *ctas, double *ops,
                              cudaStream_t s) {
  if ((n != 128 && n != 256) || iters < 1) return cudaErrorInvalidValue;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const size_t smem = 128 * 128 + (size_t)n * 128 + 64 + 1024;
  auto kern = n == 256 ? tc::k_tc_i8_peak<256> : tc::k_tc_i8_peak<128>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  count_launch();
  kern<<<sms, 128, smem, s>>>(iters, err, sink);
  if (ctas) *ctas = sms;
  if (ops) *ops = (double)sms * iters * 4 * 2.0 * 128 * n * 32;
  return cudaGetLastError();
}

}  // namespace si
