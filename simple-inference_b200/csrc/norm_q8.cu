// norm_q8.cu -- Q8_0 activation quantiser and RMSNorm (+ fused Q8).
//
// Q8_0 (qwen_one_layer.c:98-116): one warp per 32-element block, lane = element.
// RMSNorm (qwen_one_layer.c:164-169): sum of squares in fp64, then
// inv = 1 / sqrtf((float)(ss / n) + eps) and out = (x * inv) * w, each product
// rounded separately.  The fp64 tree sum differs from the reference's serial
// fp64 sum only in the last bits of a double, far below the float rounding.
#include "si_common.cuh"
#include "si_kernels.cuh"

namespace si {

// grid: one warp per block; x [M][K] contiguous, so block index is global.
__global__ void k_q8_quantize(const float *__restrict__ x, size_t nblocks,
                              int8_t *__restrict__ qs, uint16_t *__restrict__ d) {
  size_t blk = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (blk >= nblocks) return;  // whole warp exits together
  uint16_t d16;
  int8_t q = q8_lane(x[blk * 32 + lane], d16);
  qs[blk * 32 + lane] = q;
  if (lane == 0) d[blk] = d16;
}

// One CTA per row.  out (fp32) and the Q8 pair are each optional.
__global__ void __launch_bounds__(256) k_rmsnorm_q8(const float *__restrict__ x,
                                                    const float *__restrict__ w, int n, float eps,
                                                    float *__restrict__ out,
                                                    int8_t *__restrict__ qs,
                                                    uint16_t *__restrict__ d) {
  const int row = blockIdx.x;
  const float *xr = x + (size_t)row * n;
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    double v = (double)xr[i];
    ss = __dadd_rn(ss, __dmul_rn(v, v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  __shared__ double part[8];
  __shared__ float s_inv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t = __dadd_rn(t, part[i]);
    float mean = (float)__ddiv_rn(t, (double)n);
    s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  }
  __syncthreads();
  const float inv = s_inv;
  const int nblocks = n / 32;
  for (int b = warp; b < nblocks; b += (int)(blockDim.x >> 5)) {
    int i = b * 32 + lane;
    float v = __fmul_rn(xr[i], inv);
    if (w) v = __fmul_rn(v, w[i]);
    if (out) out[(size_t)row * n + i] = v;
    if (qs) {
      uint16_t d16;
      int8_t q = q8_lane(v, d16);
      qs[(size_t)row * n + i] = q;
      if (lane == 0) d[(size_t)row * nblocks + b] = d16;
    }
  }
}

__global__ void k_add(const float *__restrict__ a, const float *__restrict__ b,
                      float *__restrict__ y, size_t n) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __fadd_rn(a[i], b[i]);
}

cudaError_t launch_q8_quantize(const float *x, int M, int K, int8_t *qs, uint16_t *d,
                               cudaStream_t s) {
  size_t nblocks = (size_t)M * (K / 32);
  if (nblocks == 0) return cudaSuccess;
  size_t threads = nblocks * 32;
  k_q8_quantize<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, nblocks, qs, d);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm_q8(const float *x, const float *w, int M, int n, float eps,
                              float *out, int8_t *qs, uint16_t *d, cudaStream_t s) {
  if (M == 0) return cudaSuccess;
  k_rmsnorm_q8<<<M, 256, 0, s>>>(x, w, n, eps, out, qs, d);
  return cudaGetLastError();
}

cudaError_t launch_add(const float *a, const float *b, float *y, size_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  k_add<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a, b, y, n);
  return cudaGetLastError();
}

}  // namespace si
