// gemv.cu -- Q4_0 x Q8_0 matrix-vector product for small token counts (decode).
//
// Reference: matvec_q4q8 (qwen_one_layer.c:148-162) and the column-SoA
// fused_column_matvec (fused_layer.h:169-245): out[n] = bias[n] followed, block
// by block IN ORDER, by  out[n] += ((float)isum * dw) * dx.
//
// Mapping.  One CTA owns one 32-row tile of the SoA layout and the whole K
// range, for up to MT tokens.  Lane = row, so every warp load of one block is
// 512 contiguous bytes and every activation load is a warp-wide broadcast.
// The 8 warps split each chunk of CB = 8*U blocks (warp w takes U consecutive
// blocks) and compute the per-block terms in parallel: the int32 block sums are
// exact, and each term ((float)isum*dw)*dx is rounded exactly as the
// reference rounds it.  The terms go to shared memory; then warp m adds token
// m's terms to its running sum in block order.  The result is bit-identical to
// the reference's serial loop while all warps stream weights.  Terms are
// double-buffered so one __syncthreads per chunk suffices, and the next
// chunk's weight vectors are prefetched into registers before the current
// chunk's terms are computed.
//
// SwiGLU mode runs the gate and up tiles of the same rows through the CTA,
// then forms act = silu(g) * u and quantises it to Q8_0 directly: the 32 rows
// of a tile are exactly one Q8 block of the down projection's input.
#include "si_common.cuh"
#include "si_kernels.cuh"

namespace si {

namespace {
constexpr int kWarps = 8;

__device__ __forceinline__ float silu_mul(float g, float u) {
  float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(s, u);
}

template <int MT, int U>
__device__ __forceinline__ float tile_dot(const uint8_t *__restrict__ nib,
                                          const uint16_t *__restrict__ scl, int tile, int KB,
                                          int K, const int8_t *__restrict__ xq,
                                          const uint16_t *__restrict__ xd, int m0, int mcount,
                                          float init, float *T, int32_t *isum_out, int N) {
  constexpr int CB = kWarps * U;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint4 *wv = reinterpret_cast<const uint4 *>(nib) + (size_t)tile * KB * SI_RT;
  const uint16_t *sv = scl + (size_t)tile * KB * SI_RT;
  const int nchunks = (KB + CB - 1) / CB;
  float acc = init;

  uint4 wcur[U];
  uint16_t scur[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    int b = warp * U + u;
    if (b < KB) {
      wcur[u] = __ldg(wv + (size_t)b * SI_RT + lane);
      scur[u] = __ldg(sv + (size_t)b * SI_RT + lane);
    }
  }
  for (int c = 0; c < nchunks; ++c) {
    uint4 wnext[U];
    uint16_t snext[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      int b = (c + 1) * CB + warp * U + u;
      if (b < KB) {
        wnext[u] = __ldg(wv + (size_t)b * SI_RT + lane);
        snext[u] = __ldg(sv + (size_t)b * SI_RT + lane);
      }
    }
    float *Tb = T + (size_t)(c & 1) * MT * CB * 32;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      int b = c * CB + warp * U + u;
      if (b < KB) {
        float dw = f16_to_f32(scur[u]);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < mcount) {
            const int8_t *xa = xq + (size_t)(m0 + m) * K + (size_t)b * 32;
            int4 a0 = __ldg(reinterpret_cast<const int4 *>(xa));
            int4 a1 = __ldg(reinterpret_cast<const int4 *>(xa + 16));
            float dx = f16_to_f32(__ldg(xd + (size_t)(m0 + m) * KB + b));
            int is = block_isum(wcur[u], a0, a1);
            Tb[((size_t)m * CB + warp * U + u) * 32 + lane] = block_term(is, dw, dx);
            if (isum_out)
              isum_out[((size_t)(m0 + m) * N + (size_t)tile * SI_RT + lane) * KB + b] = is;
          }
        }
      }
    }
    __syncthreads();
    if (warp < mcount) {
      const int nvalid = min(CB, KB - c * CB);
      const float *Tm = Tb + (size_t)warp * CB * 32 + lane;
      for (int j = 0; j < nvalid; ++j) acc = __fadd_rn(acc, Tm[j * 32]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      wcur[u] = wnext[u];
      scur[u] = snext[u];
    }
  }
  __syncthreads();  // the caller may reuse T for a second matrix
  return acc;
}

template <int MT, int U, bool SWIGLU>
__global__ void __launch_bounds__(kWarps * 32) k_gemv(const GemvArgs a) {
  extern __shared__ float T[];  // [2][MT][CB][32]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int m0 = blockIdx.y * MT;
  const int mcount = min(MT, a.M - m0);
  const int KB = a.K / 32;
  const int row = tile * SI_RT + lane;

  float init = 0.0f;
  if (!SWIGLU && a.bias && warp < mcount) init = a.bias[row];
  float acc = tile_dot<MT, U>(a.nib, a.scl, tile, KB, a.K, a.xq, a.xd, m0, mcount, init, T,
                              a.isum_out, a.N);
  if (!SWIGLU) {
    if (warp < mcount) {
      size_t o = (size_t)(m0 + warp) * a.N + row;
      a.out[o] = a.resid ? __fadd_rn(a.resid[o], acc) : acc;
    }
  } else {
    float up = tile_dot<MT, U>(a.nib2, a.scl2, tile, KB, a.K, a.xq, a.xd, m0, mcount, 0.0f, T,
                               nullptr, a.N);
    if (warp < mcount) {
      float act = silu_mul(acc, up);
      size_t o = (size_t)(m0 + warp) * a.N + row;
      if (a.out) a.out[o] = act;
      uint16_t d16;
      int8_t q = q8_lane(act, d16);
      a.act_qs[o] = q;
      if (lane == 0) a.act_d[(size_t)(m0 + warp) * (a.N / 32) + tile] = d16;
    }
  }
}

template <int MT, int U, bool SWIGLU>
cudaError_t run(const GemvArgs &a, cudaStream_t s) {
  constexpr int CB = kWarps * U;
  size_t smem = (size_t)2 * MT * CB * 32 * sizeof(float);
  auto kern = k_gemv<MT, U, SWIGLU>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(a.N / SI_RT, (a.M + MT - 1) / MT);
  kern<<<grid, kWarps * 32, smem, s>>>(a);
  return cudaGetLastError();
}

template <bool SWIGLU>
cudaError_t dispatch(const GemvArgs &a, cudaStream_t s) {
  if (a.M <= 1) return run<1, 4, SWIGLU>(a, s);
  if (a.M <= 2) return run<2, 4, SWIGLU>(a, s);
  if (a.M <= 4) return run<4, 2, SWIGLU>(a, s);
  return run<8, 2, SWIGLU>(a, s);
}
}  // namespace

cudaError_t launch_gemv(const GemvArgs &a, bool swiglu, cudaStream_t s) {
  if (a.M <= 0) return cudaSuccess;
  return swiglu ? dispatch<true>(a, s) : dispatch<false>(a, s);
}

}  // namespace si
