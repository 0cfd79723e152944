// gemv_gguf.cu -- Q4_0 x Q8_0 GEMV straight from row-major GGUF blocks.
//
// The layout the reference's matvec_q4q8 reads (qwen_one_layer.c:148-162) and
// its Llama-style pair schedule walks (bench_llama_fusion.c:79-96): row n is
// KB consecutive 18-byte blocks, each an fp16 scale then 16 bytes of nibbles
// (low nibble of byte j = element j, high = element j + 16).  No repack: this
// kernel measures what skipping the device SoA layout costs.
//
// One warp per row.  The row streams in chunks of 32 blocks (576 bytes: 36
// aligned 16-byte loads shared by the lanes, or 72 8-byte loads where rows are
// only 8-byte aligned; the next chunk's loads in flight while this one is
// used) through shared memory, where lane i finds block i
// at byte 18i -- 2-byte aligned, so its nibble words are funnel-shifted out of
// aligned 32-bit words.  Lane i forms block i's term per token exactly as the
// reference: isum from dp4a over the nibbles XORed with 0x88 and moved to the
// high half of each byte (16*(q-8), so the sum is 16*isum), then
// ((float)isum * dw) * dx, each product rounded.  The terms of a chunk are then
// added to the running sum in block order by the lane that owns the token
// (lane t for token t), from the bias on: the reference's serial chain, so the
// output is bit-identical to matvec_q4q8.
#include <type_traits>

#include "si_common.cuh"
#include "si_kernels.cuh"

namespace si {
namespace {

constexpr int kRowsPerCta = 8;
constexpr int kChunk = 32;                 // blocks per chunk
constexpr int kChunkBytes = kChunk * 18;   // 576 = 36 x 16

// Piece: the load width (16 bytes when rows start 16-byte aligned, KB % 8 == 0;
// else 8 bytes, KB % 4 == 0 -- the 72B down projection's 924 blocks per row).
template <int PIECE>
struct ChunkPieces {
  using T = typename std::conditional<PIECE == 16, uint4, uint2>::type;
  static constexpr int PER_LANE = (kChunkBytes / PIECE + 31) / 32;
};

template <int MT, int PIECE>
__global__ void __launch_bounds__(kRowsPerCta * 32)
    k_gemv_gguf(const uint8_t *__restrict__ w, int N, int KB, const int8_t *__restrict__ xq,
                const uint16_t *__restrict__ xd, int M, const float *__restrict__ bias,
                float *__restrict__ out) {
  using CP = ChunkPieces<PIECE>;
  using P = typename CP::T;
  __shared__ __align__(16) uint8_t chunk_s[kRowsPerCta][kChunkBytes + 16];
  __shared__ float term_s[kRowsPerCta][MT][kChunk + 1];
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerCta + warp;
  if (row >= N) return;  // warp-level work only: no block barrier below
  const P *wr = reinterpret_cast<const P *>(w + (size_t)row * KB * 18);
  const int K = KB * 32;
  // Weights are never written by an earlier kernel: the first chunk's loads
  // go out before the wait for the previous kernel.
  P cur[CP::PER_LANE];
  auto load = [&](int g, P (&r)[CP::PER_LANE]) {
    const int pieces = min(kChunk, KB - g) * 18 / PIECE;
    const P *src = wr + (size_t)g * 18 / PIECE;
#pragma unroll
    for (int k = 0; k < CP::PER_LANE; ++k)
      if (lane + 32 * k < pieces) r[k] = __ldg(src + lane + 32 * k);
  };
  load(0, cur);
  pdl_wait();
  float s = (lane < M && bias) ? bias[row] : 0.0f;  // lane t: token t's running sum
  for (int g = 0; g < KB; g += kChunk) {
    const int nb = min(kChunk, KB - g);
    // Stage this chunk; start the next one's loads.
    P *dst = reinterpret_cast<P *>(chunk_s[warp]);
    const int pieces = nb * 18 / PIECE;
#pragma unroll
    for (int k = 0; k < CP::PER_LANE; ++k)
      if (lane + 32 * k < pieces) dst[lane + 32 * k] = cur[k];
    if (g + kChunk < KB) load(g + kChunk, cur);
    __syncwarp();
    float t[MT];
    if (lane < nb) {
      const uint8_t *blk = chunk_s[warp] + lane * 18;
      const float dw = f16_to_f32(*reinterpret_cast<const uint16_t *>(blk));
      // The 16 nibble bytes start at byte 18*lane + 2: funnel them out of the
      // five aligned words that cover them.
      const int off = lane * 18 + 2, a0 = off & ~3, sh = (off & 3) * 8;
      const uint32_t *wa = reinterpret_cast<const uint32_t *>(chunk_s[warp] + a0);
      uint32_t u[5];
#pragma unroll
      for (int k = 0; k < 5; ++k) u[k] = wa[k];
      int lo[4], hi[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t x = __funnelshift_r(u[k], u[k + 1], sh) ^ 0x88888888u;
        lo[k] = (int)((x << 4) & 0xF0F0F0F0u);
        hi[k] = (int)(x & 0xF0F0F0F0u);
      }
      const int b = g + lane;
#pragma unroll
      for (int tk = 0; tk < MT; ++tk) {
        if (tk < M) {
          const int4 *xa = reinterpret_cast<const int4 *>(xq + (size_t)tk * K + (size_t)b * 32);
          const int4 a0v = xa[0], a1v = xa[1];
          int acc = 0;
          acc = __dp4a(lo[0], a0v.x, acc);
          acc = __dp4a(lo[1], a0v.y, acc);
          acc = __dp4a(lo[2], a0v.z, acc);
          acc = __dp4a(lo[3], a0v.w, acc);
          acc = __dp4a(hi[0], a1v.x, acc);
          acc = __dp4a(hi[1], a1v.y, acc);
          acc = __dp4a(hi[2], a1v.z, acc);
          acc = __dp4a(hi[3], a1v.w, acc);
          const float dx = f16_to_f32(xd[(size_t)tk * KB + b]);
          t[tk] = __fmul_rn(__fmul_rn((float)(acc >> 4), dw), dx);
        }
      }
#pragma unroll
      for (int tk = 0; tk < MT; ++tk)
        if (tk < M) term_s[warp][tk][lane] = t[tk];
    }
    __syncwarp();
    if (lane < M)
      for (int k = 0; k < nb; ++k) s = __fadd_rn(s, term_s[warp][lane][k]);
    __syncwarp();
  }
  if (lane < M) out[(size_t)lane * N + row] = s;
}

}  // namespace

bool gemv_gguf_supported(int N, int K, int M) {
  return N > 0 && K > 0 && K % 128 == 0 && M >= 1 && M <= 8;
}

template <int PIECE>
cudaError_t launch_pieces(const uint8_t *w, int N, int KB, const int8_t *xq, const uint16_t *xd,
                          int M, const float *bias, float *out, cudaStream_t s) {
  const dim3 grid((N + kRowsPerCta - 1) / kRowsPerCta), block(kRowsPerCta * 32);
  if (M == 1)
    return launch_pdl(k_gemv_gguf<1, PIECE>, grid, block, 0, s, w, N, KB, xq, xd, M, bias, out);
  if (M <= 4)
    return launch_pdl(k_gemv_gguf<4, PIECE>, grid, block, 0, s, w, N, KB, xq, xd, M, bias, out);
  return launch_pdl(k_gemv_gguf<8, PIECE>, grid, block, 0, s, w, N, KB, xq, xd, M, bias, out);
}

cudaError_t launch_gemv_gguf(const uint8_t *w, int N, int K, const int8_t *xq, const uint16_t *xd,
                             int M, const float *bias, float *out, cudaStream_t s) {
  if (!gemv_gguf_supported(N, K, M)) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(xq)) & 15)
    return cudaErrorInvalidValue;
  const int KB = K / 32;
  return KB % 8 == 0 ? launch_pieces<16>(w, N, KB, xq, xd, M, bias, out, s)
                     : launch_pieces<8>(w, N, KB, xq, xd, M, bias, out, s);
}

}  // namespace si
