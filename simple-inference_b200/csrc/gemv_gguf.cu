// gemv_gguf.cu -- Q4_0 x Q8_0 GEMV straight from row-major GGUF blocks.
//
// The layout the reference's matvec_q4q8 reads (qwen_one_layer.c:148-162) and
// its Llama-style pair schedule walks (bench_llama_fusion.c:79-96): row n is
// KB consecutive 18-byte blocks, each an fp16 scale then 16 bytes of nibbles
// (low nibble of byte j = element j, high = element j + 16).  No repack: this
// kernel measures what skipping the device SoA layout costs.
//
// A CTA owns RPC rows (16 or 32) and walks K in chunks of 32 blocks through
// a 4-stage shared-memory ring filled with cp.async three chunks ahead: per
// stage the RPC rows' bytes (576 per row: 16-byte pieces, or 8-byte pieces
// where rows are only 8-byte aligned -- the 72B down projection's 924 blocks
// per row) and the chunk's activations (int8 blocks and fp16 scales), which
// the rows share.  Eight warps compute the terms, each for RPC/8 rows in turn
// with lane i on block i: in the staged row block i sits at byte 18i --
// 2-byte aligned, so its nibble words are funnel-shifted out of aligned
// 32-bit words -- and its term per token is formed exactly as the reference
// does: isum from dp4a over the nibbles XORed with 0x88 and moved to the high
// half of each byte (16*(q-8), so the sum is 16*isum), then ((float)isum *
// dw) * dx, each product rounded.  Then warp t adds token t's terms, one lane
// per row, to the running sums in block order, from the bias on: the
// reference's serial chain for every row at once, so the output is
// bit-identical to matvec_q4q8.
#include <type_traits>

#include "si_common.cuh"
#include "si_kernels.cuh"
#include "si_tma.cuh"

namespace si {
namespace {

constexpr int kChunk = 32;                 // blocks per chunk
constexpr int kChunkBytes = kChunk * 18;   // 576 = 36 x 16
constexpr int kStages = 4;                 // ring stages (chunks in flight: kStages - 1)

template <int PIECE>
__device__ __forceinline__ void cp_async_piece(uint32_t dst, const void *src) {
  if constexpr (PIECE == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}

constexpr int kWarps = 8;
constexpr int kRowBytes = kChunkBytes + 16;  // staged row, padded

// Shared memory of one CTA: the ring's rows [stage][RPC][592], the
// activations [stage][token][32 blocks x 32], their scales [stage][token][32]
// and two buffers of terms [buffer][token][RPC][33].
template <int MT, int RPC>
struct GgufSmem {
  static constexpr int W = 0;
  static constexpr int ACT = W + kStages * RPC * kRowBytes;
  static constexpr int XD = ACT + kStages * MT * kChunk * 32;
  static constexpr int TERM = XD + kStages * MT * kChunk * 2;
  static constexpr int TERMS = MT * RPC * (kChunk + 1);  // floats per term buffer
  static constexpr int BYTES = TERM + 2 * TERMS * 4;
  static_assert(ACT % 16 == 0 && XD % 16 == 0 && TERM % 16 == 0, "alignment");
};

// Piece: the load width (16 bytes when rows start 16-byte aligned, KB % 8 == 0;
// else 8 bytes, KB % 4 == 0).
template <int MT, int PIECE, int RPC>
__global__ void __launch_bounds__(kWarps * 32)
    k_gemv_gguf(const uint8_t *__restrict__ w, int N, int KB, const int8_t *__restrict__ xq,
                const uint16_t *__restrict__ xd, int M, const float *__restrict__ bias,
                float *__restrict__ out) {
  static_assert(MT <= kWarps && RPC % kWarps == 0 && RPC <= 32, "shape");
  using S = GgufSmem<MT, RPC>;
  constexpr int NT = kWarps * 32, RPW = RPC / kWarps;
  extern __shared__ __align__(16) uint8_t smem_g[];
  uint8_t *w_s = smem_g + S::W;                                   // [stage][RPC][kRowBytes]
  int8_t *act_s = reinterpret_cast<int8_t *>(smem_g + S::ACT);   // [stage][MT][1024]
  uint16_t *xd_s = reinterpret_cast<uint16_t *>(smem_g + S::XD); // [stage][MT][32]
  float *term_s = reinterpret_cast<float *>(smem_g + S::TERM);   // [2][MT][RPC][33]
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * RPC;
  const int K = KB * 32;
  const int nchunks = (KB + kChunk - 1) / kChunk;
  // Chunk c into stage c % kStages: warp w's rows, then the CTA's share of the
  // activations and their scales; one commit group per chunk and thread.
  auto issue_weights = [&](int c) {
    const int b0 = c * kChunk, nb = min(kChunk, KB - b0);
    const int pieces = nb * 18 / PIECE;
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int r = warp * RPW + j;
      if (row0 + r < N) {
        const uint8_t *src = w + (size_t)(row0 + r) * KB * 18 + (size_t)b0 * 18;
        const uint32_t dst = smem_u32(w_s + ((c % kStages) * RPC + r) * kRowBytes);
        for (int k = lane; k < pieces; k += 32) cp_async_piece<PIECE>(dst + k * PIECE, src + k * PIECE);
      }
    }
  };
  auto issue_acts = [&](int c) {
    const int b0 = c * kChunk, nb = min(kChunk, KB - b0);
    const int st = c % kStages;
    for (int p = threadIdx.x; p < MT * kChunk * 2; p += NT) {
      const int tk = p / (kChunk * 2), q = p % (kChunk * 2);
      if (tk < M && q / 2 < nb)
        cp_async_piece<16>(smem_u32(act_s + (st * MT + tk) * kChunk * 32 + q * 16),
                           xq + (size_t)tk * K + (size_t)b0 * 32 + q * 16);
    }
    // Scales: 4-byte pieces of two (K % 128 == 0, so KB and nb are even and
    // every piece is 4-byte aligned).
    for (int p = threadIdx.x; p < MT * kChunk / 2; p += NT) {
      const int tk = p / (kChunk / 2), bl = 2 * (p % (kChunk / 2));
      if (tk < M && bl < nb)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                         smem_u32(xd_s + (st * MT + tk) * kChunk + bl)),
                     "l"(xd + (size_t)tk * KB + b0 + bl)
                     : "memory");
    }
  };
  auto commit = [] { asm volatile("cp.async.commit_group;" ::: "memory"); };
  // Weights are never written by an earlier kernel: their first chunks go out
  // before the wait for the previous kernel.
  for (int c = 0; c < kStages - 1; ++c)
    if (c < nchunks) issue_weights(c);
  pdl_wait();
  for (int c = 0; c < kStages - 1; ++c) {
    if (c < nchunks) issue_acts(c);
    commit();
  }
  // Warp t (t < M) keeps token t's running sums, lane r for row row0 + r.
  const int mrow = row0 + lane;
  const bool merger = warp < M && lane < RPC && mrow < N;
  float s = (merger && bias) ? bias[mrow] : 0.0f;
  // Chunk c's terms go to buffer c & 1 and are added while chunk c + 1 is
  // computed (by the merging warps first), so one barrier per chunk orders
  // both: a buffer is rewritten two chunks later, after the next barrier.
  auto merge = [&](int c) {
    if (!merger) return;
    const int nb = min(kChunk, KB - c * kChunk);
    const float *tr = term_s + (c & 1) * S::TERMS + (warp * RPC + lane) * (kChunk + 1);
    if (nb == kChunk) {  // all 32 terms loaded first, then the chain of adds
      float v[kChunk];
#pragma unroll
      for (int k = 0; k < kChunk; ++k) v[k] = tr[k];
#pragma unroll
      for (int k = 0; k < kChunk; ++k) s = __fadd_rn(s, v[k]);
    } else {
      for (int k = 0; k < nb; ++k) s = __fadd_rn(s, tr[k]);
    }
  };
  for (int c = 0; c < nchunks; ++c) {
    const int nb = min(kChunk, KB - c * kChunk);
    const int st = c % kStages;
    asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 2) : "memory");
    __syncthreads();  // chunk c visible, chunk c - 1's terms in; stage (c - 1) % kStages free
    if (c + kStages - 1 < nchunks) {
      issue_weights(c + kStages - 1);
      issue_acts(c + kStages - 1);
    }
    commit();
    if (c > 0) merge(c - 1);
    float *tb = term_s + (c & 1) * S::TERMS;
    if (lane < nb) {
      // This lane's block of the chunk: activations and scales per token.
      int4 av[MT][2];
      float dx[MT];
#pragma unroll
      for (int tk = 0; tk < MT; ++tk)
        if (tk < M) {
          const int4 *xa = reinterpret_cast<const int4 *>(act_s + (st * MT + tk) * kChunk * 32 + lane * 32);
          av[tk][0] = xa[0];
          av[tk][1] = xa[1];
          dx[tk] = f16_to_f32(xd_s[(st * MT + tk) * kChunk + lane]);
        }
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        const int r = warp * RPW + j;
        const uint8_t *wrow = w_s + (st * RPC + r) * kRowBytes;
        const float dw = f16_to_f32(*reinterpret_cast<const uint16_t *>(wrow + lane * 18));
        // The 16 nibble bytes start at byte 18*lane + 2: funnel them out of
        // the five aligned words that cover them.
        const int off = lane * 18 + 2, a0 = off & ~3, sh = (off & 3) * 8;
        const uint32_t *wa = reinterpret_cast<const uint32_t *>(wrow + a0);
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
#pragma unroll
        for (int tk = 0; tk < MT; ++tk) {
          if (tk < M) {
            int acc = 0;
            acc = __dp4a(lo[0], av[tk][0].x, acc);
            acc = __dp4a(lo[1], av[tk][0].y, acc);
            acc = __dp4a(lo[2], av[tk][0].z, acc);
            acc = __dp4a(lo[3], av[tk][0].w, acc);
            acc = __dp4a(hi[0], av[tk][1].x, acc);
            acc = __dp4a(hi[1], av[tk][1].y, acc);
            acc = __dp4a(hi[2], av[tk][1].z, acc);
            acc = __dp4a(hi[3], av[tk][1].w, acc);
            tb[(tk * RPC + r) * (kChunk + 1) + lane] =
                __fmul_rn(__fmul_rn((float)(acc >> 4), dw), dx[tk]);
          }
        }
      }
    }
  }
  __syncthreads();
  merge(nchunks - 1);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (merger) out[(size_t)warp * N + mrow] = s;
}

}  // namespace

bool gemv_gguf_supported(int N, int K, int M) {
  return N > 0 && K > 0 && K % 128 == 0 && M >= 1 && M <= 8;
}

template <int PIECE>
cudaError_t launch_pieces(const uint8_t *w, int N, int KB, const int8_t *xq, const uint16_t *xd,
                          int M, const float *bias, float *out, cudaStream_t s) {
  // 32 rows per CTA when that still gives every SM two CTAs, else 16 (more
  // CTAs, each with a shorter chunk step); eight tokens always take 16.
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  auto go = [&](auto mt, auto rpc) -> cudaError_t {
    constexpr int MT = decltype(mt)::value, RPC = decltype(rpc)::value;
    auto kern = k_gemv_gguf<MT, PIECE, RPC>;
    const int bytes = GgufSmem<MT, RPC>::BYTES;
    if (bytes > 48 * 1024) {
      const cudaError_t e =
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      if (e != cudaSuccess) return e;
    }
    return launch_pdl(kern, dim3((N + RPC - 1) / RPC), dim3(kWarps * 32), bytes, s, w, N, KB, xq,
                      xd, M, bias, out);
  };
  using I1 = std::integral_constant<int, 1>;
  using I4 = std::integral_constant<int, 4>;
  using I8 = std::integral_constant<int, 8>;
  using R16 = std::integral_constant<int, 16>;
  using R32 = std::integral_constant<int, 32>;
  const bool wide = (N + 31) / 32 >= 2 * sms;
  if (M == 1) return wide ? go(I1{}, R32{}) : go(I1{}, R16{});
  if (M <= 4) return wide ? go(I4{}, R32{}) : go(I4{}, R16{});
  return go(I8{}, R16{});
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
