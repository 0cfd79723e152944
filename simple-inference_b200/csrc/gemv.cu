// gemv.cu -- Q4_0 x Q8_0 matrix-vector product for small token counts (decode).
//
// Reference: matvec_q4q8 (qwen_one_layer.c:148-162) and the column-SoA
// fused_column_matvec (fused_layer.h:169-245): out[n] = bias[n] followed, block
// by block IN ORDER, by  out[n] += ((float)isum * dw) * dx.
//
// Mapping.  One CTA owns an RW-row slice (32, 16 or 8 rows) of one 32-row
// tile of the SoA layout and the whole K range, for up to MT tokens; narrow
// slices give matrices with few tiles enough CTAs to fill the GPU.  Weights,
// their scales and the int8 activations stream through a shared-memory ring
// of chunks filled by cp.async (16-byte pieces: a slice of one block is RW*16
// contiguous bytes).  The ring holds up to 8 chunks: for the small decode
// matrices the whole slice is requested at once; the activation scales of the
// CTA's tokens are staged once.  The 8 warps
// split each chunk of blocks and compute the per-block terms in parallel: the
// int32 block sums are exact, and each term ((float)isum*dw)*dx is rounded
// exactly as the reference rounds it.  The terms go to shared memory; then one
// thread per (token, row) adds them to its running sum in block order, while
// the other warps go on to the next chunk.  The result is bit-identical to the
// reference's serial loop.
//
// SwiGLU mode runs the gate and up tiles of the same rows through the CTA,
// then forms act = silu(g) * u and quantises it to Q8_0 directly: the 32 rows
// of a tile are exactly one Q8 block of the down projection's input.
#include "si_common.cuh"
#include "si_kernels.cuh"

namespace si {

namespace {
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxStages = 8;         // chunks in the shared-memory ring, at most
constexpr size_t kSmemBudget = 200 * 1024;

__device__ __forceinline__ float silu_mul(float g, float u) {
  float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(s, u);
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Wait until at most n of this thread's copy groups are still pending.
__device__ __forceinline__ void cp_async_wait_n(int n) {
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    case 4: cp_async_wait<4>(); break;
    case 5: cp_async_wait<5>(); break;
    case 6: cp_async_wait<6>(); break;
    default: cp_async_wait<7>(); break;
  }
}

// Shape of one instantiation.  A chunk is CB blocks of the RW-row slice; the
// thread (warp w, lane = bo*RW + rl) owns pieces u < U of each chunk: block
// (w*U + u)*BPL + bo, row rl -- for loading and for computing.
template <int MT, int U, int RW>
struct Shape {
  static constexpr int BPL = SI_RT / RW;
  static constexpr int CB = kWarps * U * BPL;
  static constexpr int NIB = CB * RW * 16;      // bytes of nibbles per chunk
  static constexpr int SCL = CB * RW * 2;       // bytes of scales per chunk
  static constexpr int ACT = MT * CB * 32;      // bytes of int8 activations per chunk
  static constexpr int STAGE = NIB + SCL + ACT;
  static constexpr int TERMS = MT * CB * RW;    // floats per term buffer
  // Shared memory: a ring of ns chunks, two term buffers, then the activation
  // scales [MT][KB] fp16.
  static constexpr size_t TERM_BYTES = 2 * TERMS * sizeof(float);
  static size_t smem(int ns, int KB) {
    return (size_t)ns * STAGE + TERM_BYTES + (size_t)MT * KB * sizeof(uint16_t);
  }
  static_assert(SCL / 16 <= kThreads, "one 16-byte scale piece per thread at most");
};

// Streams the RW-row slice (rows r0.. of tile `tile`) of one matrix -- or, with
// SWIGLU, of the gate matrix followed by the up matrix as blocks [0, KB) and
// [KB, 2KB) -- and returns in merge thread t < RW*mcount (token t/RW, row t%RW)
// the in-order sums: `first` gets bias + the terms of blocks [0, KB), the
// return value those of [KB, 2KB) (SWIGLU) or the same sum (otherwise).
template <int MT, int U, int RW, bool SWIGLU>
__device__ __forceinline__ float slice_dot(const GemvArgs &a, int tile, int r0, int m0,
                                           int mcount, float &first, uint8_t *smem, int ns) {
  using S = Shape<MT, U, RW>;
  constexpr int CB = S::CB, BPL = S::BPL;
  const int KB = a.K / 32;
  const int NB = SWIGLU ? 2 * KB : KB;  // blocks streamed
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bo = lane / RW, rl = lane % RW;
  const int tm = threadIdx.x / RW, tr = threadIdx.x % RW;  // merge role: token, row
  const int nchunks = (NB + CB - 1) / CB;
  uint8_t *ring = smem;
  float *T = reinterpret_cast<float *>(smem + (size_t)ns * S::STAGE);
  uint16_t *dxs = reinterpret_cast<uint16_t *>(smem + (size_t)ns * S::STAGE + S::TERM_BYTES);
  const size_t tile_off = (size_t)tile * KB * SI_RT;

  // Weights and their scales of chunk c (no kernel writes them).
  auto issue_w = [&](int c) {
    if (c < nchunks) {
      uint8_t *st = ring + (size_t)(c % ns) * S::STAGE;
      uint4 *nb = reinterpret_cast<uint4 *>(st);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int bl = (warp * U + u) * BPL + bo;
        const int b = c * CB + bl;
        if (b < NB) {
          const bool second = SWIGLU && b >= KB;
          const uint8_t *src = second ? a.nib2 : a.nib;
          const int bb = second ? b - KB : b;
          cp_async16(nb + bl * RW + rl,
                     src + ((tile_off + (size_t)bb * SI_RT + r0 + rl) << 4));
        }
      }
      // Scales: 8 rows (16 bytes) per piece.
      constexpr int PIECES = S::SCL / 16, PPB = RW / 8;
      if (threadIdx.x < PIECES) {
        const int bl = threadIdx.x / PPB, rg = (threadIdx.x % PPB) * 8;
        const int b = c * CB + bl;
        if (b < NB) {
          const bool second = SWIGLU && b >= KB;
          const uint16_t *src = second ? a.scl2 : a.scl;
          const int bb = second ? b - KB : b;
          cp_async16(st + S::NIB + (size_t)(bl * RW + rg) * 2,
                     src + tile_off + (size_t)bb * SI_RT + r0 + rg);
        }
      }
    }
  };
  // int8 activations of chunk c's blocks: [token][block][32 B].
  auto issue_a = [&](int c) {
    if (c < nchunks) {
      uint8_t *st = ring + (size_t)(c % ns) * S::STAGE;
      for (int i = threadIdx.x; i < mcount * CB * 2; i += kThreads) {
        const int m = i / (CB * 2), bl = (i / 2) % CB, h = i & 1;
        const int b = c * CB + bl;
        if (b < NB) {
          const int bx = (SWIGLU && b >= KB) ? b - KB : b;
          cp_async16(st + S::NIB + S::SCL + ((size_t)(m * CB + bl) * 32 + h * 16),
                     a.xq + (size_t)(m0 + m) * a.K + (size_t)bx * 32 + h * 16);
        }
      }
    }
  };

  // Copy groups: one per prologue chunk (weights only), then one with the
  // prologue chunks' activations, then one per later chunk (weights and
  // activations); empty groups keep the count uniform.  The weights of the
  // prologue chunks are requested before the previous kernel has finished.
  for (int c = 0; c < ns - 1; ++c) {
    issue_w(c);
    cp_async_commit();
  }
  pdl_wait();
  float acc = 0.0f;
  if (!SWIGLU && a.bias && tm < mcount) acc = a.bias[tile * SI_RT + r0 + tr];
  for (int c = 0; c < ns - 1; ++c) issue_a(c);
  cp_async_commit();
  // All activation scales of the CTA's tokens, once (visible after the first
  // barrier of the chunk loop).
  for (int i = threadIdx.x; i < mcount * KB; i += kThreads)
    dxs[i] = a.xd[(size_t)(m0 + i / KB) * KB + i % KB];
  for (int c = 0; c < nchunks; ++c) {
    issue_w(c + ns - 1);
    issue_a(c + ns - 1);
    cp_async_commit();
    // Chunk c's data is in group c (prologue weights) and the activation group,
    // or in group c+1 for later chunks: at most min(c+1, ns-1) newer groups.
    cp_async_wait_n(c + 1 < ns - 1 ? c + 1 : ns - 1);
    __syncthreads();  // chunk c landed for every thread; term buffer c&1 is free
    const uint8_t *st = ring + (size_t)(c % ns) * S::STAGE;
    const uint4 *nb = reinterpret_cast<const uint4 *>(st);
    const uint16_t *sb = reinterpret_cast<const uint16_t *>(st + S::NIB);
    const int4 *ab = reinterpret_cast<const int4 *>(st + S::NIB + S::SCL);
    float *Tb = T + (size_t)(c & 1) * S::TERMS;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int bl = (warp * U + u) * BPL + bo;
      const int b = c * CB + bl;
      if (b < NB) {
        const int bx = (SWIGLU && b >= KB) ? b - KB : b;  // activation block
        const uint4 w = nb[bl * RW + rl];
        const float dw = f16_to_f32(sb[bl * RW + rl]);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < mcount) {
            const int4 a0 = ab[(m * CB + bl) * 2], a1 = ab[(m * CB + bl) * 2 + 1];
            const float dx = f16_to_f32(dxs[m * KB + bx]);
            const int is = block_isum(w, a0, a1);
            Tb[((size_t)m * CB + bl) * RW + rl] = block_term(is, dw, dx);
            if (!SWIGLU && a.isum_out)
              a.isum_out[((size_t)(m0 + m) * a.N + (size_t)tile * SI_RT + r0 + rl) * KB + b] = is;
          }
        }
      }
    }
    __syncthreads();  // terms of chunk c visible
    if (tm < mcount) {
      // The adds are a serial chain; load the terms 16 at a time ahead of it
      // so only the add latency remains.
      const int nvalid = min(CB, NB - c * CB);
      const float *Tm = Tb + (size_t)tm * CB * RW + tr;
      // Register double buffer: the next 16 terms are loaded while the current
      // 16 are added.
      int j = 0;
      float v[16], w[16];
      if (nvalid >= 16) {
#pragma unroll
        for (int q = 0; q < 16; ++q) v[q] = Tm[q * RW];
      }
      for (; j + 16 <= nvalid; j += 16) {
        const bool next = j + 32 <= nvalid;
        if (next) {
#pragma unroll
          for (int q = 0; q < 16; ++q) w[q] = Tm[(j + 16 + q) * RW];
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          if (SWIGLU && c * CB + j + q == KB) {
            first = acc;
            acc = 0.0f;
          }
          acc = __fadd_rn(acc, v[q]);
        }
        if (next) {
#pragma unroll
          for (int q = 0; q < 16; ++q) v[q] = w[q];
        }
      }
      for (; j < nvalid; ++j) {
        if (SWIGLU && c * CB + j == KB) {
          first = acc;
          acc = 0.0f;
        }
        acc = __fadd_rn(acc, Tm[j * RW]);
      }
    }
  }
  cp_async_wait<0>();
  if (!SWIGLU) first = acc;
  return acc;
}

// Grid: (N/32 tiles x 32/RW row slices, token groups of MT).
template <int MT, int U, int RW, bool SWIGLU>
__global__ void __launch_bounds__(kThreads) k_gemv(const GemvArgs a, int ns) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int SLICES = SI_RT / RW;
  const int tile = blockIdx.x / SLICES, r0 = (blockIdx.x % SLICES) * RW;
  const int m0 = blockIdx.y * MT;
  const int mcount = min(MT, a.M - m0);
  const int tm = threadIdx.x / RW, tr = threadIdx.x % RW;
  const int row = tile * SI_RT + r0 + tr;

  pdl_trigger();
  float gate = 0.0f;
  const float acc = slice_dot<MT, U, RW, SWIGLU>(a, tile, r0, m0, mcount, gate, smem, ns);
  if (tm >= mcount) return;
  const size_t o = (size_t)(m0 + tm) * a.N + row;
  if (!SWIGLU) {
    a.out[o] = a.resid ? __fadd_rn(a.resid[o], acc) : acc;
  } else {
    // RW == 32: warp m holds token m's 32 outputs of the tile, one Q8 block.
    const float act = silu_mul(gate, acc);
    if (a.out) a.out[o] = act;
    uint16_t d16;
    const int8_t q = q8_lane(act, d16);
    a.act_qs[o] = q;
    if (tr == 0) a.act_d[(size_t)(m0 + tm) * (a.N / 32) + tile] = d16;
  }
}

template <int MT, int U, int RW, bool SWIGLU>
cudaError_t run(const GemvArgs &a, cudaStream_t s) {
  static_assert(!SWIGLU || RW == SI_RT, "the SwiGLU Q8 epilogue needs whole 32-row tiles");
  static_assert(MT * RW <= kThreads, "one merge thread per (token, row)");
  using S = Shape<MT, U, RW>;
  // Ring depth: every chunk of the slice in flight at once when it fits (the
  // small decode matrices are latency-bound), else as many as the budget holds.
  const int KB = a.K / 32, NB = SWIGLU ? 2 * KB : KB;
  const int nchunks = (NB + S::CB - 1) / S::CB;
  int ns = nchunks < 2 ? 2 : (nchunks > kMaxStages ? kMaxStages : nchunks);
  while (ns > 2 && S::smem(ns, KB) > kSmemBudget) --ns;
  const size_t smem = S::smem(ns, KB);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  auto kern = k_gemv<MT, U, RW, SWIGLU>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(a.N / SI_RT * (SI_RT / RW), (a.M + MT - 1) / MT);
  return launch_pdl(kern, grid, dim3(kThreads), smem, s, a, ns);
}

// Row slices per tile: enough CTAs to occupy every SM when the matrix has few
// 32-row tiles (the decode projections of the smaller models).
template <int MT, int U, bool SWIGLU>
cudaError_t pick_rows(const GemvArgs &a, cudaStream_t s) {
  if (SWIGLU) return run<MT, U, 32, true>(a, s);
  const int tiles = a.N / SI_RT;
  if (tiles < 160) return run<MT, U, 8, false>(a, s);
  if (tiles < 320) return run<MT, U, 16, false>(a, s);
  return run<MT, U, 32, false>(a, s);
}

template <bool SWIGLU>
cudaError_t dispatch(const GemvArgs &a, cudaStream_t s) {
  if (a.M <= 1) return pick_rows<1, 4, SWIGLU>(a, s);
  if (a.M <= 2) return pick_rows<2, 4, SWIGLU>(a, s);
  if (a.M <= 4) return pick_rows<4, 2, SWIGLU>(a, s);
  return pick_rows<8, 2, SWIGLU>(a, s);
}
}  // namespace

cudaError_t launch_gemv(const GemvArgs &a, bool swiglu, cudaStream_t s) {
  if (a.M <= 0) return cudaSuccess;
  if ((reinterpret_cast<uintptr_t>(a.nib) | reinterpret_cast<uintptr_t>(a.scl)) & 15)
    return cudaErrorInvalidValue;
  if (swiglu && ((reinterpret_cast<uintptr_t>(a.nib2) | reinterpret_cast<uintptr_t>(a.scl2)) & 15))
    return cudaErrorInvalidValue;
  return swiglu ? dispatch<true>(a, s) : dispatch<false>(a, s);
}

}  // namespace si
