// gemm_tc.cu -- tcgen05 (sm_100a) Q4_0 x Q8_0 GEMM for prefill and batched decode.
//
// Reference semantics: matvec_q4q8 (qwen_one_layer.c:148-162) applied to every
// token, as the weight-stationary prefill does chunk by chunk on the K3
// (prefill_weight_stationary.h:94-106, 207-239): out[t][n] = bias[n], then for
// each 32-wide block b in order  out += ((float)isum(n,t,b) * dw[n,b]) * dx[t,b].
//
// Tile: 128 weight rows (TMEM lanes) x 128 tokens (TMEM columns).  Per K block
// one tcgen05.mma.kind::i8 (K = 32 = one Q4_0/Q8_0 block) writes the exact int32
// block sums of the whole tile into a fresh TMEM accumulator; the epilogue
// warps rescale it in fp32 and add it to register accumulators in block order,
// so results are bit-identical to the reference's serial loop.  Four TMEM
// accumulators (512 columns) let the MMA run up to four blocks ahead of the
// rescale.
//
// Warp roles (384 threads):
//   warp 0      TMA producer (packed Q4 nibbles, int8 activations) and the
//               loader of the activation scales for each stage
//   warp 1      TMEM allocation; lane 0 issues the MMAs and commits
//   warps 2-3   nibble unpack: Q4 -> signed int8 in the 128B-swizzled K-major
//               layout the MMA reads (byte = 16*(q-8), so sums are 16*isum)
//   warps 4-11  epilogue: TMEM -> registers, rescale, accumulate, store
// Stages hold 4 blocks (K = 128 bytes, one swizzle row) and are 4 deep.  Every
// wait is bounded (about 2 s); on expiry the kernel records SI_ERR_TIMEOUT in
// the context's error word, stops all roles, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "si_common.cuh"
#include "si_kernels.cuh"

namespace si {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int KBS = 4;                    // blocks per stage
constexpr int STAGES = 4;
constexpr int NACC = 4;                   // TMEM accumulators (= blocks per stage)
constexpr uint32_t TMEM_COLS = NACC * BN; // 512
constexpr int THREADS = 384;
constexpr int EPI_WARP0 = 4, EPI_WARPS = 8;

constexpr int A_INT8_BYTES = BM * 128;       // 16 KB, SW128 K-major
constexpr int B_BYTES = BN * 128;            // 16 KB, SW128 K-major (TMA swizzled)
constexpr int A_PACK_BYTES = BM * KBS * 16;  // 8 KB
constexpr int DX_BYTES = KBS * BN * 4;       // 2 KB

constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_INT8_BYTES;
constexpr int OFF_PACK = OFF_B + STAGES * B_BYTES;
constexpr int OFF_DX = OFF_PACK + STAGES * A_PACK_BYTES;
constexpr int OFF_BAR = OFF_DX + STAGES * DX_BYTES;
constexpr int NBAR = 5 * STAGES + 2 * NACC;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;  // + alignment slack

static_assert(KBS == NACC, "one accumulator per block of a stage");

struct Params {
  int N, K, M;              // rows (or gate rows for SwiGLU), inputs, tokens
  const uint16_t *scl, *scl2;
  const uint16_t *xd;       // [M][K/32] fp16
  const float *bias, *resid;
  float *out;
  int8_t *act_qs;
  uint16_t *act_d;
  int *err;
};

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
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
// Bounded wait: false if the 2 s deadline passes or another role aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (*abort) return false;
      if (globaltimer() - t0 > 2000000000ull) return false;
    }
  }
}
// The same for a whole warp: lane 0 waits, the outcome is broadcast, so all
// lanes leave together (no divergence at later warp-synchronous steps).
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile int *abort) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  // Each lane observes the completed phase itself (its own acquire); the phase
  // cannot advance again before this warp proceeds, so this returns at once.
  if (ok) ok = mbar_wait(bar, parity, abort);
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
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// K-major operand in the 128-byte swizzle: 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::i8 instruction descriptor: s32 accumulate, signed A and B, both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <bool SWIGLU>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_q4q8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                const __grid_constant__ CUtensorMap tmB, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = p.K / 32;
  const int G = KB / KBS;  // stages over K
  const int t0 = blockIdx.y * BN;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  // barrier indices
  const int B_TMA = 0, B_AREADY = STAGES, B_SEMPTY = 2 * STAGES, B_DXFULL = 3 * STAGES,
            B_DXEMPTY = 4 * STAGES, B_ACCFULL = 5 * STAGES, B_ACCEMPTY = 5 * STAGES + NACC;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC + 16);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar(B_TMA + s), 1);
      mbar_init(bar(B_AREADY + s), 64);
      mbar_init(bar(B_SEMPTY + s), 1);
      mbar_init(bar(B_DXFULL + s), 1);
      mbar_init(bar(B_DXEMPTY + s), EPI_WARPS);
    }
    for (int j = 0; j < NACC; ++j) {
      mbar_init(bar(B_ACCFULL + j), 1);
      mbar_init(bar(B_ACCEMPTY + j), EPI_WARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto fail = [&]() {
    if (p.err) atomicCAS(p.err, 0, 6 /* SI_ERR_TIMEOUT */);
    *abort_flag = 1;
  };

  if (warp == 0) {
    // ---------------- producer: TMA + activation scales ----------------
    for (int g = 0; g < G; ++g) {
      const int s = g % STAGES;
      const uint32_t ph = ((g / STAGES) & 1) ^ 1;
      if (!mbar_wait_warp(bar(B_SEMPTY + s), ph, abort_flag) ||
          !mbar_wait_warp(bar(B_DXEMPTY + s), ph, abort_flag)) {
        if (lane == 0) fail();
        break;
      }
      if (lane == 0) {
        mbar_expect_tx(bar(B_TMA + s), A_PACK_BYTES + B_BYTES);
        uint32_t pack = smem_u32(smem + OFF_PACK + s * A_PACK_BYTES);
        if (SWIGLU) {
          tma_load_4d(pack, &tmA, 0, 0, g * KBS, blockIdx.x * 2, bar(B_TMA + s));
          tma_load_4d(pack + A_PACK_BYTES / 2, &tmA2, 0, 0, g * KBS, blockIdx.x * 2,
                      bar(B_TMA + s));
        } else {
          tma_load_4d(pack, &tmA, 0, 0, g * KBS, blockIdx.x * 4, bar(B_TMA + s));
        }
        tma_load_2d(smem_u32(smem + OFF_B + s * B_BYTES), &tmB, g * 128, t0, bar(B_TMA + s));
      }
      float *dx = reinterpret_cast<float *>(smem + OFF_DX + s * DX_BYTES);
#pragma unroll
      for (int i = 0; i < BN / 32; ++i) {
        const int tl = lane + 32 * i, t = t0 + tl;
        uint2 v = make_uint2(0, 0);
        if (t < p.M) v = __ldg(reinterpret_cast<const uint2 *>(p.xd + (size_t)t * KB + g * KBS));
        dx[0 * BN + tl] = f16_to_f32((uint16_t)v.x);
        dx[1 * BN + tl] = f16_to_f32((uint16_t)(v.x >> 16));
        dx[2 * BN + tl] = f16_to_f32((uint16_t)v.y);
        dx[3 * BN + tl] = f16_to_f32((uint16_t)(v.y >> 16));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_DXFULL + s));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(BM, BN);
      for (int g = 0; g < G; ++g) {
        const int s = g % STAGES;
        if (!mbar_wait(bar(B_AREADY + s), (g / STAGES) & 1, abort_flag)) {
          fail();
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(smem + OFF_A + s * A_INT8_BYTES);
        const uint32_t b0 = smem_u32(smem + OFF_B + s * B_BYTES);
        bool ok = true;
        for (int j = 0; j < KBS; ++j) {
          if (!mbar_wait(bar(B_ACCEMPTY + j), (g & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          mma_i8(tmem_base + j * BN, smem_desc(a0 + 32 * j), smem_desc(b0 + 32 * j), idesc, 0);
          mma_commit(bar(B_ACCFULL + j));
        }
        if (!ok) {
          fail();
          break;
        }
        mma_commit(bar(B_SEMPTY + s));
      }
    }
  } else if (warp < EPI_WARP0) {
    // ---------------- nibble unpack ----------------
    const int u = threadIdx.x - 64;  // 0..63
    for (int g = 0; g < G; ++g) {
      const int s = g % STAGES;
      if (!mbar_wait_warp(bar(B_TMA + s), (g / STAGES) & 1, abort_flag)) {
        fail();
        break;
      }
      const uint4 *pack = reinterpret_cast<const uint4 *>(smem + OFF_PACK + s * A_PACK_BYTES);
      uint8_t *a = smem + OFF_A + s * A_INT8_BYTES;
#pragma unroll
      for (int i = 0; i < (BM * KBS) / 64; ++i) {
        const int idx = i * 64 + u;  // [tile(4)][block(4)][row(32)]
        const int r32 = idx & 31, blk = (idx >> 5) & 3, tile = idx >> 7;
        const int r = tile * 32 + r32;
        const uint4 w = pack[idx];
        const uint4 lo = make_uint4((w.x << 4) & 0xF0F0F0F0u, (w.y << 4) & 0xF0F0F0F0u,
                                    (w.z << 4) & 0xF0F0F0F0u, (w.w << 4) & 0xF0F0F0F0u);
        const uint4 hi = make_uint4(w.x & 0xF0F0F0F0u, w.y & 0xF0F0F0F0u, w.z & 0xF0F0F0F0u,
                                    w.w & 0xF0F0F0F0u);
        uint8_t *row = a + (r >> 3) * 1024 + (r & 7) * 128;
        *reinterpret_cast<uint4 *>(row + (((2 * blk) ^ (r & 7)) << 4)) = lo;
        *reinterpret_cast<uint4 *>(row + (((2 * blk + 1) ^ (r & 7)) << 4)) = hi;
      }
      fence_proxy_async();
      mbar_arrive(bar(B_AREADY + s));
    }
  } else {
    // ---------------- epilogue ----------------
    const int e = warp - EPI_WARP0;
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int hc = e >> 2;            // column half
    const int r = q * 32 + lane;      // tile row
    // Weight row and scale pointer of this thread.
    int n;
    const uint16_t *sc;
    if (SWIGLU) {
      n = blockIdx.x * 64 + (r & 63);
      sc = (r < 64 ? p.scl : p.scl2);
    } else {
      n = blockIdx.x * BM + r;
      sc = p.scl;
    }
    const uint16_t *scrow = sc + (size_t)(n >> 5) * KB * 32 + (n & 31);
    float acc[64];
    const float init = (!SWIGLU && p.bias) ? p.bias[n] : 0.0f;
#pragma unroll
    for (int c = 0; c < 64; ++c) acc[c] = init;
    bool ok = true;
    uint16_t dw_next = __ldg(scrow);
    for (int b = 0; b < KB && ok; ++b) {
      const int g = b / KBS, j = b % KBS, s = g % STAGES;
      const float dw16 = __fmul_rn(f16_to_f32(dw_next), 0.0625f);  // sums are 16*isum
      if (b + 1 < KB) dw_next = __ldg(scrow + (size_t)(b + 1) * 32);
      if (j == 0 && !mbar_wait_warp(bar(B_DXFULL + s), (g / STAGES) & 1, abort_flag)) {
        ok = false;
        break;
      }
      if (!mbar_wait_warp(bar(B_ACCFULL + j), g & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t d0[32], d1[32];
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + j * BN + hc * 64;
      tmem_ld32(taddr, d0);
      tmem_ld32(taddr + 32, d1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_ACCEMPTY + j));
      const float4 *dx4 =
          reinterpret_cast<const float4 *>(smem + OFF_DX + s * DX_BYTES) + (j * BN + hc * 64) / 4;
#pragma unroll
      for (int c4 = 0; c4 < 16; ++c4) {
        const float4 x = dx4[c4];
        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int c = c4 * 4 + k;
          const int iv = (int)(c < 32 ? d0[c] : d1[c - 32]);
          acc[c] = __fadd_rn(acc[c], __fmul_rn(__fmul_rn((float)iv, dw16), xs[k]));
        }
      }
      if (j == KBS - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_DXEMPTY + s));
      }
    }
    if (!ok && lane == 0) fail();
    if (!SWIGLU) {
      if (ok) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int t = t0 + hc * 64 + c;
          if (t < p.M) {
            const size_t o = (size_t)t * p.N + n;
            p.out[o] = p.resid ? __fadd_rn(p.resid[o], acc[c]) : acc[c];
          }
        }
      }
    } else {
      {
        // Up rows (lanes 64..127) hand their sums to the gate rows through smem
        // (the A ring is idle once every accumulator has been consumed).  Every
        // epilogue warp reaches the named barrier, aborted or not.
        float *xchg = reinterpret_cast<float *>(smem + OFF_A);  // [64 rows][BN]
        if (ok && q >= 2) {
#pragma unroll
          for (int c = 0; c < 64; ++c) xchg[(size_t)(r - 64) * BN + hc * 64 + c] = acc[c];
        }
        asm volatile("bar.sync 1, %0;" ::"r"(EPI_WARPS * 32));
        if (ok && !*abort_flag && q < 2) {
          const int I = p.N;
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const int t = t0 + hc * 64 + c;
            const float act = silu_mul(acc[c], xchg[(size_t)r * BN + hc * 64 + c]);
            uint16_t d16;
            const int8_t qv = q8_lane(act, d16);
            if (t < p.M) {
              const size_t o = (size_t)t * I + n;
              if (p.out) p.out[o] = act;
              p.act_qs[o] = qv;
              if (lane == 0) p.act_d[(size_t)t * (I / 32) + (n >> 5)] = d16;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// Row-tile SoA nibbles as a 4-D tensor: (16 bytes, 32 rows, KB blocks, N/32 tiles).
bool map_nibbles(CUtensorMap *m, const uint8_t *nib, int N, int KB, int tiles_per_box) {
  cuuint64_t dims[4] = {16, 32, (cuuint64_t)KB, (cuuint64_t)(N / 32)};
  cuuint64_t strides[3] = {16, 512, (cuuint64_t)KB * 512};
  cuuint32_t box[4] = {16, 32, (cuuint32_t)KBS, (cuuint32_t)tiles_per_box};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t *>(nib), dims,
                     strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// int8 activations [M][K] as 128-byte swizzled K-major boxes of (128 bytes, BN rows).
bool map_acts(CUtensorMap *m, const int8_t *xq, int M, int K) {
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {128, (cuuint32_t)BN};
  cuuint32_t es[2] = {1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(xq), dims, strides,
                     box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc

bool gemm_tc_supported(int N, int K, int M) {
  return M >= 1 && K % 128 == 0 && N % 128 == 0 && tc::encode_fn() != nullptr;
}

cudaError_t launch_gemm_tc(const GemvArgs &a, bool swiglu, cudaStream_t s) {
  using namespace tc;
  if (a.M <= 0) return cudaSuccess;
  if (!gemm_tc_supported(swiglu ? 2 * a.N : a.N, a.K, a.M) || (swiglu && a.N % 64))
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.xq) & 15) || (reinterpret_cast<uintptr_t>(a.nib) & 15) ||
      (reinterpret_cast<uintptr_t>(a.xd) & 7))
    return cudaErrorInvalidValue;
  CUtensorMap tmA, tmA2, tmB;
  const int KB = a.K / 32;
  if (!map_nibbles(&tmA, a.nib, a.N, KB, swiglu ? 2 : 4)) return cudaErrorInvalidValue;
  if (swiglu) {
    if (!map_nibbles(&tmA2, a.nib2, a.N, KB, 2)) return cudaErrorInvalidValue;
  } else {
    tmA2 = tmA;
  }
  if (!map_acts(&tmB, a.xq, a.M, a.K)) return cudaErrorInvalidValue;
  Params p{};
  p.N = a.N; p.K = a.K; p.M = a.M;
  p.scl = a.scl; p.scl2 = a.scl2; p.xd = a.xd; p.bias = a.bias; p.resid = a.resid;
  p.out = a.out; p.act_qs = a.act_qs; p.act_d = a.act_d; p.err = a.err;
  dim3 grid(swiglu ? a.N / 64 : a.N / BM, (a.M + BN - 1) / BN);
  auto kern = swiglu ? k_gemm_q4q8<true> : k_gemm_q4q8<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  kern<<<grid, THREADS, SMEM_BYTES, s>>>(tmA, tmA2, tmB, p);
  return cudaGetLastError();
}

}  // namespace si
