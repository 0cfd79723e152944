// gemm_tc.cu -- tcgen05 (sm_100a) Q4_0 x Q8_0 GEMM for prefill and batched decode.
//
// Reference semantics: matvec_q4q8 (qwen_one_layer.c:148-162) applied to every
// token, as the weight-stationary prefill does chunk by chunk on the K3
// (prefill_weight_stationary.h:94-106, 207-239): out[t][n] = bias[n], then for
// each 32-wide block b in order  out += ((float)isum(n,t,b) * dw[n,b]) * dx[t,b].
//
// Tile: 128 weight rows (TMEM lanes) x 128 tokens (TMEM columns).  Per K block
// one tcgen05.mma.kind::i8 (K = 32 = one Q4_0/Q8_0 block) writes the exact int32
// block sums of the whole tile into a TMEM accumulator; the epilogue warps
// rescale them in fp32 and add them to register accumulators in block order,
// so results are bit-identical to the reference's serial loop.  Four TMEM
// accumulators (512 columns) let the MMA run up to four blocks ahead of the
// rescale.
//
// Exact int -> float without a conversion instruction: after reading an
// accumulator each epilogue warp re-arms its part of it with tcgen05.st of the
// integer 0x4B400000 (the bits of C = 1.5 * 2^23), and the next MMA into it
// accumulates onto that, so every read-back is the float C + 16*isum (exact:
// |16*isum| < 2^22).  (Re-arming from shared memory with tcgen05.cp instead
// reads 64 KB of shared memory per block and measured 1.7x slower.)  The epilogue then needs three FP32 operations per (row, token,
// block) -- the floor for the reference's three roundings:
//   p   = (C + 16*isum) * dw/16 - C*dw/16   one packed FMA: round(isum*dw)
//   q   = p * dx                            one packed multiply, round-to-nearest
//   acc = acc + q                           one scalar add (a packed add after the
//                                           packed multiply is contracted by ptxas)
// A tolerance mode (`fused_rescale`) replaces the last two by one FMA, acc =
// fma(p, dx, acc): one rounding fewer per term (differences of order 2^-24 of a
// term, far inside the 1e-5 projection bar) for two FP32 operations per element.
//
// The kernel is persistent (one CTA per SM, tiles visited token-tile fastest)
// so the TMA / unpack / MMA / epilogue pipeline never drains between tiles.
//
// Warp roles (384 threads):
//   warp 0      TMA producer: packed Q4 nibbles and their fp16 scales, int8
//               activations (128-byte swizzle) and the stage's fp32
//               activation scales
//   warp 1      TMEM allocation; lane 0 issues the MMAs, two accumulator
//               commits and one stage commit per stage
//   warps 2-3   nibble unpack: Q4 -> signed int8 in the 128B-swizzled K-major
//               layout the MMA reads (byte = 16*(q-8), so sums are 16*isum)
//   warps 4-11  epilogue: warp w reads TMEM lane quarter w % 4 (32 rows) and
//               one half of the tile's tokens (64 columns, two 32-column
//               loads per block), re-arms it, rescales and accumulates in
//               registers, hands the accumulator back on an mbarrier, stores
//               per tile
// Stages hold 4 blocks (K = 128 bytes, one swizzle row) and are 4 deep.  Every
// wait is bounded (about 2 s); on expiry the kernel records SI_ERR_TIMEOUT in
// the context's error word, stops all roles, waits (bounded) for its own TMA
// loads and MMAs in flight, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "si_common.cuh"
#include "si_kernels.cuh"
#include "si_tc.cuh"
#include "si_tma.cuh"

namespace si {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int KBS = 4;                    // blocks per stage
constexpr int STAGES = 4;
constexpr int NACC = 4;                   // TMEM accumulators (= blocks per stage)
constexpr uint32_t TMEM_COLS = NACC * BN; // 512
constexpr int EPI_WARP0 = 4, EPI_WARPS = 8;
constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
constexpr int NC = BN * 4 / EPI_WARPS;    // 64 token columns per epilogue warp
constexpr uint32_t kMagic = 0x4B400000u;  // bits of 12582912.0f = 1.5 * 2^23
constexpr float kMagicF = 12582912.0f;

constexpr int A_INT8_BYTES = BM * 128;       // 16 KB, SW128 K-major
constexpr int B_BYTES = BN * 128;            // 16 KB, SW128 K-major (TMA swizzled)
constexpr int A_PACK_BYTES = BM * KBS * 16;  // 8 KB
constexpr int DX_BYTES = KBS * BN * 4;       // 2 KB
constexpr int SW_BYTES = BM * KBS * 2;       // 1 KB: weight scales [4 row tiles][4 blocks][32]
constexpr int XCHG_BYTES = 64 * BN * 4;      // SwiGLU up-row hand-off, 32 KB

constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_INT8_BYTES;
constexpr int OFF_PACK = OFF_B + STAGES * B_BYTES;
constexpr int OFF_DX = OFF_PACK + STAGES * A_PACK_BYTES;
constexpr int OFF_SW = OFF_DX + STAGES * DX_BYTES;
constexpr int OFF_XCHG = OFF_SW + STAGES * SW_BYTES;
constexpr int OFF_BAR = OFF_XCHG + XCHG_BYTES;
constexpr int NBAR = 4 * STAGES + 2 * NACC + 1;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;  // + alignment slack

static_assert(KBS == NACC, "one accumulator per block of a stage");
static_assert(NC == 64, "two 32-column TMEM loads per block and warp");
static_assert(OFF_B % 1024 == 0 && OFF_A % 1024 == 0, "alignment");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

struct Params {
  int N, K, M;              // rows (or gate rows for SwiGLU), inputs, tokens
  const uint16_t *scl, *scl2;
  int mtiles, ntiles;       // token tiles, total tiles (persistent schedule)
  const float *bias, *resid;
  float *out;
  int8_t *act_qs;
  uint16_t *act_d;
  int *err;
};

// 32 columns of this warp's 32 lanes set to v (tmem_fill32: four 8-column
// stores, so the value occupies 8 registers rather than 32).
__device__ __forceinline__ void tmem_fill32x(uint32_t taddr, uint32_t v) { tmem_fill32(taddr, v); }
// Bounded wait that ignores the abort flag: used on the way out of an aborted
// kernel for the CTA's own asynchronous copies and MMAs.
__device__ __forceinline__ bool mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_sleep(bar, parity))
    if (globaltimer() - t0 > 2000000000ull) return false;
  return true;
}

__device__ __forceinline__ void tmem_ld16r(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld16(taddr, r); }

// One 16-column chunk K of a block's rescale for this warp (columns 16K..16K+15
// of its 64).
template <bool FUSED, int K>
__device__ __forceinline__ void rescale16(float (&acc)[NC], const uint32_t (&v)[16],
                                          const float4 *dx4, float2 dw2, float2 nc2) {
#pragma unroll
  for (int c4 = 0; c4 < 4; ++c4) {
    const float4 x = dx4[K * 4 + c4];
    const float2 f0 = make_float2(__uint_as_float(v[4 * c4]), __uint_as_float(v[4 * c4 + 1]));
    const float2 f1 = make_float2(__uint_as_float(v[4 * c4 + 2]), __uint_as_float(v[4 * c4 + 3]));
    const float2 p0 = fma2_rn(f0, dw2, nc2), p1 = fma2_rn(f1, dw2, nc2);
    const int a = K * 16 + 4 * c4;
    if constexpr (FUSED) {
      const float2 s0 = fma2_rn(p0, make_float2(x.x, x.y), make_float2(acc[a], acc[a + 1]));
      const float2 s1 = fma2_rn(p1, make_float2(x.z, x.w), make_float2(acc[a + 2], acc[a + 3]));
      acc[a] = s0.x; acc[a + 1] = s0.y; acc[a + 2] = s1.x; acc[a + 3] = s1.y;
    } else {
      const float2 q0 = mul2_rn(p0, make_float2(x.x, x.y));
      const float2 q1 = mul2_rn(p1, make_float2(x.z, x.w));
      acc[a] = __fadd_rn(acc[a], q0.x);
      acc[a + 1] = __fadd_rn(acc[a + 1], q0.y);
      acc[a + 2] = __fadd_rn(acc[a + 2], q1.x);
      acc[a + 3] = __fadd_rn(acc[a + 3], q1.y);
    }
  }
}

// Bounded wait for the roles off the critical path (producer, unpack): between
// polls the warp sleeps, so it leaves the issue slots of its SM sub-partition
// to the epilogue warps that share it.
__device__ __forceinline__ bool mbar_wait_lazy_warp(uint32_t bar, uint32_t parity,
                                                    volatile int *abort) {
  bool ok = true;
  if (!mbar_try(bar, parity)) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try(bar, parity)) {
      __nanosleep(200);
      if (*abort || globaltimer() - t0 > 2000000000ull) {
        ok = false;
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, ok) != 0;
}

// (__launch_bounds__ without a minimum-blocks hint: with the hint ptxas
// schedules for 168 registers and spills; without it it needs 138.)
template <bool SWIGLU, bool FUSED>
__global__ void __launch_bounds__(THREADS)
    k_gemm_q4q8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmD,
                const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmS2,
                const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<1024>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = p.K / 32;
  const int G = KB / KBS;  // stages per tile

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  // tma_full[s]: packed A, B and the scales of stage s landed; a_ready[s]: A
  // unpacked; stage_empty[s]: the stage's MMAs finished; dx_empty[s]: every
  // epilogue warp is done with the stage's scales; acc_full[h]: accumulators
  // 2h and 2h+1 hold blocks 2h and 2h+1 of a stage (two commits per stage: an
  // mbarrier wait costs a few hundred cycles even when already complete, and
  // the epilogue starting block 2 never waits on the MMA that its release of
  // accumulator 3 a stage earlier unblocked); acc_empty[j]: every epilogue
  // warp has read accumulator j; final: the MMA thread's last tcgen05
  // operations completed.
  const int B_TMA = 0, B_AREADY = STAGES, B_SEMPTY = 2 * STAGES, B_DXEMPTY = 3 * STAGES,
            B_ACCFULL = 4 * STAGES, B_ACCEMPTY = 4 * STAGES + NACC,
            B_FINAL = 4 * STAGES + 2 * NACC;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC + 16);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar(B_TMA + s), 1);
      mbar_init(bar(B_AREADY + s), 64);
      mbar_init(bar(B_SEMPTY + s), 1);
      mbar_init(bar(B_DXEMPTY + s), EPI_WARPS);
    }
    for (int j = 0; j < NACC; ++j) {
      mbar_init(bar(B_ACCFULL + j), 1);  // only the first two are used
      mbar_init(bar(B_ACCEMPTY + j), EPI_WARPS);
    }
    mbar_init(bar(B_FINAL), 1);
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
  // Persistent schedule: tiles are visited token-tile fastest, so the CTAs in
  // flight share each weight tile through L2 while it streams from HBM once.
  const int tiles_per_row = SWIGLU ? 2 : 4;  // 32-row tiles of each weight matrix per CTA tile

  if (warp == 0) {
    // ---------------- producer ----------------
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x) {
      const int nt = tile / p.mtiles, t0 = (tile % p.mtiles) * BN;
      for (int g = 0; g < G; ++g) {
        const int s = it % STAGES;
        const uint32_t ph = ((it / STAGES) & 1) ^ 1;
        if (!mbar_wait_lazy_warp(bar(B_SEMPTY + s), ph, abort_flag) ||
            !mbar_wait_lazy_warp(bar(B_DXEMPTY + s), ph, abort_flag)) {
          if (lane == 0) fail();
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t full = bar(B_TMA + s);
          mbar_expect_tx(full, A_PACK_BYTES + B_BYTES + DX_BYTES + SW_BYTES);
          const uint32_t pack = smem_u32(smem + OFF_PACK + s * A_PACK_BYTES);
          tma_load_2d(pack, &tmA, g * 256, nt * tiles_per_row, full);
          if (SWIGLU) tma_load_2d(pack + A_PACK_BYTES / 2, &tmA2, g * 256, nt * 2, full);
          tma_load_2d(smem_u32(smem + OFF_B + s * B_BYTES), &tmB, g * 128, t0, full);
          tma_load_2d(smem_u32(smem + OFF_DX + s * DX_BYTES), &tmD, t0, g * KBS, full);
          const uint32_t sw = smem_u32(smem + OFF_SW + s * SW_BYTES);
          tma_load_2d(sw, &tmS, g * 128, nt * tiles_per_row, full);
          if (SWIGLU) tma_load_2d(sw + SW_BYTES / 2, &tmS2, g * 128, nt * 2, full);
        }
        ++it;
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      // Let the loads this warp issued land before the CTA can exit.
      for (int k = it > STAGES ? it - STAGES : 0; k < it; ++k)
        mbar_drain(bar(B_TMA + k % STAGES), (k / STAGES) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(BM, BN);
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x) {
        for (int g = 0; g < G; ++g, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(bar(B_AREADY + s), (it / STAGES) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + OFF_A + s * A_INT8_BYTES);
          const uint32_t b0 = smem_u32(smem + OFF_B + s * B_BYTES);
          for (int j = 0; j < KBS; ++j) {
            // Use number `it` of accumulator j needs every epilogue warp to
            // have read and re-armed its previous block (it + 1 completions,
            // counting the initial one).
            if (!mbar_wait(bar(B_ACCEMPTY + j), it & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            mma_i8(tmem_base + j * BN, smem_desc(a0 + 32 * j), smem_desc(b0 + 32 * j), idesc, 1);
            if (j % 2 == 1) mma_commit(bar(B_ACCFULL + j / 2));
          }
          if (!ok) break;
          mma_commit(bar(B_SEMPTY + s));
        }
      }
      if (!ok) fail();
      // Every tcgen05 operation this thread issued has completed before TMEM
      // can be freed.
      mma_commit(bar(B_FINAL));
      mbar_drain(bar(B_FINAL), 0);
    }
    __syncwarp();
  } else if (warp < EPI_WARP0) {
    // ---------------- nibble unpack ----------------
    const int u = threadIdx.x - 64;  // 0..63
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x) {
      for (int g = 0; g < G; ++g, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait_lazy_warp(bar(B_TMA + s), (it / STAGES) & 1, abort_flag)) {
          if (lane == 0) fail();
          ok = false;
          break;
        }
        const uint4 *pack = reinterpret_cast<const uint4 *>(smem + OFF_PACK + s * A_PACK_BYTES);
        uint8_t *a = smem + OFF_A + s * A_INT8_BYTES;
#pragma unroll 4
        for (int i = 0; i < (BM * KBS) / 64; ++i) {
          const int idx = i * 64 + u;  // [tile(4)][block(4)][row(32)] x 16 bytes
          const int r32 = idx & 31, blk = (idx >> 5) & 3, tl = idx >> 7;
          const int r = tl * 32 + r32;
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
    }
  } else {
    // ---------------- epilogue ----------------
    const int e = warp - EPI_WARP0;
    const int q = warp & 3;       // TMEM lane quarter this warp may access
    const int hc = e >> 2;        // token half of the tile
    const int r = q * 32 + lane;  // tile row
    const uint32_t tcol = tmem_base + ((uint32_t)(q * 32) << 16) + hc * NC;
    // Every accumulator starts armed and free.
    for (int j = 0; j < NACC; ++j) {
      tmem_fill32x(tcol + j * BN, kMagic);
      tmem_fill32x(tcol + j * BN + 32, kMagic);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int j = 0; j < NACC; ++j) mbar_arrive(bar(B_ACCEMPTY + j));
    // SwiGLU hand-off, [token column][row]: consecutive lanes, consecutive
    // words.  Gate warp (q, hc) and up warp (q + 2, hc) hold the same 32
    // intermediate rows and 64 tokens; each hands the other one half of its
    // columns, so both share the activation and Q8 work.
    float *xchg = reinterpret_cast<float *>(smem + OFF_XCHG);
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
      const int nt = tile / p.mtiles, t0 = (tile % p.mtiles) * BN;
      const int n = SWIGLU ? nt * 64 + (r & 63) : nt * BM + r;
      float acc[NC];
      const float init = (!SWIGLU && p.bias) ? p.bias[n] : 0.0f;
#pragma unroll
      for (int c = 0; c < NC; ++c) acc[c] = init;
      // Software pipeline over the tile's blocks in 16-column chunks: the
      // TMEM load of the next chunk is always in flight while the current one
      // is rescaled (va / vb alternate).  The four blocks of a stage are
      // unrolled, so every TMEM, scale and dx offset is a constant.
      uint32_t va[16], vb[16];
      if (!mbar_wait2_warp(bar(B_TMA + it % STAGES), (it / STAGES) & 1, bar(B_ACCFULL), it & 1,
                           abort_flag))
        ok = false;
      if (ok) {
        tc_fence_after();
        tmem_ld16r(tcol, va);
      }
#pragma unroll 1
      for (int g = 0; ok && g < G; ++g) {
        const int itg = it + g, s = itg % STAGES;
        const uint16_t *swp = reinterpret_cast<const uint16_t *>(smem + OFF_SW + s * SW_BYTES) +
                              (r >> 5) * KBS * 32 + lane;
        const float4 *dxs = reinterpret_cast<const float4 *>(smem + OFF_DX + s * DX_BYTES) +
                            hc * NC / 4;
#pragma unroll
        for (int j = 0; j < KBS; ++j) {
          // (C + D) * dw/16 - C * dw/16 = isum * dw in one rounding: C*dw/16
          // is exact (dw has 11 significant bits, C/16 = 3*2^18).
          const float dw16 = __fmul_rn(f16_to_f32(swp[j * 32]), 0.0625f);
          const float ncdw = -__fmul_rn(kMagicF, dw16);
          const float2 dw2 = make_float2(dw16, dw16), nc2 = make_float2(ncdw, ncdw);
          const float4 *dx4 = dxs + j * BN / 4;
          const uint32_t ta = tcol + j * BN;
          tmem_wait_ld();               // va: chunk 0
          tmem_ld16r(ta + 16, vb);
          rescale16<FUSED, 0>(acc, va, dx4, dw2, nc2);
          tmem_wait_ld();               // vb: chunk 1
          tmem_ld16r(ta + 32, va);
          rescale16<FUSED, 1>(acc, vb, dx4, dw2, nc2);
          tmem_wait_ld();               // va: chunk 2
          tmem_ld16r(ta + 48, vb);
          rescale16<FUSED, 2>(acc, va, dx4, dw2, nc2);
          tmem_wait_ld();               // vb: chunk 3 -- the whole block is read
          // Re-arm this warp's part of the accumulator, then start the next
          // block's first chunk.
          tmem_fill32x(ta, kMagic);
          tmem_fill32x(ta + 32, kMagic);
          bool next = j + 1 < KBS || g + 1 < G;
          if (j == 1) {
            if (!mbar_wait_warp(bar(B_ACCFULL + 1), itg & 1, abort_flag)) ok = next = false;
          } else if (j == KBS - 1 && next) {  // a new stage: its scales and first two blocks
            const int itn = itg + 1;
            if (!mbar_wait2_warp(bar(B_TMA + itn % STAGES), (itn / STAGES) & 1, bar(B_ACCFULL),
                                 itn & 1, abort_flag))
              ok = next = false;
          }
          if (next) {
            tc_fence_after();
            tmem_ld16r(tcol + ((j + 1) % KBS) * BN, va);
          }
          rescale16<FUSED, 3>(acc, vb, dx4, dw2, nc2);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B_ACCEMPTY + j));
        }
        if (lane == 0) mbar_arrive(bar(B_DXEMPTY + s));
      }
      tmem_wait_ld();  // nothing may be left in flight (an aborted prefetch)
      it += G;
      if (!ok && lane == 0) fail();
      if (!SWIGLU) {
        if (!ok) break;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const int t = t0 + hc * NC + c;
          if (t < p.M) {
            const size_t o = (size_t)t * p.N + n;
            p.out[o] = p.resid ? __fadd_rn(p.resid[o], acc[c]) : acc[c];
          }
        }
      } else {
        // Gate warps (q < 2) pass columns 32..63 of their gate sums, up warps
        // columns 0..31 of their up sums; every epilogue warp reaches both
        // named barriers, aborted or not.
        const bool gate = q < 2;
        float *xg = xchg + hc * (2 * 32 * 64);  // [gate sums 32 cols][up sums 32 cols] x 64 rows
        const int rr = r & 63;
        if (ok) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            if (gate) xg[c * 64 + rr] = acc[32 + c];
            else xg[(32 + c) * 64 + rr] = acc[c];
          }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(EPI_WARPS * 32));
        if (ok && !*abort_flag) {
          const int I = p.N;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            // gate warps: columns 0..31 (own gate, partner's up);
            // up warps: columns 32..63 (partner's gate, own up).
            const float gv = gate ? acc[c] : xg[c * 64 + rr];
            const float uv = gate ? xg[(32 + c) * 64 + rr] : acc[32 + c];
            const int t = t0 + hc * NC + (gate ? c : 32 + c);
            const float act = silu_mul(gv, uv);
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
        asm volatile("bar.sync 1, %0;" ::"r"(EPI_WARPS * 32));  // xchg free for the next tile
        if (!ok || *abort_flag) break;
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

// Activation scales fp16 [M][KB] -> fp32 [KB][Mp] (Mp = M rounded up to 4, zero
// padded): the layout the GEMM's TMA loads per stage.
__global__ void k_scales_t(const uint16_t *__restrict__ xd, int M, int KB, int Mp,
                           float *__restrict__ dT) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
  if (t < Mp) dT[(size_t)b * Mp + t] = t < M ? f16_to_f32(xd[(size_t)t * KB + b]) : 0.0f;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
}  // namespace tc

cudaError_t launch_scales_t(const uint16_t *xd, int M, int KB, float *dT, cudaStream_t s) {
  const int Mp = (M + 3) & ~3;
  return launch_pdl(tc::k_scales_t, dim3((Mp + 127) / 128, KB), dim3(128), 0, s, xd, M, KB, Mp, dT);
}

bool gemm_tc_supported(int N, int K, int M) {
  return M >= 1 && K % 128 == 0 && N % 128 == 0 && tma_encode_fn() != nullptr;
}

size_t gemm_tc_scratch_bytes(int K, int M) {
  return (size_t)(K / 32) * ((M + 3) & ~3) * sizeof(float);
}

cudaError_t launch_gemm_tc(const GemvArgs &a, bool swiglu, cudaStream_t s) {
  using namespace tc;
  if (a.M <= 0) return cudaSuccess;
  if (!gemm_tc_supported(swiglu ? 2 * a.N : a.N, a.K, a.M) || (swiglu && a.N % 64) || !a.scratch)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.xq) & 15) || (reinterpret_cast<uintptr_t>(a.nib) & 15) ||
      (reinterpret_cast<uintptr_t>(a.scratch) & 15) || (reinterpret_cast<uintptr_t>(a.scl) & 15) ||
      (swiglu && ((reinterpret_cast<uintptr_t>(a.nib2) & 15) ||
                  (reinterpret_cast<uintptr_t>(a.scl2) & 15))))
    return cudaErrorInvalidValue;
  const int KB = a.K / 32, Mp = (a.M + 3) & ~3;
  float *dT = a.scratch;
  cudaError_t e = launch_pdl(k_scales_t, dim3((Mp + 127) / 128, KB), dim3(128), 0, s,
                             (const uint16_t *)a.xd, a.M, KB, Mp, dT);
  if (e != cudaSuccess) return e;

  CUtensorMap tmA, tmA2, tmB, tmD, tmS, tmS2;
  // Nibbles of a 32-row tile are contiguous over K ([KB][32][16] bytes): a 2-D view
  // of 8-byte elements, (KB*64, rows/32), box = 4 blocks x (4 or 2) row-tiles.
  const int rt = a.N / 32, per = swiglu ? 2 : 4;
  cuuint64_t dA[2] = {(cuuint64_t)KB * 64, (cuuint64_t)rt};
  cuuint64_t sA[1] = {(cuuint64_t)KB * 512};
  cuuint32_t bA[2] = {256, (cuuint32_t)per};
  if (!tma_encode(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, a.nib, dA, sA, bA,
              CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  if (swiglu) {
    if (!tma_encode(&tmA2, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, a.nib2, dA, sA, bA,
                CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  } else {
    tmA2 = tmA;
  }
  cuuint64_t dB[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
  cuuint64_t sB[1] = {(cuuint64_t)a.K};
  cuuint32_t bB[2] = {128, (cuuint32_t)BN};
  if (!tma_encode(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a.xq, dB, sB, bB,
              CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  cuuint64_t dD[2] = {(cuuint64_t)Mp, (cuuint64_t)KB};
  cuuint64_t sD[1] = {(cuuint64_t)Mp * 4};
  cuuint32_t bD[2] = {(cuuint32_t)BN, (cuuint32_t)KBS};
  if (!tma_encode(&tmD, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dT, dD, sD, bD,
              CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  // Weight scales [rows/32][KB][32] fp16 as a 2-D view (KB*32, rows/32); box =
  // 4 blocks x (4 or 2) row tiles, matching the nibble box.
  cuuint64_t dS[2] = {(cuuint64_t)KB * 32, (cuuint64_t)rt};
  cuuint64_t sS[1] = {(cuuint64_t)KB * 64};
  cuuint32_t bS[2] = {128, (cuuint32_t)per};
  if (!tma_encode(&tmS, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.scl, dS, sS, bS,
              CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  if (swiglu) {
    if (!tma_encode(&tmS2, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.scl2, dS, sS, bS,
                CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  } else {
    tmS2 = tmS;
  }

  // SM count of the device this launch targets (the caller made it current).
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return cudaErrorInvalidDevice;
  Params p{};
  p.N = a.N; p.K = a.K; p.M = a.M;
  p.scl = a.scl; p.scl2 = a.scl2; p.bias = a.bias; p.resid = a.resid;
  p.out = a.out; p.act_qs = a.act_qs; p.act_d = a.act_d; p.err = a.err;
  p.mtiles = (a.M + BN - 1) / BN;
  p.ntiles = (swiglu ? a.N / 64 : a.N / BM) * p.mtiles;
  const int grid = p.ntiles < sms ? p.ntiles : sms;
  auto kern = swiglu ? (a.fused_rescale ? k_gemm_q4q8<true, true> : k_gemm_q4q8<true, false>)
                     : (a.fused_rescale ? k_gemm_q4q8<false, true> : k_gemm_q4q8<false, false>);
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  count_launch();
  kern<<<grid, THREADS, SMEM_BYTES, s>>>(tmA, tmA2, tmB, tmD, tmS, tmS2, p);
  return cudaGetLastError();
}

}  // namespace si
