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
// rescale.  The accumulators are pre-set to the integer 0x4B400000 and the MMA
// accumulates onto it, so each read-back is already the float C + 16*isum; one
// exact FMA per element folds that into round(isum*dw), then a
// round-to-nearest multiply by dx (packed in pairs) and a scalar add keep the
// reference's rounding.
//
// The kernel is persistent (one CTA per SM, tiles visited token-tile fastest)
// so the TMA / unpack / MMA / epilogue pipeline never drains between tiles.
//
// Warp roles (640 threads):
//   warp 0      TMA producer: packed Q4 nibbles and their fp16 scales, int8
//               activations (128-byte swizzle) and the stage's fp32
//               activation scales
//   warp 1      TMEM allocation; lane 0 issues the MMAs, one commit per stage
//   warps 2-3   nibble unpack: Q4 -> signed int8 in the 128B-swizzled K-major
//               layout the MMA reads (byte = 16*(q-8), so sums are 16*isum)
//   warps 4-19  epilogue (4 per TMEM lane quarter, 32 columns each, read in
//               double-buffered 8-column chunks): TMEM -> registers, rescale,
//               accumulate, re-arm, store
// Stages hold 4 blocks (K = 128 bytes, one swizzle row) and are 4 deep.  The
// epilogue hands each accumulator back to the MMA issuer on an mbarrier.  Every wait is
// bounded (about 2 s); on expiry the kernel records SI_ERR_TIMEOUT in the
// context's error word, stops all roles, frees its TMEM and returns.
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
constexpr int EPI_WARP0 = 4, EPI_WARPS = 16;
constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
constexpr uint32_t kMagic = 0x4B400000u;  // bits of 12582912.0f = 1.5 * 2^23
constexpr float kMagicF = 12582912.0f;

constexpr int A_INT8_BYTES = BM * 128;       // 16 KB, SW128 K-major
constexpr int B_BYTES = BN * 128;            // 16 KB, SW128 K-major (TMA swizzled)
constexpr int A_PACK_BYTES = BM * KBS * 16;  // 8 KB
constexpr int DX_BYTES = KBS * BN * 4;       // 2 KB
constexpr int SW_BYTES = BM * KBS * 2;       // 1 KB: weight scales [4 row tiles][4 blocks][32]

constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_INT8_BYTES;
constexpr int OFF_PACK = OFF_B + STAGES * B_BYTES;
constexpr int OFF_DX = OFF_PACK + STAGES * A_PACK_BYTES;
constexpr int XCHG_BYTES = 64 * BN * 4;      // SwiGLU up-row hand-off, 32 KB
constexpr int OFF_SW = OFF_DX + STAGES * DX_BYTES;
constexpr int OFF_XCHG = OFF_SW + STAGES * SW_BYTES;
constexpr int OFF_BAR = OFF_XCHG + XCHG_BYTES;
constexpr int NBAR = 4 * STAGES + 2 * NACC + NACC;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;  // + alignment slack

static_assert(KBS == NACC, "one accumulator per block of a stage");

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

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// Columns per epilogue warp: the 4 TMEM lane quarters x (EPI_WARPS / 4) slices.
constexpr int NC = BN * 4 / EPI_WARPS;
constexpr int CW = 8;         // columns per TMEM load chunk
constexpr int NCH = NC / CW;  // chunks per block
static_assert(NCH >= 2 && NCH % 2 == 0, "chunk double-buffering needs an even chunk count");

// One CW-column chunk h of the rescale: acc[h*CW + c] += ((C+D)*dw16 - C*dw16) * dx.
// The fold is a packed FMA (exact, see above) and the product a packed
// multiply; the sum stays scalar so product and sum keep the reference's
// separate roundings.
__device__ __forceinline__ void rescale(float (&acc)[NC], int h, const uint32_t (&d)[CW],
                                        const float4 *dx4, float2 dw2, float2 nc2) {
#pragma unroll
  for (int c4 = 0; c4 < CW / 4; ++c4) {
    const float4 x = dx4[h * (CW / 4) + c4];
    const float2 f0 = make_float2(__uint_as_float(d[4 * c4]), __uint_as_float(d[4 * c4 + 1]));
    const float2 f1 = make_float2(__uint_as_float(d[4 * c4 + 2]), __uint_as_float(d[4 * c4 + 3]));
    const float2 p0 = fma2_rn(f0, dw2, nc2), p1 = fma2_rn(f1, dw2, nc2);
    const int a = h * CW + 4 * c4;
    // Packed product, scalar sum: with both packed, ptxas fuses them into one
    // packed FMA (a single rounding) despite the explicit .rn -- measured here;
    // either one packed alone keeps both roundings.
    const float2 q0 = mul2_rn(p0, make_float2(x.x, x.y)), q1 = mul2_rn(p1, make_float2(x.z, x.w));
    acc[a] = __fadd_rn(acc[a], q0.x);
    acc[a + 1] = __fadd_rn(acc[a + 1], q0.y);
    acc[a + 2] = __fadd_rn(acc[a + 2], q1.x);
    acc[a + 3] = __fadd_rn(acc[a + 3], q1.y);
  }
}

template <bool SWIGLU>
__global__ void __launch_bounds__(THREADS, 1)
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
  // tma_full: packed A + B + activation scales landed; a_ready: A unpacked;
  // stage_empty: the MMAs of the stage finished; dx_empty: the epilogue used
  // the stage's scales; acc_full[h]: accumulators 2h and 2h+1 of a stage
  // written (two commits per stage, so the epilogue starting a stage never
  // waits on the MMA that the release of its last accumulator unblocks);
  // acc_empty[j]: every epilogue warp re-armed accumulator j (the MMA thread
  // sleeps in try_wait rather than polling, so no issue slots go to waiting).
  const int B_TMA = 0, B_AREADY = STAGES, B_SEMPTY = 2 * STAGES, B_DXEMPTY = 3 * STAGES,
            B_ACCFULL = 4 * STAGES, B_ACCEMPTY = 4 * STAGES + 2 * NACC;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC + 16);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar(B_TMA + s), 1);
      mbar_init(bar(B_AREADY + s), 64);
      mbar_init(bar(B_SEMPTY + s), 1);
      mbar_init(bar(B_DXEMPTY + s), EPI_WARPS);
    }
    mbar_init(bar(B_ACCFULL), 1);
    mbar_init(bar(B_ACCFULL + 1), 1);
    for (int j = 0; j < NACC; ++j) mbar_init(bar(B_ACCEMPTY + j), EPI_WARPS);
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
      for (int g = 0; g < G; ++g, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = ((it / STAGES) & 1) ^ 1;
        if (!mbar_wait2_warp(bar(B_SEMPTY + s), ph, bar(B_DXEMPTY + s), ph, abort_flag)) {
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
        __syncwarp();
      }
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
          for (int j = 0; j < KBS && ok; ++j) {
            // Use number `it` of accumulator j needs the epilogue to have
            // (re)armed it with the magic constant it+1 times (each of its warps).
            if (!mbar_wait(bar(B_ACCEMPTY + j), it & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            mma_i8(tmem_base + j * BN, smem_desc(a0 + 32 * j), smem_desc(b0 + 32 * j), idesc, 1);
            // Phase `it` of acc_full[h]: block sums 2h and 2h+1 of the stage are in TMEM.
            if (j % 2 == 1) mma_commit(bar(B_ACCFULL + j / 2));
          }
          if (!ok) break;
          mma_commit(bar(B_SEMPTY + s));
        }
      }
      if (!ok) fail();
    }
  } else if (warp < EPI_WARP0) {
    // ---------------- nibble unpack ----------------
    const int u = threadIdx.x - 64;  // 0..63
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x) {
      for (int g = 0; g < G; ++g, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait_warp(bar(B_TMA + s), (it / STAGES) & 1, abort_flag)) {
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
    // Warp e: lane quarter q = warp % 4, column slice hc = e / 4 (NC columns).
    // Each warp walks its columns of every block in CW-column chunks,
    // software-pipelined: the TMEM load of chunk k+1 is in flight while chunk k
    // is rescaled, and the accumulator's re-arm store overlaps the last chunk.
    const int e = warp - EPI_WARP0;
    const int q = warp & 3;       // TMEM lane quarter this warp may access
    const int hc = e >> 2;        // column slice of the tile
    const int r = q * 32 + lane;  // tile row
    const uint32_t tcol = tmem_base + ((uint32_t)(q * 32) << 16) + hc * NC;
    // Accumulators hold C + 16*isum as float bits: the MMA accumulates onto the
    // integer 0x4B400000 (C = 1.5*2^23 as a float), so C + D is an exactly
    // representable float in [2^23, 2^24) and no int->float conversion is needed.
    for (int j = 0; j < NACC; ++j)
      for (int f = 0; f < NC / 32; ++f) tmem_fill32(tcol + j * BN + 32 * f, kMagic);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int j = 0; j < NACC; ++j) mbar_arrive(bar(B_ACCEMPTY + j));
    float *xchg = reinterpret_cast<float *>(smem + OFF_XCHG);  // [64 rows][BN]
    int pending = -1;  // accumulator re-armed but not yet handed back to the MMA
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
      const int nt = tile / p.mtiles, t0 = (tile % p.mtiles) * BN;
      const int n = SWIGLU ? nt * 64 + (r & 63) : nt * BM + r;
      float acc[NC];
      const float init = (!SWIGLU && p.bias) ? p.bias[n] : 0.0f;
#pragma unroll
      for (int c = 0; c < NC; ++c) acc[c] = init;
      const int it0 = it;  // stage counter at the tile's first block
      uint32_t dbuf[2][CW];
      // Prime: block 0 of the tile, chunk 0.
      if (!mbar_wait2_warp(bar(B_TMA + it0 % STAGES), (it0 / STAGES) & 1, bar(B_ACCFULL),
                           it0 & 1, abort_flag))
        ok = false;
      if (ok) {
        tc_fence_after();
        tmem_ld<CW>(tcol, dbuf[0]);
        tmem_wait_ld();
      }
      for (int b = 0; ok && b < KB; ++b) {
        const int j = b % KBS, itb = it0 + b / KBS, s = itb % STAGES;
        // This row's scale of block b, staged by TMA with the stage's tiles
        // ([row tile][block][32 rows] fp16; SwiGLU: gate tiles 0-1, up tiles 2-3).
        const uint16_t dw_cur = reinterpret_cast<const uint16_t *>(
            smem + OFF_SW + s * SW_BYTES)[((r >> 5) * KBS + j) * 32 + lane];
        // (C + D) * dw/16 - C * dw/16 = isum * dw in one rounding: C*dw/16 is exact
        // (dw has 11 significant bits, C/16 = 3*2^18), so this equals the
        // reference's (float)isum * dw.
        const float dw16 = __fmul_rn(f16_to_f32(dw_cur), 0.0625f);
        const float ncdw = -__fmul_rn(kMagicF, dw16);
        const float2 dw2 = make_float2(dw16, dw16), nc2 = make_float2(ncdw, ncdw);
        const float4 *dx4 = reinterpret_cast<const float4 *>(smem + OFF_DX + s * DX_BYTES) +
                            (j * BN + hc * NC) / 4;
        const uint32_t ta = tcol + j * BN;
        bool more = b + 1 < KB;
#pragma unroll
        for (int h = 0; h < NCH; ++h) {  // dbuf[h & 1] holds chunk h on entry
          if (h + 1 < NCH) {
            tmem_ld<CW>(ta + (h + 1) * CW, dbuf[(h + 1) & 1]);
          } else {
            // Every chunk of block b is in registers.  Hand back the accumulator
            // re-armed one block ago (its store has long completed, so this wait
            // is short), then re-arm this one and start block b+1 (next
            // accumulator, maybe next stage) into dbuf[0].
            if (pending >= 0) {
              tmem_wait_st();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(bar(B_ACCEMPTY + pending));
            }
#pragma unroll
            for (int f = 0; f < NC / 32; ++f) tmem_fill32(ta + 32 * f, kMagic);
            pending = j;
            // Blocks 2-3 of a stage are committed together; the MMAs behind that
            // commit needed only releases made before this point.
            if (more && j == KBS / 2 - 1 &&
                !mbar_wait_warp(bar(B_ACCFULL + 1), itb & 1, abort_flag)) {
              ok = false;
              more = false;
            }
            if (more && j != KBS - 1) {
              tc_fence_after();
              tmem_ld<CW>(tcol + (j + 1) * BN, dbuf[0]);
            }
          }
          rescale(acc, h, dbuf[h & 1], dx4, dw2, nc2);
          if (h + 1 < NCH) tmem_wait_ld();
        }
        if (j == KBS - 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B_DXEMPTY + s));
          if (more) {
            // A new stage: its scales and its first two block sums (their
            // accumulators were released during blocks 1 and 2 of this stage).
            const int it1 = itb + 1;
            if (!mbar_wait2_warp(bar(B_TMA + it1 % STAGES), (it1 / STAGES) & 1, bar(B_ACCFULL),
                                 it1 & 1, abort_flag)) {
              ok = false;
              more = false;
            } else {
              tc_fence_after();
              tmem_ld<CW>(tcol, dbuf[0]);
            }
          }
        }
        if (more) tmem_wait_ld();
      }
      it = it0 + G;
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
        // Up rows (lanes 64..127) hand their sums to the gate rows.  Every
        // epilogue warp reaches both named barriers, aborted or not.
        if (ok && q >= 2) {
#pragma unroll
          for (int c = 0; c < NC; ++c) xchg[(size_t)(r - 64) * BN + hc * NC + c] = acc[c];
        }
        asm volatile("bar.sync 1, %0;" ::"r"(EPI_WARPS * 32));
        if (ok && !*abort_flag && q < 2) {
          const int I = p.N;
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            const int t = t0 + hc * NC + c;
            const float act = silu_mul(acc[c], xchg[(size_t)r * BN + hc * NC + c]);
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
    tmem_wait_st();  // the last re-arm completes before TMEM is freed
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
  auto kern = swiglu ? k_gemm_q4q8<true> : k_gemm_q4q8<false>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  count_launch();
  kern<<<grid, THREADS, SMEM_BYTES, s>>>(tmA, tmA2, tmB, tmD, tmS, tmS2, p);
  return cudaGetLastError();
}

}  // namespace si
