// attention_tc.cu -- causal prefill attention on the tcgen05 tensor cores.
//
// Same function as the prefill path of attention.cu (attention_flash,
// attention_kernels.h:80-164, applied to query token t of a prefill with
// context prefix + t + 1, prefill_weight_stationary.h:173-177): per head h with
// KV group g = h / (Hq/Hkv), softmax over the keys of (q . k) / sqrt(D), times V.
//
// Precision.  The score and P.V contractions run as fp16 MMAs with fp32
// accumulation on split operands: every fp32 input x is carried as
// hi = fp16(x), lo = fp16(x - hi) (22 significant bits together), and a product
// a.b is formed as a_hi.b_hi + a_hi.b_lo + a_lo.b_hi -- the dropped lo.lo term
// is below 2^-22 of it.  K and V from an fp16 cache are exact in one half, so
// their lo parts (and the MMAs with them) are skipped.  The result agrees with
// the fp32 kernel of attention.cu to about 1e-6 relative, not bit for bit; the
// context option that asks for exact attention selects that kernel instead.
//
// Layout.  Pre-pass kernels write the splits: Q scaled by log2(e)/sqrt(D) (so
// scores come out in log2 units for exp2) as [T][Hq][D] halves, K as
// [Hkv][Lp][D] and V transposed as [Hkv][D][Lp] (Lp = the context rounded up
// to 64 keys, zero padded), so every MMA operand is a K-major tile that TMA
// loads with the 128-byte swizzle.  One CTA takes 128 query rows -- TQ tokens
// x the G heads of one KV group, so each K/V tile serves all G heads -- and
// walks the keys in tiles of 64:
//   S  = Q.K^T        TMEM, 128 x 64 fp32, double-buffered (the next tile's
//                     scores are computed while this one's softmax runs)
//   P  = exp2(S - m)  softmax warps, one row per thread, written to shared
//                     memory as fp16 hi/lo in the swizzled K-major layout
//   O += P.V          TMEM, 128 x 128 fp32, restarted every kWindow tiles:
//                     the softmax warps add each finished window into a
//                     second TMEM accumulator with fp32 adds, so the tensor
//                     core's accumulation error is bounded by one window's
//                     MMAs (measured 1.5e-4 relative at 32768 keys without
//                     the windows) and stays flat with the context length
// The running max m is only raised (and O and the row sum rescaled) when a
// tile's max exceeds it by more than 2^8, so P stays below 256 and the rescale
// -- a read-modify-write of the O rows -- is rare after the first tile.
//
// Warp roles (192 threads): warp 0 TMA producer; warp 1 TMEM allocation and
// MMA issue (one thread); warps 2-5 softmax, one per TMEM lane quarter, then
// the epilogue O / l.  Every wait is bounded (about 2 s; SI_ERR_TIMEOUT in the
// context's error word); on expiry every role stops, the CTA's own TMA loads
// and MMAs in flight are waited for (bounded) and TMEM is freed.
#include "si_common.cuh"
#include "si_kernels.cuh"
#include "si_tc.cuh"
#include "si_tma.cuh"

namespace si {
namespace atc {
using namespace si::tc;

constexpr int D = 128;
constexpr int BK = 64;                    // keys per tile
constexpr int ROWS = 128;                 // query rows per CTA
constexpr int STAGES = 2;
constexpr int THREADS = 192;
constexpr float kRescaleLog2 = 8.0f;
constexpr int kWindow = 8;                // tiles per O window (512 keys)
constexpr uint32_t TMEM_COLS = 512;       // S0, S1 (64 each), O window (128), O total (128)
constexpr uint32_t COL_S0 = 0, COL_O = 128, COL_OT = 256;

constexpr int Q_CHUNK = ROWS * 128;       // 64 dims x 128 rows (fp16), one swizzle column
constexpr int Q_BYTES = 2 * Q_CHUNK;      // one split of Q: 32 KB
constexpr int K_CHUNK = BK * 128;         // 64 dims x 64 keys
constexpr int K_BYTES = 2 * K_CHUNK;      // one split of a K tile: 16 KB
constexpr int V_BYTES = D * 128;          // one split of a V^T tile (128 dims x 64 keys): 16 KB
constexpr int STAGE_BYTES = 2 * K_BYTES + 2 * V_BYTES;  // hi + lo: 64 KB
constexpr int P_BYTES = ROWS * 128;       // one split of P (128 rows x 64 keys): 16 KB

constexpr int OFF_Q = 0;                               // qh, ql
constexpr int OFF_KV = OFF_Q + 2 * Q_BYTES;            // [stage][kh, kl, vh, vl]
constexpr int OFF_P = OFF_KV + STAGES * STAGE_BYTES;   // ph, pl
constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
constexpr int NBAR = 12;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

struct Params {
  int T, Hq, Hkv, G, TQ, prefix, Lp, ntiles_rows, kv_split;
  float *out;  // [T][Hq][D]
  int *err;
};

// kind::f16 instruction descriptor: fp32 accumulate, fp16 A and B, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
__device__ __forceinline__ bool mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_sleep(bar, parity))
    if (globaltimer() - t0 > 2000000000ull) return false;
  return true;
}
// 2^x by the hardware's approximate exponential (relative error a few units
// of 2^-23, far inside the attention bar; 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(THREADS, 1)
    k_attn_prefill_tc(const __grid_constant__ CUtensorMap tmQh,
                      const __grid_constant__ CUtensorMap tmQl,
                      const __grid_constant__ CUtensorMap tmKh,
                      const __grid_constant__ CUtensorMap tmKl,
                      const __grid_constant__ CUtensorMap tmVh,
                      const __grid_constant__ CUtensorMap tmVl, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<1024>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.y;
  const int rt = p.ntiles_rows - 1 - (int)blockIdx.x;  // longest row tiles first
  const int t0 = rt * p.TQ;
  const int rows = p.G * p.TQ;
  const int last_tok = min(p.T, t0 + p.TQ) - 1;
  const int nkt = (p.prefix + last_tok + 1 + BK - 1) / BK;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int B_Q = 0, B_KVF = 1, B_KVE = 3, B_SF = 5, B_SE = 7, B_PF = 9, B_PV = 10, B_FIN = 11;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC + 16);

  if (threadIdx.x == 0) {
    mbar_init(bar(B_Q), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar(B_KVF + s), 1);
      mbar_init(bar(B_KVE + s), 1);
      mbar_init(bar(B_SF + s), 1);
      mbar_init(bar(B_SE + s), 4);
    }
    mbar_init(bar(B_PF), 4);
    mbar_init(bar(B_PV), 1);
    mbar_init(bar(B_FIN), 1);
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
  const uint32_t tmem = *tmem_slot;
  auto fail = [&]() {
    if (p.err) atomicCAS(p.err, 0, 6 /* SI_ERR_TIMEOUT */);
    *abort_flag = 1;
  };
  const int nsplit = p.kv_split ? 2 : 1;  // K / V halves per tile
  const int npass = p.kv_split ? 3 : 2;   // split MMAs per contraction

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint32_t qb = smem_u32(smem + OFF_Q);
      mbar_expect_tx(bar(B_Q), 4 * 128 * rows);
      for (int c = 0; c < 2; ++c) {
        tma_load_3d(qb + c * Q_CHUNK, &tmQh, c * 64, g * p.G, t0, bar(B_Q));
        tma_load_3d(qb + Q_BYTES + c * Q_CHUNK, &tmQl, c * 64, g * p.G, t0, bar(B_Q));
      }
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < nkt; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(bar(B_KVE + s), ((i / STAGES) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t st = smem_u32(smem + OFF_KV + s * STAGE_BYTES);
        mbar_expect_tx(bar(B_KVF + s), nsplit * (K_BYTES + V_BYTES));
        const int krow = g * p.Lp + i * BK;
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(st + c * K_CHUNK, &tmKh, c * 64, krow, bar(B_KVF + s));
          if (p.kv_split) tma_load_2d(st + K_BYTES + c * K_CHUNK, &tmKl, c * 64, krow, bar(B_KVF + s));
        }
        tma_load_2d(st + 2 * K_BYTES, &tmVh, i * BK, g * D, bar(B_KVF + s));
        if (p.kv_split) tma_load_2d(st + 2 * K_BYTES + V_BYTES, &tmVl, i * BK, g * D, bar(B_KVF + s));
        ++issued;
      }
      if (!ok) {
        fail();
        mbar_drain(bar(B_Q), 0);
        for (int k = issued > STAGES ? issued - STAGES : 0; k < issued; ++k)
          mbar_drain(bar(B_KVF + k % STAGES), (k / STAGES) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t qh = smem_u32(smem + OFF_Q), ql = qh + Q_BYTES;
      const uint32_t ph = smem_u32(smem + OFF_P), pl = ph + P_BYTES;
      const uint32_t id_s = idesc_f16(ROWS, BK), id_o = idesc_f16(ROWS, D);
      bool ok = mbar_wait(bar(B_Q), 0, abort_flag);
      for (int i = 0; ok && i <= nkt; ++i) {
        if (i < nkt) {
          const int s = i % STAGES, sb = i % 2;
          if (!mbar_wait(bar(B_KVF + s), (i / STAGES) & 1, abort_flag) ||
              (i >= 2 && !mbar_wait(bar(B_SE + sb), ((i / 2) - 1) & 1, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t kh = smem_u32(smem + OFF_KV + s * STAGE_BYTES), kl = kh + K_BYTES;
          const uint32_t dS = tmem + COL_S0 + sb * BK;
          // S = Qh.Kh [+ Qh.Kl] + Ql.Kh over D in K-steps of 16 (32 bytes).
          uint32_t acc = 0;
          for (int pass = 0; pass < npass; ++pass) {
            const uint32_t a = pass == npass - 1 ? ql : qh;
            const uint32_t b = (p.kv_split && pass == 1) ? kl : kh;
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
              const uint32_t off = (k & 3) * 32;
              mma_f16(dS, smem_desc(a + (k >> 2) * Q_CHUNK + off),
                      smem_desc(b + (k >> 2) * K_CHUNK + off), id_s, acc);
              acc = 1;
            }
          }
          mma_commit(bar(B_SF + sb));
        }
        if (i >= 1) {
          const int j = i - 1, s = j % STAGES;
          if (!mbar_wait(bar(B_PF), j & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t vh = smem_u32(smem + OFF_KV + s * STAGE_BYTES + 2 * K_BYTES),
                         vl = vh + V_BYTES;
          // O += Ph.Vh [+ Ph.Vl] + Pl.Vh over the tile's 64 keys; a window's
          // first tile overwrites O (the softmax warps have moved it on).
          uint32_t acc = j % kWindow != 0;
          for (int pass = 0; pass < npass; ++pass) {
            const uint32_t a = pass == npass - 1 ? pl : ph;
            const uint32_t b = (p.kv_split && pass == 1) ? vl : vh;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              mma_f16(tmem + COL_O, smem_desc(a + k * 32), smem_desc(b + k * 32), id_o, acc);
              acc = 1;
            }
          }
          mma_commit(bar(B_PV));
          mma_commit(bar(B_KVE + s));
        }
      }
      if (!ok) fail();
      mma_commit(bar(B_FIN));
      mbar_drain(bar(B_FIN), 0);
    }
    __syncwarp();
  } else {
    // ---------------- softmax (warps 2-5) and epilogue ----------------
    const int q = warp & 3;  // TMEM lane quarter
    const int r = q * 32 + lane;
    const int tl = r / p.G, hh = r - tl * p.G;
    const int tok = t0 + tl;
    const bool valid = r < rows && tok < p.T;
    const int pos = p.prefix + tok;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    uint8_t *prow_h = smem + OFF_P + (r >> 3) * 1024 + (r & 7) * 128;
    uint8_t *prow_l = prow_h + P_BYTES;
    for (int i = 0; i < nkt; ++i) {
      const int sb = i % 2;
      if (!mbar_wait_warp(bar(B_SF + sb), (i / 2) & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s0[32], s1[32];
      tmem_ld32(tmem + lane_off + COL_S0 + sb * BK, s0);
      tmem_ld32(tmem + lane_off + COL_S0 + sb * BK + 32, s1);
      tmem_wait_ld();
      float sv[BK];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        sv[j] = __uint_as_float(s0[j]);
        sv[32 + j] = __uint_as_float(s1[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_SE + sb));
      // Mask keys past this row's position (and every key of a padding row).
      const int key0 = i * BK;
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < BK; ++j) {
        if (!valid || key0 + j > pos) sv[j] = -INFINITY;
        mt = fmaxf(mt, sv[j]);
      }
      float alpha = 1.0f;
      const bool resc = valid && mt > m + kRescaleLog2;
      if (resc) {
        alpha = exp2f(m - mt);  // 0 on the first tile (m = -inf)
        m = mt;
      }
      float sum = 0.0f;
      uint32_t hw[32], lw[32];
#pragma unroll
      for (int j = 0; j < BK; j += 2) {
        const float p0 = valid ? ex2_approx(sv[j] - m) : 0.0f;
        const float p1 = valid ? ex2_approx(sv[j + 1] - m) : 0.0f;
        sum += p0 + p1;
        // hi = fp16(p), lo = fp16(p - hi), two values per packed conversion.
        const __half2 h = __floats2half2_rn(p0, p1);
        const float2 hf = __half22float2(h);
        const __half2 lo = __floats2half2_rn(p0 - hf.x, p1 - hf.y);
        hw[j / 2] = *reinterpret_cast<const uint32_t *>(&h);
        lw[j / 2] = *reinterpret_cast<const uint32_t *>(&lo);
      }
      l = fmaf(l, alpha, sum);
      // P and O belong to the previous tile's P.V until it has completed.
      if (i >= 1 && !mbar_wait_warp(bar(B_PV), (i - 1) & 1, abort_flag)) {
        ok = false;
        break;
      }
      // Tile i-1 closed a window: O total = (O total + O) * alpha, and the
      // next P.V restarts O.  Otherwise a raised max rescales O (and O total
      // once it holds a window).
      const bool flush = i >= 1 && i % kWindow == 0;
      const bool have_total = i > kWindow;
      if (flush || (i >= 1 && __any_sync(0xffffffffu, resc))) {
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t ov[32], tv[32];
          tmem_ld32(tmem + lane_off + COL_O + c, ov);
          if (have_total) tmem_ld32(tmem + lane_off + COL_OT + c, tv);
          tmem_wait_ld();
          if (flush) {
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const float t = have_total ? __uint_as_float(tv[k]) + __uint_as_float(ov[k])
                                         : __uint_as_float(ov[k]);
              tv[k] = __float_as_uint(t * alpha);
            }
            tmem_st32(tmem + lane_off + COL_OT + c, tv);
          } else {
#pragma unroll
            for (int k = 0; k < 32; ++k) ov[k] = __float_as_uint(__uint_as_float(ov[k]) * alpha);
            tmem_st32(tmem + lane_off + COL_O + c, ov);
            if (have_total) {
#pragma unroll
              for (int k = 0; k < 32; ++k) tv[k] = __float_as_uint(__uint_as_float(tv[k]) * alpha);
              tmem_st32(tmem + lane_off + COL_OT + c, tv);
            }
          }
        }
        tmem_wait_st();
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int sw = (c ^ (r & 7)) << 4;
        *reinterpret_cast<uint4 *>(prow_h + sw) =
            make_uint4(hw[4 * c], hw[4 * c + 1], hw[4 * c + 2], hw[4 * c + 3]);
        *reinterpret_cast<uint4 *>(prow_l + sw) =
            make_uint4(lw[4 * c], lw[4 * c + 1], lw[4 * c + 2], lw[4 * c + 3]);
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PF));
    }
    if (ok && !mbar_wait_warp(bar(B_PV), (nkt - 1) & 1, abort_flag)) ok = false;
    if (!ok) {
      if (lane == 0) fail();
    } else {
      tc_fence_after();
      const float inv = valid ? 1.0f / l : 0.0f;
      float *orow = p.out + ((size_t)tok * p.Hq + (size_t)g * p.G + hh) * D;
      // The open window (tiles since the last flush) plus O total, if any.
      const bool have_total = nkt > kWindow;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t ov[32], tv[32];
        tmem_ld32(tmem + lane_off + COL_O + c, ov);
        if (have_total) tmem_ld32(tmem + lane_off + COL_OT + c, tv);
        tmem_wait_ld();
        if (have_total) {
#pragma unroll
          for (int k = 0; k < 32; ++k)
            ov[k] = __float_as_uint(__uint_as_float(tv[k]) + __uint_as_float(ov[k]));
        }
        if (valid) {
#pragma unroll
          for (int k = 0; k < 32; k += 4)
            *reinterpret_cast<float4 *>(orow + c + k) =
                make_float4(__uint_as_float(ov[k]) * inv, __uint_as_float(ov[k + 1]) * inv,
                            __uint_as_float(ov[k + 2]) * inv, __uint_as_float(ov[k + 3]) * inv);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS));
}

// q (fp32, [T][Hq][D]) * scale -> hi / lo halves, four elements per step (n is
// a multiple of 4: D is 128), two per packed conversion.
__global__ void k_split_q(const float *__restrict__ q, size_t n, float scale,
                          __half *__restrict__ qh, __half *__restrict__ ql) {
  pdl_trigger();
  pdl_wait();
  const float4 *q4 = reinterpret_cast<const float4 *>(q);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 4;
       i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = q4[i];
    const float x0 = __fmul_rn(v.x, scale), x1 = __fmul_rn(v.y, scale);
    const float x2 = __fmul_rn(v.z, scale), x3 = __fmul_rn(v.w, scale);
    const __half2 h01 = __floats2half2_rn(x0, x1), h23 = __floats2half2_rn(x2, x3);
    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
    const __half2 l01 = __floats2half2_rn(x0 - f01.x, x1 - f01.y);
    const __half2 l23 = __floats2half2_rn(x2 - f23.x, x3 - f23.y);
    reinterpret_cast<__half2 *>(qh)[2 * i] = h01;
    reinterpret_cast<__half2 *>(qh)[2 * i + 1] = h23;
    reinterpret_cast<__half2 *>(ql)[2 * i] = l01;
    reinterpret_cast<__half2 *>(ql)[2 * i + 1] = l23;
  }
}

// K and V of sequence seq, positions [0, L) (zero beyond, up to Lp), split into
// hi / lo halves: K as [Hkv][Lp][D], V transposed as [Hkv][D][Lp].  One CTA per
// (64 positions, KV head); V goes through shared memory for the transpose.
template <bool F32>
__global__ void __launch_bounds__(256) k_split_kv(const void *__restrict__ kc,
                                                  const void *__restrict__ vc, int seq,
                                                  int max_ctx, int Hkv, int L, int Lp,
                                                  __half *__restrict__ kh, __half *__restrict__ kl,
                                                  __half *__restrict__ vh, __half *__restrict__ vl) {
  pdl_trigger();
  pdl_wait();
  __shared__ __half sh[BK][D + 8], sl[BK][D + 8];
  const int p0 = blockIdx.x * BK, g = blockIdx.y;
  for (int e = threadIdx.x; e < BK * D; e += blockDim.x) {
    const int pp = e / D, d = e % D, pos = p0 + pp;
    float k = 0.0f, v = 0.0f;
    if (pos < L) {
      const size_t src = (((size_t)seq * max_ctx + pos) * Hkv + g) * D + d;
      if (F32) {
        k = reinterpret_cast<const float *>(kc)[src];
        v = reinterpret_cast<const float *>(vc)[src];
      } else {
        k = f16_to_f32(reinterpret_cast<const uint16_t *>(kc)[src]);
        v = f16_to_f32(reinterpret_cast<const uint16_t *>(vc)[src]);
      }
    }
    const __half khi = __float2half_rn(k), vhi = __float2half_rn(v);
    const size_t kd = ((size_t)g * Lp + pos) * D + d;
    kh[kd] = khi;
    if (F32) kl[kd] = __float2half_rn(k - __half2float(khi));
    sh[pp][d] = vhi;
    sl[pp][d] = __float2half_rn(v - __half2float(vhi));
  }
  __syncthreads();
  for (int e = threadIdx.x; e < BK * D; e += blockDim.x) {
    const int d = e / BK, pp = e % BK;
    const size_t vd = ((size_t)g * D + d) * Lp + p0 + pp;
    vh[vd] = sh[pp][d];
    if (F32) vl[vd] = sl[pp][d];
  }
}

}  // namespace atc

bool attn_tc_supported(const AttnArgs &a) {
  return a.head_dim == atc::D && !a.tok_ctx && !a.tok_seq && a.T >= 16 && a.n_kv_heads > 0 &&
         a.n_q_heads % a.n_kv_heads == 0 && a.n_q_heads / a.n_kv_heads <= 8 &&
         tma_encode_fn() != nullptr;
}

size_t attn_tc_scratch_bytes(const AttnArgs &a) {
  const size_t L = (size_t)(a.ctx0 - 1 + a.T);  // keys of the last token
  const size_t Lp = (L + atc::BK - 1) / atc::BK * atc::BK;
  const size_t q = (size_t)a.T * a.n_q_heads * atc::D;
  const size_t kv = (size_t)a.n_kv_heads * Lp * atc::D;
  return (2 * q + 4 * kv) * sizeof(__half) + 4 * 256;
}

cudaError_t launch_attention_tc(const AttnArgs &a, void *scratch, size_t scratch_bytes,
                                cudaStream_t s) {
  using namespace atc;
  if (!attn_tc_supported(a) || !scratch || scratch_bytes < attn_tc_scratch_bytes(a))
    return cudaErrorInvalidValue;
  const int prefix = a.ctx0 - 1;
  const int L = prefix + a.T;
  const int Lp = (L + BK - 1) / BK * BK;
  const int G = a.n_q_heads / a.n_kv_heads, TQ = ROWS / G;
  const size_t q = (size_t)a.T * a.n_q_heads * D, kv = (size_t)a.n_kv_heads * Lp * D;
  auto align = [](char *p) { return reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(p) + 255) & ~(uintptr_t)255); };
  char *cur = align(static_cast<char *>(scratch));
  __half *qh = reinterpret_cast<__half *>(cur); cur = align(cur + q * 2);
  __half *ql = reinterpret_cast<__half *>(cur); cur = align(cur + q * 2);
  __half *kh = reinterpret_cast<__half *>(cur); cur = align(cur + kv * 2);
  __half *kl = reinterpret_cast<__half *>(cur); cur = align(cur + kv * 2);
  __half *vh = reinterpret_cast<__half *>(cur); cur = align(cur + kv * 2);
  __half *vl = reinterpret_cast<__half *>(cur);

  const float scale = 1.4426950408889634f / sqrtf((float)D);
  if (reinterpret_cast<uintptr_t>(a.q) & 15) return cudaErrorMisalignedAddress;  // float4 reads
  cudaError_t e = launch_pdl(k_split_q, dim3((unsigned)((q + 255) / 256 < 4096 ? (q + 255) / 256 : 4096)),
                             dim3(256), 0, s, a.q, q, scale, qh, ql);
  if (e != cudaSuccess) return e;
  e = a.kv_f32 ? launch_pdl(k_split_kv<true>, dim3(Lp / BK, a.n_kv_heads), dim3(256), 0, s,
                            a.kc, a.vc, a.seq0, a.max_ctx, a.n_kv_heads, L, Lp, kh, kl, vh, vl)
               : launch_pdl(k_split_kv<false>, dim3(Lp / BK, a.n_kv_heads), dim3(256), 0, s,
                            a.kc, a.vc, a.seq0, a.max_ctx, a.n_kv_heads, L, Lp, kh, kl, vh, vl);
  if (e != cudaSuccess) return e;

  CUtensorMap mQh, mQl, mKh, mKl, mVh, mVl;
  cuuint64_t dQ[3] = {(cuuint64_t)D, (cuuint64_t)a.n_q_heads, (cuuint64_t)a.T};
  cuuint64_t sQ[2] = {(cuuint64_t)D * 2, (cuuint64_t)a.n_q_heads * D * 2};
  cuuint32_t bQ[3] = {64, (cuuint32_t)G, (cuuint32_t)TQ};
  cuuint64_t dK[2] = {(cuuint64_t)D, (cuuint64_t)a.n_kv_heads * Lp};
  cuuint64_t sK[1] = {(cuuint64_t)D * 2};
  cuuint32_t bK[2] = {64, (cuuint32_t)BK};
  cuuint64_t dV[2] = {(cuuint64_t)Lp, (cuuint64_t)a.n_kv_heads * D};
  cuuint64_t sV[1] = {(cuuint64_t)Lp * 2};
  cuuint32_t bV[2] = {(cuuint32_t)BK, (cuuint32_t)D};
  const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  if (!tma_encode(&mQh, F16, 3, qh, dQ, sQ, bQ, SW) || !tma_encode(&mQl, F16, 3, ql, dQ, sQ, bQ, SW) ||
      !tma_encode(&mKh, F16, 2, kh, dK, sK, bK, SW) || !tma_encode(&mKl, F16, 2, kl, dK, sK, bK, SW) ||
      !tma_encode(&mVh, F16, 2, vh, dV, sV, bV, SW) || !tma_encode(&mVl, F16, 2, vl, dV, sV, bV, SW))
    return cudaErrorInvalidValue;
  Params p{};
  p.T = a.T; p.Hq = a.n_q_heads; p.Hkv = a.n_kv_heads; p.G = G; p.TQ = TQ;
  p.prefix = prefix; p.Lp = Lp; p.ntiles_rows = (a.T + TQ - 1) / TQ; p.kv_split = a.kv_f32 ? 1 : 0;
  p.out = a.out; p.err = a.err;
  e = cudaFuncSetAttribute(k_attn_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  count_launch();
  k_attn_prefill_tc<<<dim3(p.ntiles_rows, a.n_kv_heads), THREADS, SMEM_BYTES, s>>>(
      mQh, mQl, mKh, mKl, mVh, mVl, p);
  return cudaGetLastError();
}

}  // namespace si
