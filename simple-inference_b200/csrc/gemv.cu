// gemv.cu -- Q4_0 x Q8_0 matrix-vector product for small token counts (decode).
//
// Reference: matvec_q4q8 (qwen_one_layer.c:148-162) and the column-SoA
// fused_column_matvec (fused_layer.h:169-245): out[n] = bias[n] followed, block
// by block IN ORDER, by  out[n] += ((float)isum * dw) * dx.
//
// Mapping.  One CTA owns an RW-row slice (32, 16 or 8 rows) of one 32-row
// tile of the SoA layout and the whole K range, for up to MT tokens; narrow
// slices give matrices with few tiles enough CTAs to fill the GPU, and where
// the slices number between one and two CTA slots per SM a CTA streams two
// slices back to back instead of a second wave starting.  The slice
// streams through a shared-memory ring of up to 8 chunks of CB blocks: a
// producer thread issues three 2-D TMA loads per chunk (nibbles RW*16 B x CB,
// their fp16 scales, the int8 activations of the chunk's blocks) on the
// stage's full mbarrier and refills a stage as soon as its empty mbarrier says
// the compute warps are done with it.  Eight compute warps take the chunk's
// (row, block) pieces and compute the terms in parallel: the int32 block sums
// are exact and each term ((float)isum*dw)*dx is rounded exactly as the
// reference rounds it.  The terms go to term buffers in shared memory, where
// dedicated merge warps -- one thread per (token, row) -- add them to the
// running sums in block order, each buffer handed over on its own pair of
// mbarriers, so loads, terms and adds of neighbouring chunks overlap.  The
// result is bit-identical to the reference's serial loop.
//
// For small token counts this kernel is HBM-bound: at one token the 72B down
// projection (136 MB of weights) streams at about 90 % of the measured copy
// bandwidth.
//
// SwiGLU mode streams the gate rows and then the up rows of the same slice
// through the ring, then forms act = silu(g) * u and quantises it to Q8_0
// directly: the 32 rows of a tile are exactly one Q8 block of the down
// projection's input.
#include <type_traits>

#include "si_common.cuh"
#include "si_kernels.cuh"
#include "si_tma.cuh"

namespace si {

namespace {
constexpr int kComputeWarps = 8;
constexpr int kMaxRing = 8;               // ring stages, at most
constexpr size_t kCtaBudget = 113 * 1024; // shared memory that keeps two CTAs per SM

__device__ __forceinline__ float silu_mul(float g, float u) {
  float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(s, u);
}

// Shape of one instantiation.  A chunk is CB blocks of the RW-row slice; the
// compute thread (compute warp w, lane = bo*RW + rl) owns pieces u < U of each
// chunk: block (w*U + u)*BPL + bo, row rl.
template <int MT, int RW>
struct Shape {
  static constexpr int BPL = SI_RT / RW;
  static constexpr int CB0 = (4096 / (MT * RW)) < (1024 / RW) ? 4096 / (MT * RW) : 1024 / RW;
  static constexpr int CB = CB0 < 64 ? CB0 : 64;            // nibbles <= 16 KB per stage
  static constexpr int U = CB / (kComputeWarps * BPL);
  static constexpr int MW = (MT * RW + 31) / 32;            // merge warps
  static constexpr int WARPS = 1 + kComputeWarps + MW;      // producer, compute, merge
  static constexpr int THREADS = WARPS * 32;
  static constexpr int NIB = CB * RW * 16;                  // [CB][RW][16 B]
  static constexpr int SCL = CB * RW * 2;                   // [CB][RW] fp16
  static constexpr int ACT = MT * CB * 32;                  // [MT][CB][32 B]
  static constexpr int STAGE = NIB + SCL + ACT;
  static constexpr int TERMS = MT * CB * RW;                // floats per term buffer
  static constexpr int NTB = TERMS * 4 <= 8192 ? 4 : 2;     // term buffers
  // Shared memory: ns ring stages, NTB term buffers, 256 B of barriers and the
  // abort flag, dx/16 as fp32 [KB][MT], alignment slack.
  __host__ __device__ static size_t fixed(int ns) {
    return (size_t)ns * STAGE + (size_t)NTB * TERMS * sizeof(float) + 256;
  }
  static size_t smem(int ns, int KB) { return fixed(ns) + (size_t)MT * KB * sizeof(float) + 128; }
  static_assert(U >= 1 && U * kComputeWarps * BPL == CB, "chunk shape");
  static_assert(NIB % 128 == 0 && SCL % 128 == 0 && ACT % 128 == 0, "TMA destinations");
};

// Grid: (N/32 tiles x 32/RW row slices, token groups of MT).
//
// Roles.  Warp 0 is the producer: one thread streams the slice's chunks
// through the ring (three 2-D TMA loads per chunk on the stage's full
// barrier), refilling a stage as soon as the eight compute warps have
// released it on its empty barrier.  The compute warps turn a chunk's
// (row, block) pieces into terms in a term buffer and publish it on that
// buffer's full barrier; the merge warps -- one thread per (token, row) --
// add the terms to the running sums in block order and release the buffer.
// No role waits for another except through these barriers, so the loads of
// later chunks, the terms of the current one and the adds of the previous
// one overlap.
//
// Term.  ((float)isum * dw) * dx is computed as ((float)(16*isum) * dw) *
// (dx/16): the dp4a of the pre-shifted nibbles returns 16*isum, exact in fp32,
// and scaling by a power of two commutes with both roundings (the products
// stay far inside the normal range), so the term is bit-identical to the
// reference's.
template <int MT, int RW, bool SWIGLU, bool MULTI>
__global__ void __launch_bounds__(Shape<MT, RW>::THREADS, 2)
    k_gemv(const __grid_constant__ CUtensorMap tmN, const __grid_constant__ CUtensorMap tmN2,
           const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmS2,
           const __grid_constant__ CUtensorMap tmX, const GemvArgs a, int ns) {
  using S = Shape<MT, RW>;
  constexpr int CB = S::CB, BPL = S::BPL, U = S::U, SLICES = SI_RT / RW, NTB = S::NTB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<128>(smem_raw);
  float *T = reinterpret_cast<float *>(smem + ns * S::STAGE);            // [NTB][MT][CB][RW]
  uint64_t *bars = reinterpret_cast<uint64_t *>(T + NTB * S::TERMS);
  uint64_t *full = bars, *empty = bars + kMaxRing;                       // [ns] each
  uint64_t *tfull = bars + 2 * kMaxRing, *tempty = tfull + 4;            // [NTB] each
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tempty + 4);
  float *dxs = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(bars) + 256);  // [KB][MT]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Units (an RW-row slice of a tile) of this CTA: blockIdx.x + i * gridDim.x.
  // One, or (MULTI) where the units fill between one and two CTA slots per
  // SM, up to two streamed back to back through the same ring (the second
  // unit's loads overlap the first one's tail instead of a second wave's
  // start-up).
  const int units = (a.N / SI_RT) * SLICES;
  const int nu = MULTI ? (units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 1;
  auto unit_tile = [&](int i) { return ((int)blockIdx.x + i * (int)gridDim.x) / SLICES; };
  auto unit_r0 = [&](int i) { return ((int)blockIdx.x + i * (int)gridDim.x) % SLICES * RW; };
  const int m0 = blockIdx.y * MT, mcount = min(MT, a.M - m0);
  const int KB = a.K / 32;
  const int npass = (KB + CB - 1) / CB;                 // chunks per matrix
  const int nchunks = SWIGLU ? 2 * npass : npass;       // chunks per unit
  const int ntot = nu * nchunks;
  auto bar = [&](uint64_t *b, int i) { return smem_u32(b + i); };

  pdl_trigger();

  // Chunk c of unit i: pass c / npass (gate, then up), blocks [cc*CB, cc*CB + CB).
  auto load_weights = [&](int i, int c, int slot) {
    const int pass = c >= npass, cc = pass ? c - npass : c;
    uint8_t *st = smem + slot * S::STAGE;
    const int y = unit_tile(i) * KB + cc * CB, r0 = unit_r0(i);
    mbar_expect_tx(bar(full, slot), S::STAGE);
    tma_load_2d(smem_u32(st), pass ? &tmN2 : &tmN, r0 * 2, y, bar(full, slot));
    tma_load_2d(smem_u32(st + S::NIB), pass ? &tmS2 : &tmS, r0, y, bar(full, slot));
  };
  auto load_acts = [&](int c, int slot) {
    const int cc = c >= npass ? c - npass : c;
    tma_load_2d(smem_u32(smem + slot * S::STAGE + S::NIB + S::SCL), &tmX, cc * CB * 4, m0,
                bar(full, slot));
  };
  // Thread 0 sets the barriers up and requests the weights of the first
  // chunks right away -- before the previous kernel (which may still be
  // running) has produced the activations.
  const int pre = ntot < ns ? ntot : ns;
  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmN)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmS)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
    for (int i = 0; i < ns; ++i) {
      mbar_init(bar(full, i), 1);
      mbar_init(bar(empty, i), kComputeWarps * 32);
    }
    for (int i = 0; i < NTB; ++i) {
      mbar_init(bar(tfull, i), kComputeWarps * 32);
      mbar_init(bar(tempty, i), S::MW * 32);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int g = 0; g < pre; ++g) load_weights(g / nchunks, g % nchunks, g);
  }
  pdl_wait();
  if (threadIdx.x == 0)
    for (int g = 0; g < pre; ++g) load_acts(g % nchunks, g);
  for (int i = threadIdx.x; i < mcount * KB; i += blockDim.x) {
    const int m = i / KB, b = i - m * KB;
    dxs[b * MT + m] = __fmul_rn(f16_to_f32(a.xd[(size_t)(m0 + m) * KB + b]), 0.0625f);
  }
  __syncthreads();  // barriers initialised, dxs visible

  if (warp == 0) {
    // ---- producer ----
    if (lane != 0) return;
    int slot = pre == ns ? 0 : pre, phase = 0;
    int issued = pre;
    int ui = pre / nchunks, uc = pre - ui * nchunks;  // unit and chunk of the next load
    for (int g = pre; g < ntot; ++g) {
      if (!mbar_wait(bar(empty, slot), phase, abort_flag)) {
        *abort_flag = 1;
        raise_error(a.err, 6 /* SI_ERR_TIMEOUT */);
        break;
      }
      load_weights(ui, uc, slot);
      load_acts(uc, slot);
      ++issued;
      if (++slot == ns) { slot = 0; phase ^= 1; }
      if (++uc == nchunks) { uc = 0; ++ui; }
    }
    if (*abort_flag) {
      // Let the copies still in flight land before the CTA's shared memory
      // goes away (bounded: the waits give up after their deadline).
      const int first = issued > ns ? issued - ns : 0;
      int none = 0;
      for (int c = first; c < issued; ++c) mbar_wait(bar(full, c % ns), (c / ns) & 1, &none);
    }
    return;
  }

  if (warp <= kComputeWarps) {
    // ---- compute ----
    const int cw = warp - 1;
    const int bo = lane / RW, rl = lane % RW;
    const bool want_isum = !SWIGLU && a.isum_out != nullptr;
    int slot = 0, sp = 0, tb = 0, tp = 0;
    int ui = 0, c = 0, tile = unit_tile(0), r0 = unit_r0(0);  // the chunk's unit
    for (int g = 0; g < ntot; ++g) {
      if constexpr (MULTI) {
        if (c == nchunks) {
          c = 0;
          ++ui;
          tile = unit_tile(ui);
          r0 = unit_r0(ui);
        }
      }
      const int cc = c >= npass ? c - npass : c;
      bool ok = mbar_wait(bar(full, slot), sp, abort_flag);
      if (ok && g >= NTB) ok = mbar_wait(bar(tempty, tb), tp ^ 1, abort_flag);
      if (!ok) {
        *abort_flag = 1;
        raise_error(a.err, 6 /* SI_ERR_TIMEOUT */);
        return;
      }
      const uint8_t *st = smem + slot * S::STAGE;
      const uint4 *nb = reinterpret_cast<const uint4 *>(st);
      const uint16_t *sb = reinterpret_cast<const uint16_t *>(st + S::NIB);
      const int4 *ab = reinterpret_cast<const int4 *>(st + S::NIB + S::SCL);
      float *Tb = T + tb * S::TERMS;
      auto pieces = [&](auto whole) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int bl = (cw * U + u) * BPL + bo;
          const int bx = cc * CB + bl;  // block within the matrix
          if (decltype(whole)::value || bx < KB) {
            const uint4 w = nb[bl * RW + rl];
            const float dw = f16_to_f32(sb[bl * RW + rl]);
            const int lo[4] = {lo_nib_s8x16(w.x), lo_nib_s8x16(w.y), lo_nib_s8x16(w.z),
                               lo_nib_s8x16(w.w)};
            const int hi[4] = {hi_nib_s8x16(w.x), hi_nib_s8x16(w.y), hi_nib_s8x16(w.z),
                               hi_nib_s8x16(w.w)};
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              if (MT == 1 || m < mcount) {
                const int4 a0 = ab[(m * CB + bl) * 2], a1 = ab[(m * CB + bl) * 2 + 1];
                int s16 = __dp4a(lo[0], a0.x, 0);
                s16 = __dp4a(lo[1], a0.y, s16);
                s16 = __dp4a(lo[2], a0.z, s16);
                s16 = __dp4a(lo[3], a0.w, s16);
                s16 = __dp4a(hi[0], a1.x, s16);
                s16 = __dp4a(hi[1], a1.y, s16);
                s16 = __dp4a(hi[2], a1.z, s16);
                s16 = __dp4a(hi[3], a1.w, s16);
                Tb[(m * CB + bl) * RW + rl] =
                    __fmul_rn(__fmul_rn((float)s16, dw), dxs[bx * MT + m]);
                if (want_isum)
                  a.isum_out[((size_t)(m0 + m) * a.N + (size_t)tile * SI_RT + r0 + rl) * KB + bx] =
                      s16 >> 4;
              }
            }
          }
        }
      };
      if (cc * CB + CB <= KB) pieces(std::true_type{});
      else pieces(std::false_type{});
      mbar_arrive(bar(empty, slot));  // this thread is done with the stage
      mbar_arrive(bar(tfull, tb));    // and its terms are written
      if (++slot == ns) { slot = 0; sp ^= 1; }
      if (++tb == NTB) { tb = 0; tp ^= 1; }
      ++c;
    }
    return;
  }

  // ---- merge: thread (token tm, row tr) ----
  const int mt = threadIdx.x - (1 + kComputeWarps) * 32;
  const int tm = mt / RW, tr = mt % RW;
  const bool merging = tm < mcount;
  int tb = 0, tp = 0;
  for (int i = 0; i < nu; ++i) {
    const int tile = unit_tile(i), r0 = unit_r0(i);
    float acc = 0.0f, first = 0.0f;
    if (!SWIGLU && merging && a.bias) acc = a.bias[tile * SI_RT + r0 + tr];
    for (int c = 0; c < nchunks; ++c) {
      const int cc = c >= npass ? c - npass : c;
      if (!mbar_wait(bar(tfull, tb), tp, abort_flag)) {
        *abort_flag = 1;
        raise_error(a.err, 6 /* SI_ERR_TIMEOUT */);
        return;
      }
      if (merging) {
        // The adds are a serial chain; load the terms 16 at a time ahead of it.
        const int nvalid = min(CB, KB - cc * CB);
        const float *Tm = T + tb * S::TERMS + tm * CB * RW + tr;
        if (SWIGLU && c == npass) {  // the up rows begin
          first = acc;
          acc = 0.0f;
        }
        int j = 0;
        for (; j + 16 <= nvalid; j += 16) {
          float v[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) v[q] = Tm[(j + q) * RW];
#pragma unroll
          for (int q = 0; q < 16; ++q) acc = __fadd_rn(acc, v[q]);
        }
        for (; j < nvalid; ++j) acc = __fadd_rn(acc, Tm[j * RW]);
      }
      mbar_arrive(bar(tempty, tb));
      if (++tb == NTB) { tb = 0; tp ^= 1; }
    }
    if (!merging) continue;
    const int row = tile * SI_RT + r0 + tr;
    const size_t o = (size_t)(m0 + tm) * a.N + row;
    if (!SWIGLU) {
      a.out[o] = a.resid ? __fadd_rn(a.resid[o], acc) : acc;
    } else {
      // RW == 32: merge warp m holds token m's 32 outputs of the tile, one Q8 block.
      const float act = silu_mul(first, acc);
      if (a.out) a.out[o] = act;
      uint16_t d16;
      const int8_t q = q8_lane(act, d16);
      a.act_qs[o] = q;
      if (tr == 0) a.act_d[(size_t)(m0 + tm) * (a.N / 32) + tile] = d16;
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core form (3..16 tokens per CTA).  One CTA per 32-row tile and the
// whole K range.  Per block and 16-row group, one mma.sync m16n8k32
// (s8 x s8 -> s32) per 8 tokens takes the weight rows as its 16 M-rows: lane
// (g, c) holds nibble word c of rows g and g+8, whose low nibbles are elements
// 4c..4c+3 and high nibbles 16+4c..16+4c+3 -- exactly the four A registers of
// the fragment -- and the B fragment is token g's activation bytes 4c..4c+3
// and 16+4c..16+4c+3.  The result is the exact 16*isum of every (row, token)
// pair of the block, in registers: lane (g, c) owns rows g, g+8 x tokens 2c,
// 2c+1 of each octet.
//
// Order.  Each output is bias + term(block 0) + term(block 1) + ... added one
// at a time, the reference's serial chain, so the result is bit-identical to
// the dp4a form and to matvec_q4q8.  The terms themselves are independent, so
// the CTA runs four phases of warps per 16-row group: phase k computes the
// terms of chunks k, k+4, ... into registers while the other phases compute
// theirs, then waits on a named barrier for the running sums of the previous
// chunk (phase k-1), adds its chunk's terms in block order, and hands the sums
// on through shared memory to phase k+1.  Only the adds are serial.
//
// Terms.  term = ((float)isum * dw) * dx is computed as
// ((float)(16*isum) * dw) * (dx/16): 16*isum is exact in fp32 and scaling by a
// power of two commutes with rounding, so both products round exactly as the
// reference's do; dx/16 is kept per (block, token) in shared memory.
//
// Pipeline.  A producer warp streams the tile through a ring of 5-12 chunks of
// CB blocks (nibbles, fp16 scales and the chunk's activations: three or five
// 2-D TMA loads on the stage's full barrier); the two warps of a phase release
// a stage on its empty barrier.  CB = 9 or 5 (1 mod 4) keeps the B-fragment
// loads at two-way bank conflicts.  The per-block rescale has to see every
// block's integer sums, which mma.sync returns in registers; a tcgen05 MMA
// would put each block's sums in tensor memory and need a round trip per block.
constexpr int kMmaPhases = 4;
// G: 16-row groups per CTA -- 2 (a whole 32-row tile), or 1 (half a tile, for
// matrices with fewer tiles than SMs: twice the CTAs).
__host__ __device__ constexpr int mma_warps(int G) { return kMmaPhases * G + 1; }  // + producer
constexpr int kMmaMaxRing = 12;                                 // stages, at most
constexpr size_t kMmaCtaBudget = 113 * 1024;  // shared memory that keeps two CTAs per SM
constexpr size_t kMmaCtaBudget3 = 74 * 1024;  // ... and three

template <int MT, bool SWIGLU, int G = 2>
struct MmaShape {
  static constexpr int RWS = 16 * G;                  // rows per CTA
  static constexpr int W = SWIGLU ? 2 : 1;            // weight streams
  static constexpr int NT = MT / 8;                   // token octets
  // A chunk's terms stay in registers until the hand-off (36-80 per lane);
  // mma groups of GB blocks in flight.
  static constexpr int CB = W * NT == 1 ? 9 : 5;      // blocks per chunk
  static constexpr int GB = W * NT == 1 ? 3 : 1;
  static constexpr int MINB = NT == 2 ? 1 : 2;        // CTAs per SM the registers allow
  static constexpr int NIB = CB * RWS * 16;           // [CB][RWS rows][16 B]
  static constexpr int SCL = (CB * RWS * 2 + 127) / 128 * 128;    // [CB][RWS] fp16, padded
  static constexpr int ACT = MT * CB * 32;            // [MT][CB][32 B]
  static constexpr int WS = (NIB + SCL + 127) / 128 * 128;        // one weight stream
  static constexpr int STAGE = W * WS + (ACT + 127) / 128 * 128;
  static constexpr int TX = W * (NIB + CB * RWS * 2) + ACT;  // bytes the TMA boxes deliver
  static constexpr int NV = W * NT * 4;               // sums per lane
  static constexpr int ACCS = G * 32 * NV;            // hand-off floats
  // ring, 256 B of barriers and flags, hand-off sums, the per-warp amax of
  // the Q8 epilogue, dx/16 per (block, token) as fp32, slack
  static size_t smem(int ns, int KB) {
    return (size_t)ns * STAGE + 256 + ACCS * 4 + G * MT * 4 + (size_t)KB * MT * 4 + 128;
  }
  static_assert(NIB % 128 == 0 && WS % 128 == 0 && STAGE % 128 == 0, "TMA destinations");
};

// The accumulator input is the integer 0x4B400000, so each result is
// 0x4B400000 + 16*isum: the bit pattern of the float 1.5*2^23 + 16*isum.
constexpr int kMagicBits = 0x4B400000;
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(kMagicBits));
}
// Packed f32x2 arithmetic as explicit .rn PTX: each lane is one IEEE
// operation with its own rounding (explicit instructions are not contracted).
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int threads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// MB: CTAs per SM the launch is built for (registers; the ring is sized to
// match): MmaShape::MINB, or 3 for one-token-octet shapes whose tiles need
// between two and three per SM to fit in one wave.
template <int MT, bool SWIGLU, bool ISUM, int MB, int G>
__global__ void __launch_bounds__(mma_warps(G) * 32, MB)
    k_gemv_mma(const __grid_constant__ CUtensorMap tmN, const __grid_constant__ CUtensorMap tmN2,
               const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmS2,
               const __grid_constant__ CUtensorMap tmX, const GemvArgs a, int ns) {
  static_assert(G == 2 || !SWIGLU, "the SwiGLU Q8 epilogue needs whole 32-row tiles");
  using S = MmaShape<MT, SWIGLU, G>;
  constexpr int CB = S::CB, NT = S::NT, W = S::W, NV = S::NV, P = kMmaPhases, RWS = S::RWS;
  constexpr int WARPS = mma_warps(G);
  constexpr int HAND = 2 * G * 32;  // threads in one hand-off
  // Named barriers: 1..P hand-offs (id 1+k: into phase k), P+1 the compute
  // warps' start, P+2 the Q8 epilogue's warps.
  constexpr int kBarStart = P + 1, kBarEpi = P + 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_align<128>(smem_raw);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + ns * S::STAGE);   // [kMmaMaxRing]
  uint64_t *empty = full + kMmaMaxRing;                                  // [kMmaMaxRing]
  volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kMmaMaxRing);
  float *acc_s = reinterpret_cast<float *>(smem + ns * S::STAGE + 256);  // [group][lane][NV]
  unsigned *red = reinterpret_cast<unsigned *>(acc_s + S::ACCS);         // [group][MT]
  float *dxs = reinterpret_cast<float *>(red + G * MT);                  // [KB][MT], dx/16

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  // CTA x: 32-row tile x / (2 / G), its RWS-row slice x % (2 / G).
  const int tile = blockIdx.x / (2 / G), slice = blockIdx.x % (2 / G);
  const int rbase = tile * SI_RT + slice * RWS;  // the CTA's first row
  const int m0 = blockIdx.y * MT, mcount = min(MT, a.M - m0);
  const int KB = a.K / 32, nchunks = (KB + CB - 1) / CB;
  auto fb = [&](int i) { return smem_u32(full + i); };
  auto eb = [&](int i) { return smem_u32(empty + i); };

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < ns; ++i) {
      mbar_init(fb(i), 1);
      mbar_init(eb(i), G);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == WARPS - 1) {
    // ---- producer ----------------------------------------------------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmN)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmS)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
      // Ring position (slot, wrap) advanced incrementally: ns is a runtime value.
      auto weights = [&](int ci, int slot) {
        uint8_t *st = smem + slot * S::STAGE;
        const int y = tile * KB + ci * CB;
        mbar_expect_tx(fb(slot), S::TX);
        tma_load_2d(smem_u32(st), &tmN, slice * RWS * 2, y, fb(slot));
        tma_load_2d(smem_u32(st + S::NIB), &tmS, slice * RWS, y, fb(slot));
        if (SWIGLU) {
          tma_load_2d(smem_u32(st + S::WS), &tmN2, 0, y, fb(slot));
          tma_load_2d(smem_u32(st + S::WS + S::NIB), &tmS2, 0, y, fb(slot));
        }
      };
      auto acts = [&](int ci, int slot) {
        tma_load_2d(smem_u32(smem + slot * S::STAGE + W * S::WS), &tmX, ci * CB * 4, m0, fb(slot));
      };
      // The first ring's weights go out before the previous kernel has
      // produced the activations.
      const int pre = nchunks < ns ? nchunks : ns;
      for (int ci = 0; ci < pre; ++ci) weights(ci, ci);
      pdl_wait();
      for (int ci = 0; ci < pre; ++ci) acts(ci, ci);
      int slot = 0, wrap = 0;  // chunk ci = ns * (wrap + 1) + slot reuses slot
      for (int ci = pre; ci < nchunks; ++ci) {
        if (!mbar_wait(eb(slot), wrap & 1, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        weights(ci, slot);
        acts(ci, slot);
        if (++slot == ns) {
          slot = 0;
          ++wrap;
        }
      }
    }
    return;
  }

  // ---- compute warps: phase k, 16-row group rg ---------------------------
  const int k = warp / G, rg = warp % G;
  pdl_wait();
  {
    // Eight independent loads in flight per thread (a K of 29568 has 7392
    // scales per 8 tokens).
    constexpr int NTH = (WARPS - 1) * 32;
    for (int i0 = threadIdx.x; i0 < MT * KB; i0 += 8 * NTH) {
      uint16_t v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + j * NTH, m = i / KB, blk = i % KB;
        v[j] = (i < MT * KB && m < mcount) ? a.xd[(size_t)(m0 + m) * KB + blk] : (uint16_t)0;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + j * NTH;
        if (i < MT * KB) dxs[(i % KB) * MT + i / KB] = __fmul_rn(f16_to_f32(v[j]), 0.0625f);
      }
    }
  }
  named_sync(kBarStart, (WARPS - 1) * 32);  // dxs visible

  const int r0 = rbase + 16 * rg + g;  // this lane's rows r0 and r0 + 8
  // sums [stream][octet][row half][token of the pair]
  float acc[W][NT][2][2];
  bool ok = true;
  int last = -1;  // the chunk whose sums this warp holds at the end
  int slot = k, phase = 0;  // ring position of chunk ci (k < P < ns), advanced below
  for (int ci = k; ci < nchunks; ci += P) {
    const bool got = ok && mbar_wait(fb(slot), phase, abort_flag);
    if (!got) {
      ok = false;
      *abort_flag = 1;
    }
    const uint8_t *st = smem + slot * S::STAGE;
    const uint8_t *act = st + W * S::WS;
    const int nb = min(CB, KB - ci * CB);
    float t[CB][W][NT][2][2];
    auto group = [&](auto nbc, int bl0) {
      constexpr int NB = decltype(nbc)::value;
      int d[NB][W][NT][4];
      uint32_t dwp[NB][W][2];
      float2 dx[NB][NT];
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const int bl = bl0 + j, bx = ci * CB + bl;
        uint32_t b[NT][2];
#pragma unroll
        for (int q = 0; q < NT; ++q) {
          const uint32_t *ar = reinterpret_cast<const uint32_t *>(act + ((g + 8 * q) * CB + bl) * 32);
          b[q][0] = ar[c];
          b[q][1] = ar[4 + c];
          dx[j][q] = *reinterpret_cast<const float2 *>(dxs + bx * MT + 8 * q + 2 * c);
        }
#pragma unroll
        for (int wi = 0; wi < W; ++wi) {
          const uint8_t *ws = st + wi * S::WS;
          const uint8_t *wr = ws + bl * (RWS * 16) + (16 * rg + g) * 16 + 4 * c;
          const uint32_t w0 = *reinterpret_cast<const uint32_t *>(wr);
          const uint32_t w8 = *reinterpret_cast<const uint32_t *>(wr + 8 * 16);
          const uint32_t a0 = (uint32_t)lo_nib_s8x16(w0), a2 = (uint32_t)hi_nib_s8x16(w0);
          const uint32_t a1 = (uint32_t)lo_nib_s8x16(w8), a3 = (uint32_t)hi_nib_s8x16(w8);
#pragma unroll
          for (int q = 0; q < NT; ++q) mma_s8_16832(d[j][wi][q], a0, a1, a2, a3, b[q][0], b[q][1]);
          const uint16_t *sr = reinterpret_cast<const uint16_t *>(ws + S::NIB) + bl * RWS + 16 * rg + g;
          dwp[j][wi][0] = sr[0];
          dwp[j][wi][1] = sr[8];
        }
      }
#pragma unroll
      for (int j = 0; j < NB; ++j) {
#pragma unroll
        for (int wi = 0; wi < W; ++wi) {
          // One row, the lane's two tokens (2c, 2c+1) per packed operation --
          // the mma's adjacent result registers and the adjacent dx/16 pair:
          // the mma result 0x4B400000 + d (d = 16*isum) is the float
          // 1.5*2^23 + d (|d| < 2^22), and fma(f, dw, -1.5*2^23*dw) =
          // round(d * dw) with one rounding -- the product (float)d * dw
          // without an int-to-float conversion, which runs on a narrow pipe.
          // -1.5*2^23*dw is exact (fp16 dw).
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float x = f16_to_f32((uint16_t)dwp[j][wi][h]);
            const float2 dw = make_float2(x, x);
            const float2 nk = mul2_rn(dw, make_float2(-12582912.0f, -12582912.0f));
#pragma unroll
            for (int q = 0; q < NT; ++q) {
              float2 f = make_float2(__int_as_float(d[j][wi][q][2 * h]),
                                     __int_as_float(d[j][wi][q][2 * h + 1]));
              f = mul2_rn(fma2_rn(f, dw, nk), dx[j][q]);
              t[bl0 + j][wi][q][h][0] = f.x;
              t[bl0 + j][wi][q][h][1] = f.y;
            }
          }
        }
        if constexpr (ISUM) {
          const int bx = ci * CB + bl0 + j;
#pragma unroll
          for (int q = 0; q < NT; ++q)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int tok = 8 * q + 2 * c + e;
                if (tok < mcount)
                  a.isum_out[((size_t)(m0 + tok) * a.N + r0 + 8 * h) * KB + bx] =
                      (d[j][0][q][2 * h + e] - kMagicBits) >> 4;
              }
        }
      }
    };
    if (got) {
      if (nb == CB) {
#pragma unroll
        for (int bl0 = 0; bl0 + S::GB <= CB; bl0 += S::GB)
          group(std::integral_constant<int, S::GB>{}, bl0);
#pragma unroll
        for (int bl = CB / S::GB * S::GB; bl < CB; ++bl) group(std::integral_constant<int, 1>{}, bl);
      } else {
#pragma unroll
        for (int bl = 0; bl < CB; ++bl)
          if (bl < nb) group(std::integral_constant<int, 1>{}, bl);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(eb(slot));  // stage free for the producer
    // Running sums of the previous chunk, then this chunk's terms in order.
    float *ac = &acc[0][0][0][0];
    if (ci == 0) {
#pragma unroll
      for (int wi = 0; wi < W; ++wi)
#pragma unroll
        for (int q = 0; q < NT; ++q)
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int e = 0; e < 2; ++e)
              acc[wi][q][h][e] = (!SWIGLU && a.bias) ? a.bias[r0 + 8 * h] : 0.0f;
    } else {
      named_sync(1 + k, HAND);
      const float *src = acc_s + (rg * 32 + lane) * NV;
#pragma unroll
      for (int i = 0; i < NV; ++i) ac[i] = src[i];
    }
    if (got) {
      if (nb == CB) {
#pragma unroll
        for (int bl = 0; bl < CB; ++bl) {
          const float *tb = &t[bl][0][0][0][0];
#pragma unroll
          for (int i = 0; i < NV; ++i) ac[i] = __fadd_rn(ac[i], tb[i]);
        }
      } else {
#pragma unroll
        for (int bl = 0; bl < CB; ++bl)
          if (bl < nb) {
            const float *tb = &t[bl][0][0][0][0];
#pragma unroll
            for (int i = 0; i < NV; ++i) ac[i] = __fadd_rn(ac[i], tb[i]);
          }
      }
    }
    if (ci + 1 < nchunks) {
      float *dst = acc_s + (rg * 32 + lane) * NV;
#pragma unroll
      for (int i = 0; i < NV; ++i) dst[i] = ac[i];
      named_arrive(1 + (k + 1) % P, HAND);
    }
    last = ci;
    slot += P;
    if (slot >= ns) {
      slot -= ns;
      phase ^= 1;
    }
  }
  if (last != nchunks - 1) return;  // another phase holds the final sums
  if (*abort_flag) ok = false;
  if (!ok) {
    if (lane == 0) raise_error(a.err, 6 /* SI_ERR_TIMEOUT */);
    return;
  }

  if (!SWIGLU && a.peer.world > 0) {
    // Row-parallel tensor parallelism: the partial sums go to this rank's slot
    // on every rank (peer stores over NVLink), each value in one 8-byte word
    // with the call's epoch in its upper half -- the reader polls the words
    // themselves, so there is no fence and no separate flag.  The tile's sums
    // are gathered in shared memory first ([token][32 rows], over the hand-off
    // area, free once both warps have read their sums), so each token's 32
    // rows cross NVLink as 256 contiguous bytes.
    const PeerOut &pr = a.peer;
    const unsigned long long ep = peer_epoch(pr);
    const size_t slot0 = ((size_t)(ep & 1) * pr.world + pr.rank) * pr.slot;
    const unsigned long long tag = (unsigned long long)(unsigned)ep << 32;
    named_sync(kBarEpi, G * 32);
    float *tile_s = acc_s;  // MT * RWS floats == S::ACCS
#pragma unroll
    for (int q = 0; q < NT; ++q)
#pragma unroll
      for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          tile_s[(8 * q + 2 * c + e) * RWS + 16 * rg + g + 8 * h] = acc[0][q][h][e];
    named_sync(kBarEpi, G * 32);
    constexpr int R4 = RWS / 4;      // four-row pieces per token
    const int et = rg * 32 + lane;   // token et / R4, rows 4 * (et % R4) ..
    for (int i = et; i < mcount * R4; i += G * 32) {
      const int tok = i / R4, r4 = (i % R4) * 4;
      const float4 v = *reinterpret_cast<const float4 *>(tile_s + tok * RWS + r4);
      const unsigned long long w0 = tag | __float_as_uint(v.x), w1 = tag | __float_as_uint(v.y);
      const unsigned long long w2 = tag | __float_as_uint(v.z), w3 = tag | __float_as_uint(v.w);
      const size_t o = slot0 + (size_t)(m0 + tok) * a.N + (size_t)rbase + r4;
      for (int dst = 0; dst < pr.world; ++dst) {
        unsigned long long *wp = reinterpret_cast<unsigned long long *>(pr.base[dst] + kPeerData) + o;
        asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(wp), "l"(w0), "l"(w1)
                     : "memory");
        asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(wp + 2), "l"(w2), "l"(w3)
                     : "memory");
      }
    }
  } else if (!SWIGLU) {
#pragma unroll
    for (int q = 0; q < NT; ++q)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tok = 8 * q + 2 * c + e;
        if (tok >= mcount) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const size_t o = (size_t)(m0 + tok) * a.N + r0 + 8 * h;
          float v = acc[0][q][h][e];
          if (a.resid) v = __fadd_rn(a.resid[o], v);
          a.out[o] = v;
        }
      }
  } else {
    // act = silu(g) * u; the tile's 32 rows of a token are one Q8 block,
    // spread over this phase's warps (16 rows each, rows g and g+8 per lane).
    float act[NT][2][2];
#pragma unroll
    for (int q = 0; q < NT; ++q)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        unsigned m = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          act[q][h][e] = silu_mul(acc[0][q][h][e], acc[1][q][h][e]);
          m = max(m, __float_as_uint(fabsf(act[q][h][e])));
        }
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 16));
        if (g == 0) red[rg * MT + 8 * q + 2 * c + e] = m;
      }
    named_sync(kBarEpi, G * 32);
#pragma unroll
    for (int q = 0; q < NT; ++q)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tok = 8 * q + 2 * c + e;
        if (tok >= mcount) continue;
        const unsigned mb = max(red[tok], red[MT + tok]);
        const float d = __fdiv_rn(__uint_as_float(mb), 127.0f);
        const float inv = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const size_t o = (size_t)(m0 + tok) * a.N + r0 + 8 * h;
          if (a.out) a.out[o] = act[q][h][e];
          int v = __float2int_rn(__fmul_rn(act[q][h][e], inv));
          v = v > 127 ? 127 : (v < -127 ? -127 : v);
          a.act_qs[o] = (int8_t)v;
        }
        if (rg == 0 && g == 0) a.act_d[(size_t)(m0 + tok) * (a.N / 32) + tile] = f32_to_f16(d);
      }
  }
}

template <int MT, bool SWIGLU, int G>
cudaError_t run_mma_g(const GemvArgs &a, int sms, cudaStream_t s) {
  using S = MmaShape<MT, SWIGLU, G>;
  const int KB = a.K / 32, tiles = a.N / SI_RT;
  const int grid_y = (a.M + MT - 1) / MT;
  // One wave: with more tiles than two CTAs per SM hold but no more than three
  // do (the 72B QKV projection's 320 tiles), three per SM -- 72 registers and
  // a shallower ring -- instead of a second, nearly empty wave.
  const bool three = G == 2 && S::MINB == 2 && (long)tiles * grid_y > 2L * sms &&
                     (long)tiles * grid_y <= 3L * sms && S::smem(5, KB) <= kMmaCtaBudget3;
  // The deepest ring (5..12 stages) that keeps that many CTAs per SM.
  int ns = kMmaMaxRing;
  const size_t budget = three ? kMmaCtaBudget3 : kMmaCtaBudget;
  while (ns > 5 && S::smem(ns, KB) > budget) --ns;
  const size_t smem = S::smem(ns, KB);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  // Nibbles [tiles*KB blocks][32 rows x 16 B] as (64 x u64, tiles*KB), a box
  // of one CTA's RWS rows; scales [tiles*KB][32] fp16 likewise; activations
  // [M][K] int8 as (K/8 x u64, M).
  CUtensorMap tmN, tmN2, tmS, tmS2, tmX;
  const cuuint64_t dN[2] = {64, (cuuint64_t)tiles * KB}, sN[1] = {512};
  const cuuint32_t bN[2] = {(cuuint32_t)S::RWS * 2, (cuuint32_t)S::CB};
  const cuuint64_t dS[2] = {32, (cuuint64_t)tiles * KB}, sS[1] = {64};
  const cuuint32_t bS[2] = {(cuuint32_t)S::RWS, (cuuint32_t)S::CB};
  const cuuint64_t dX[2] = {(cuuint64_t)a.K / 8, (cuuint64_t)a.M}, sX[1] = {(cuuint64_t)a.K};
  const cuuint32_t bX[2] = {(cuuint32_t)S::CB * 4, (cuuint32_t)MT};
  if (!tma_encode(&tmN, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, a.nib, dN, sN, bN,
                  CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !tma_encode(&tmS, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.scl, dS, sS, bS,
                  CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !tma_encode(&tmX, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, a.xq, dX, sX, bX,
                  CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  if (SWIGLU) {
    if (!tma_encode(&tmN2, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, a.nib2, dN, sN, bN,
                    CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !tma_encode(&tmS2, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.scl2, dS, sS, bS,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  } else {
    tmN2 = tmN;
    tmS2 = tmS;
  }
  constexpr int MB = S::MINB;
  constexpr int MB3 = G == 2 && S::MINB == 2 ? 3 : S::MINB;
  auto kern = (!SWIGLU && a.isum_out) ? k_gemv_mma<MT, SWIGLU, !SWIGLU, MB, G>
              : three                 ? k_gemv_mma<MT, SWIGLU, false, MB3, G>
                                      : k_gemv_mma<MT, SWIGLU, false, MB, G>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(tiles * (2 / G), grid_y);
  return launch_pdl(kern, grid, dim3(mma_warps(G) * 32), smem, s, tmN, tmN2, tmS, tmS2, tmX, a,
                    ns);
}

// Half-tile CTAs (16 rows) for plain projections with fewer tiles than SMs --
// the tensor-parallel QKV shards (1280 rows at TP = 8: 40 tiles) -- so twice
// the CTAs stream the weights; whole tiles otherwise, and always for SwiGLU
// (its Q8 block is a tile's 32 rows), the peer-store mode and the block-sum
// instantiation.
template <int MT, bool SWIGLU>
cudaError_t run_mma(const GemvArgs &a, cudaStream_t s) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long ctas = (long)(a.N / SI_RT) * ((a.M + MT - 1) / MT);
  if constexpr (!SWIGLU) {
    if (a.peer.world == 0 && !a.isum_out && ctas < sms) return run_mma_g<MT, false, 1>(a, sms, s);
  }
  return run_mma_g<MT, SWIGLU, 2>(a, sms, s);
}

template <int MT, int RW, bool SWIGLU>
cudaError_t run(const GemvArgs &a, cudaStream_t s) {
  static_assert(!SWIGLU || RW == SI_RT, "the SwiGLU Q8 epilogue needs whole 32-row tiles");
  using S = Shape<MT, RW>;
  const int KB = a.K / 32, tiles = a.N / SI_RT;
  // Ring depth: the whole slice at once when it fits (the small decode
  // matrices: one memory round trip), else the deepest ring that keeps two
  // CTAs per SM, at least three stages.
  const int nchunks = ((KB + S::CB - 1) / S::CB) * (SWIGLU ? 2 : 1);
  int ns = nchunks < kMaxRing ? nchunks : kMaxRing;
  if (ns < 2) ns = 2;
  while (ns > 3 && S::smem(ns, KB) > kCtaBudget) --ns;
  const size_t smem = S::smem(ns, KB);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  // Nibbles [tiles*KB blocks][32 rows x 16 B] as (64 x u64, tiles*KB); scales
  // [tiles*KB][32] fp16; activations [M][K] int8 as (K/8 x u64, M).
  CUtensorMap tmN, tmN2, tmS, tmS2, tmX;
  const cuuint64_t dN[2] = {64, (cuuint64_t)tiles * KB}, sN[1] = {512};
  const cuuint32_t bN[2] = {(cuuint32_t)RW * 2, (cuuint32_t)S::CB};
  const cuuint64_t dS[2] = {32, (cuuint64_t)tiles * KB}, sS[1] = {64};
  const cuuint32_t bS[2] = {(cuuint32_t)RW, (cuuint32_t)S::CB};
  const cuuint64_t dX[2] = {(cuuint64_t)a.K / 8, (cuuint64_t)a.M}, sX[1] = {(cuuint64_t)a.K};
  const cuuint32_t bX[2] = {(cuuint32_t)S::CB * 4, (cuuint32_t)MT};
  if (!tma_encode(&tmN, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, a.nib, dN, sN, bN,
                  CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !tma_encode(&tmS, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.scl, dS, sS, bS,
                  CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !tma_encode(&tmX, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, a.xq, dX, sX, bX,
                  CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  if (SWIGLU) {
    if (!tma_encode(&tmN2, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, a.nib2, dN, sN, bN,
                    CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !tma_encode(&tmS2, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a.scl2, dS, sS, bS,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
      return cudaErrorInvalidValue;
  } else {
    tmN2 = tmN;
    tmS2 = tmS;
  }
  // One CTA per unit, or -- when the units (row slices) number between one
  // and two CTA slots per SM (two CTAs per SM fit the shared-memory budget) --
  // one CTA per slot, each streaming its units back to back.
  const int units = tiles * (SI_RT / RW);
  int gx = units;
  {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int slots = 2 * sms;
    if (units > slots && units <= 2 * slots) gx = slots;
  }
  auto kern = gx < units ? k_gemv<MT, RW, SWIGLU, true> : k_gemv<MT, RW, SWIGLU, false>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(gx, (a.M + MT - 1) / MT);
  return launch_pdl(kern, grid, dim3(S::THREADS), smem, s, tmN, tmN2, tmS, tmS2, tmX, a, ns);
}

// Row slices per tile: whole 32-row tiles whenever there are enough of them
// for every SM (each CTA then streams one contiguous region: measured 10-20%
// faster than split tiles on the 7B/72B matrices), narrower slices only to
// give matrices with few tiles (the smaller models) enough CTAs.
template <int MT, bool SWIGLU>
cudaError_t pick_rows(const GemvArgs &a, cudaStream_t s) {
  if (SWIGLU) return run<MT, 32, true>(a, s);
  const int tiles = a.N / SI_RT;
  if (tiles < 74) return run<MT, 8, false>(a, s);
  if (tiles < 148) return run<MT, 16, false>(a, s);
  return run<MT, 32, false>(a, s);
}

template <bool SWIGLU>
cudaError_t dispatch(const GemvArgs &a, cudaStream_t s) {
  // The tensor-core form from 3 tokens on (or when asked for); the dp4a form
  // for 1-2 tokens, where its per-token cost is lower than one mma per block.
  const bool mma = a.variant == kGemvMma || (a.variant == kGemvAuto && a.M >= 3) ||
                   a.peer.world > 0;
  if (a.peer.world > 0 && (SWIGLU || a.M > 16)) return cudaErrorInvalidValue;
  if (mma) return a.M <= 8 ? run_mma<8, SWIGLU>(a, s) : run_mma<16, SWIGLU>(a, s);
  if (a.M <= 1) return pick_rows<1, SWIGLU>(a, s);
  if (a.M <= 2) return pick_rows<2, SWIGLU>(a, s);
  if (a.M <= 4) return pick_rows<4, SWIGLU>(a, s);
  return pick_rows<8, SWIGLU>(a, s);
}
}  // namespace

cudaError_t launch_gemv(const GemvArgs &a, bool swiglu, cudaStream_t s) {
  if (a.M <= 0) return cudaSuccess;
  if (!tma_encode_fn()) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(a.nib) | reinterpret_cast<uintptr_t>(a.scl) |
       reinterpret_cast<uintptr_t>(a.xq)) & 15)
    return cudaErrorInvalidValue;
  if (swiglu && ((reinterpret_cast<uintptr_t>(a.nib2) | reinterpret_cast<uintptr_t>(a.scl2)) & 15))
    return cudaErrorInvalidValue;
  return swiglu ? dispatch<true>(a, s) : dispatch<false>(a, s);
}

}  // namespace si
