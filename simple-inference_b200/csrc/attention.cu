// attention.cu -- GQA attention with online softmax over the KV cache.
//
// Reference: attention_flash (attention_kernels.h:80-164), one query token per
// call: per head h, group = h / (Hq/Hkv); score_t = (q . k_t) * (1/sqrtf(D)); an
// online max/normaliser; out = sum_t softmax_t * v_t.  The standard variant
// (attention_kernels.h:33-78) computes the same function with materialised scores.
// The causal prefill gives query token t of a prefill the context
// prefix + t + 1 (prefill_weight_stationary.h:173-177).
//
// Order of the arithmetic.  Every (query token, head) is evaluated by one fixed
// procedure whatever kernel runs it and however many tokens share the launch,
// so a token's output is bit-identical in a prefill, a batched decode and a
// decode of its own:
//   * keys in sub-tiles of 32 aligned positions, splits of 4 sub-tiles (128);
//   * score = fmaf chain over d = 0..D-1 from 0, times 1/sqrt(D); keys at or
//     past the context length are -inf;
//   * per sub-tile: m = max, p = expf(s - m), l = xor-butterfly sum of p over the
//     32 lanes (16, 8, 4, 2, 1), o[d] = fmaf chain over the keys in order from 0;
//   * the sub-tiles of a split, then the splits, merged in order by
//     M' = max(M, m), a = expf(M - M'), b = expf(m - M'), L = fmaf(L, a, l*b),
//     O = fmaf(O, a, o*b); out = O / L.
// The reference's serial loop sums in another order, so results agree with it
// to fp32 rounding (its own standard-vs-flash check uses 1e-5 + 1e-4*|x|).
//
// Kernels.  Decode (any token count, per-token context lengths): one CTA per
// (split, KV head, token), one warp per sub-tile; a warp stages its 32 K rows
// in shared memory with cp.async (16-byte chunks XOR-swizzled by row so that
// lane = key reads are conflict-free), scores all G = Hq/Hkv heads of the group
// with lane = key, and accumulates P.V with lane = dims straight from the
// V rows (coalesced).  Splits of a token are merged by k_attn_combine.
// Prefill (contiguous tokens of one sequence): one CTA per (64 query rows =
// 64/G tokens x G heads, KV head) walks the splits in order with K and V tiles
// of 128 keys in shared memory, S = Q.K^T and P.V as register-tiled fp32 FMA
// chains (two chains per packed f32x2 FMA), and the same merges, so it needs
// no split scratch.
#include <type_traits>

#include "si_common.cuh"
#include "si_kernels.cuh"
#include "si_tma.cuh"

namespace si {

namespace {
constexpr int kMaxGroup = 8;
constexpr int kSub = 32;           // keys per sub-tile
constexpr int kSplitKeys = 128;    // keys per split
constexpr int kSubPerSplit = kSplitKeys / kSub;
constexpr int kPrefillRows = 64;   // query rows (token x head) per prefill CTA
constexpr int kPrefillThreads = 256;
constexpr int kPrefillMinTokens = 16;

__host__ __device__ __forceinline__ int splits_for(int L) {
  const int s = (L + kSplitKeys - 1) / kSplitKeys;
  return s < 1 ? 1 : s;
}

__device__ __forceinline__ void merge_ml(float &M, float &L, float m, float l, float &a,
                                         float &b) {
  const float Mn = fmaxf(M, m);
  a = expf(__fsub_rn(M, Mn));
  b = expf(__fsub_rn(m, Mn));
  L = fmaf(L, a, __fmul_rn(l, b));
  M = Mn;
}
__device__ __forceinline__ float merge_o(float O, float a, float o, float b) {
  return fmaf(O, a, __fmul_rn(o, b));
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Packed fp32 FMA: each half is one IEEE fused multiply-add with its own
// rounding, exactly as fmaf, two chains per instruction.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Four consecutive elements of a K/V row as floats (fp16 rows convert exactly).
template <bool F32>
__device__ __forceinline__ float4 load4(const void *p) {
  if constexpr (F32) {
    return *reinterpret_cast<const float4 *>(p);
  } else {
    const uint2 x = *reinterpret_cast<const uint2 *>(p);
    return make_float4(f16_to_f32((uint16_t)x.x), f16_to_f32((uint16_t)(x.x >> 16)),
                       f16_to_f32((uint16_t)x.y), f16_to_f32((uint16_t)(x.y >> 16)));
  }
}

__device__ __forceinline__ int ctx_of(const AttnArgs &a, int t) {
  const int L = a.tok_ctx ? a.tok_ctx[t] : a.ctx0 + t;
  return L < a.max_ctx ? L : a.max_ctx;
}

// ---------------------------------------------------------------------------
// decode: one CTA per (split, KV head, token), one warp per sub-tile
// ---------------------------------------------------------------------------
template <int D, bool F32>
struct DecShape {
  static constexpr int ES = F32 ? 4 : 2;
  static constexpr int RB = D * ES;     // bytes per K row
  static constexpr int CPR = RB / 16;   // 16-byte chunks per row (8..32)
  static constexpr int RPI = 32 / CPR;  // rows one warp-wide cp.async covers
  static constexpr int NV = D / 32;     // dims per lane in P.V
  static constexpr int Q = kMaxGroup * D * 4;
  static constexpr int KW = kSub * RB;  // one warp's K rows; later its P, then its O
  static constexpr int PB = kSub * kMaxGroup * 8;  // P as (p, p) pairs per key and head
  static constexpr int bytes() { return Q + kSubPerSplit * KW + kSubPerSplit * kMaxGroup * 8; }
  static_assert(CPR >= 8 && CPR <= 32, "the row swizzle needs 8..32 chunks per row");
  static_assert(KW >= PB && KW >= kMaxGroup * D * 4, "P and O must fit over the K rows");
};

// V row chunk of one lane (NV dims) as floats.
template <int NV, bool F32>
struct VRow {
  using T = typename std::conditional<F32, typename std::conditional<NV == 4, float4, float2>::type,
                                      typename std::conditional<NV == 4, uint2, uint32_t>::type>::type;
  static __device__ __forceinline__ T load(const uint8_t *p) {
    return __ldg(reinterpret_cast<const T *>(p));
  }
  static __device__ __forceinline__ T zero() { return T{}; }
  // NV raw fp32 values in the cache's format (fp16: round to nearest even).
  static __device__ __forceinline__ T from_raw(const float *p) {
    T x;
    if constexpr (F32 && NV == 4) {
      x = make_float4(p[0], p[1], p[2], p[3]);
    } else if constexpr (F32) {
      x = make_float2(p[0], p[1]);
    } else if constexpr (NV == 4) {
      x = make_uint2((uint32_t)f32_to_f16(p[0]) | ((uint32_t)f32_to_f16(p[1]) << 16),
                     (uint32_t)f32_to_f16(p[2]) | ((uint32_t)f32_to_f16(p[3]) << 16));
    } else {
      x = (uint32_t)f32_to_f16(p[0]) | ((uint32_t)f32_to_f16(p[1]) << 16);
    }
    return x;
  }
  static __device__ __forceinline__ void to_f32(const T &x, float (&v)[NV]) {
    if constexpr (F32 && NV == 4) {
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else if constexpr (F32) {
      v[0] = x.x; v[1] = x.y;
    } else if constexpr (NV == 4) {
      v[0] = f16_to_f32((uint16_t)x.x); v[1] = f16_to_f32((uint16_t)(x.x >> 16));
      v[2] = f16_to_f32((uint16_t)x.y); v[3] = f16_to_f32((uint16_t)(x.y >> 16));
    } else {
      v[0] = f16_to_f32((uint16_t)x); v[1] = f16_to_f32((uint16_t)(x >> 16));
    }
  }
};

// One CTA per (split, KV head, head chunk, token), one warp per 32-key
// sub-tile, NP pairs of query heads: the CTA takes heads h0 .. h0 + 2 NP - 1 of
// the KV head's group of G (a head past G computes on zero queries and is
// never written).  Small grids (batch 1-2) split the group into chunks so that
// more CTAs, each with a shorter per-warp chain, share the work; each chunk's
// CTA reads the same K/V rows (the second read hits the L2), and only chunk
// 0 appends the new key.  Every per-key and per-dim loop is unrolled against
// compile-time offsets from a few per-lane bases, and a full sub-tile (the
// common case) runs without per-key predicates; a partial one zero-fills the
// K rows past the context (their scores are masked to -inf, so p = 0) and
// loads no V row there -- fmaf(0, 0, o) == o, so the results equal those of
// skipping the keys.
template <int D, bool F32, int NP>
__global__ void __launch_bounds__(kSubPerSplit * 32) k_attn_dec(const AttnArgs a) {
  using S = DecShape<D, F32>;
  using VR = VRow<S::NV, F32>;
  constexpr int NV = S::NV, NH = 2 * NP;
  extern __shared__ __align__(16) uint8_t smem[];
  float *q_s = reinterpret_cast<float *>(smem);                       // [D][8]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t *k_w = smem + S::Q + warp * S::KW;                           // [32][RB] swizzled
  float2 *ml_s = reinterpret_cast<float2 *>(smem + S::Q + kSubPerSplit * S::KW);  // [4][8]

  pdl_trigger();
  pdl_wait();
  const int Hq = a.n_q_heads, Hkv = a.n_kv_heads, G = Hq / Hkv;
  const int HS = gridDim.y / Hkv;  // head chunks per group
  const int split = blockIdx.x, kvh = blockIdx.y / HS, t = blockIdx.z;
  const int h0 = (blockIdx.y % HS) * NH;  // this CTA's first head in the group
  const int Gc = min(NH, G - h0);         // its heads
  const int seq = a.tok_seq ? a.tok_seq[t] : a.seq0;
  const int L = ctx_of(a, t);
  const int ns = splits_for(L);
  if (split >= ns) return;  // this token needs fewer splits than the grid has
  const int key0 = (split * kSubPerSplit + warp) * kSub;
  const int nvalid = L - key0 < 0 ? 0 : (L - key0 > kSub ? kSub : L - key0);
  // With raw projections, this warp's last valid key is the token's own new
  // key when the sub-tile holds position L - 1: its row comes from the
  // projections, not from the cache.
  const bool fused = a.qkv != nullptr;
  const bool has_new = fused && L - key0 >= 1 && L - key0 <= kSub;
  const int ncache = nvalid - (has_new ? 1 : 0);  // rows read from the cache
  const uint32_t rsb = (uint32_t)Hkv * D * S::ES;  // bytes between positions
  const size_t base = ((size_t)seq * a.max_ctx * Hkv + kvh) * D * S::ES;
  const uint8_t *kg = static_cast<const uint8_t *>(a.kc) + base + (size_t)key0 * rsb;
  const uint8_t *vg = static_cast<const uint8_t *>(a.vc) + base + (size_t)key0 * rsb +
                      lane * NV * S::ES;

  // K rows into shared memory: lane = chunk (lane % CPR) of rows lane / CPR + RPI i,
  // chunks XOR-swizzled by row so that lane = key reads are conflict-free.
  constexpr int NI = kSub / S::RPI;
  // V rows 0..15 of the sub-tile, in flight during the scores, and with an
  // fp16 cache rows 16..31 too (7B step at batch 1 55.5 -> 54.3 us); fp32
  // caches prefetch rows 16..31 to the L2 and load them after the first half
  // (the extra registers cost more there: 0.5B step 25.6 -> 26.0 us).
  constexpr bool kEarlyV = !F32;
  typename VR::T vb[kEarlyV ? 32 : 16];
  if (nvalid > 0) {
    const int c = lane % S::CPR, ro = lane / S::CPR;
    const uint8_t *src = kg + (size_t)ro * rsb + c * 16;
    const uint32_t dst = smem_u32(k_w) + ro * S::RB;
    const uint32_t cr = (uint32_t)(c ^ ro) << 4;
    if (ncache == kSub) {
#pragma unroll
      for (int i = 0; i < NI; ++i)
        cp_async16(dst + i * S::RPI * S::RB + (cr ^ (((S::RPI * i) & 7) << 4)),
                   src + (size_t)(i * S::RPI) * rsb, 16);
#pragma unroll
      for (int k = 0; k < 16; ++k) vb[k] = VR::load(vg + (size_t)k * rsb);
      if constexpr (kEarlyV) {
#pragma unroll
        for (int k = 16; k < 32; ++k) vb[k] = VR::load(vg + (size_t)k * rsb);
      }
    } else {
      // Rows past the cached ones are not copied (their scores are masked, or
      // the new key's row is written below).
#pragma unroll
      for (int i = 0; i < NI; ++i)
        if (ro + i * S::RPI < ncache)
          cp_async16(dst + i * S::RPI * S::RB + (cr ^ (((S::RPI * i) & 7) << 4)),
                     src + (size_t)(i * S::RPI) * rsb, 16);
#pragma unroll
      for (int k = 0; k < 16; ++k) vb[k] = k < ncache ? VR::load(vg + (size_t)k * rsb) : VR::zero();
      if constexpr (kEarlyV) {
#pragma unroll
        for (int k = 16; k < 32; ++k) vb[k] = k < ncache ? VR::load(vg + (size_t)k * rsb) : VR::zero();
      }
    }
    if constexpr (!kEarlyV) {
      // V rows 16..31 into L2 while the scores are computed.
      constexpr int LPR = (S::RB + 127) / 128;  // 128-byte lines per row
      constexpr int RPP = 32 / LPR;             // rows per warp-wide prefetch
      const uint8_t *vrow = static_cast<const uint8_t *>(a.vc) + base +
                            (size_t)(key0 + 16 + lane / LPR) * rsb + (lane % LPR) * 128;
#pragma unroll
      for (int i = 0; i < (16 + RPP - 1) / RPP; ++i)
        if (16 + lane / LPR + i * RPP < ncache)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(vrow + (size_t)(i * RPP) * rsb));
    }
  }
  // The group's queries as [D][8 heads] (heads of one dim adjacent).
  constexpr int HALF = D / 2;
  const size_t qkv_row = (size_t)(Hq + 2 * Hkv) * D;
  // The new key's raw K/V and RoPE factors (used after the staging barrier),
  // requested now so that they arrive with the staged rows.
  constexpr int KP = HALF / 32;  // rotated pairs per lane
  float nc[KP], nsn[KP], nx0[KP], nx1[KP], nvv[D / 32], nvr[NV];
  if (has_new) {
    const int pos = L - 1;
    const float *__restrict__ kraw = a.qkv + (size_t)t * qkv_row + (size_t)Hq * D + (size_t)kvh * D;
    const float *__restrict__ vraw = kraw + (size_t)Hkv * D;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      const int i = lane + 32 * j;
      nc[j] = a.cos_tab[(size_t)pos * HALF + i];
      nsn[j] = a.sin_tab[(size_t)pos * HALF + i];
      nx0[j] = kraw[i];
      nx1[j] = kraw[i + HALF];
    }
#pragma unroll
    for (int j = 0; j < D / 32; ++j) nvv[j] = vraw[lane + 32 * j];
#pragma unroll
    for (int j = 0; j < NV; ++j) nvr[j] = vraw[lane * NV + j];
  }
  if (threadIdx.x < D) {
    const int d = threadIdx.x;
    float qv[kMaxGroup];
    if (fused) {
      // rope (qwen_one_layer.c:171-183) at position L - 1, as rope_kv.cu.
      const int i = d < HALF ? d : d - HALF;
      const size_t ti = (size_t)(L - 1) * HALF + i;
      const float c = a.cos_tab[ti], sn = a.sin_tab[ti];
      const float *qg = a.qkv + (size_t)t * qkv_row + (size_t)(kvh * G + h0) * D + i;
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h) {
        if (h < Gc) {
          const float x0 = qg[(size_t)h * D], x1 = qg[(size_t)h * D + HALF];
          qv[h] = d < HALF ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn))
                           : __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn));
        } else {
          qv[h] = 0.0f;
        }
      }
    } else {
      const float *qg = a.q + ((size_t)t * Hq + (size_t)(kvh * G + h0)) * D + d;
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h) qv[h] = h < Gc ? qg[(size_t)h * D] : 0.0f;
    }
    *reinterpret_cast<float4 *>(q_s + d * kMaxGroup) = make_float4(qv[0], qv[1], qv[2], qv[3]);
    *reinterpret_cast<float4 *>(q_s + d * kMaxGroup + 4) = make_float4(qv[4], qv[5], qv[6], qv[7]);
  }
  cp_async_wait_all();
  __syncthreads();
  // The new key: rotated K and raw V appended to the cache at position L - 1
  // (rope_kv.cu's arithmetic and rounding), the K row also into this warp's
  // staged rows in the cache's format, the lane's V dims kept for P.V.  Only
  // this warp reads its staged rows, so the other warps do not wait for it.
  typename VR::T vnew = VR::zero();
  if (has_new) {
    const int pos = L - 1, r = nvalid - 1;
    const float *c = nc, *sn = nsn, *x0 = nx0, *x1 = nx1, *vv = nvv;
    vnew = VR::from_raw(nvr);
    const size_t o = (((size_t)seq * a.max_ctx + pos) * Hkv + kvh) * D;
    uint8_t *krow = k_w + r * S::RB;
    // (the fused form appends: the cache pointers are written here)
    auto put = [&](int dd, float kval) {  // dim dd: staged row (swizzled) and cache
      const int byte = dd * S::ES;
      uint8_t *p = krow + ((((byte >> 4) ^ (r & 7)) << 4) | (byte & 15));
      if constexpr (F32) {
        *reinterpret_cast<float *>(p) = kval;
        if (h0 == 0) static_cast<float *>(const_cast<void *>(a.kc))[o + dd] = kval;
      } else {
        const uint16_t hb = f32_to_f16(kval);
        *reinterpret_cast<uint16_t *>(p) = hb;
        if (h0 == 0) static_cast<uint16_t *>(const_cast<void *>(a.kc))[o + dd] = hb;
      }
    };
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      const int i = lane + 32 * j;
      put(i, __fsub_rn(__fmul_rn(x0[j], c[j]), __fmul_rn(x1[j], sn[j])));
      put(i + HALF, __fadd_rn(__fmul_rn(x1[j], c[j]), __fmul_rn(x0[j], sn[j])));
    }
    if (h0 == 0) {  // one head chunk appends the new key to the cache
#pragma unroll
      for (int j = 0; j < D / 32; ++j) {
        if constexpr (F32) static_cast<float *>(const_cast<void *>(a.vc))[o + lane + 32 * j] = vv[j];
        else static_cast<uint16_t *>(const_cast<void *>(a.vc))[o + lane + 32 * j] = f32_to_f16(vv[j]);
      }
    }
    if (r < 16) {
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if (k == r) vb[k] = vnew;
    } else if constexpr (kEarlyV) {
#pragma unroll
      for (int k = 16; k < 32; ++k)
        if (k == r) vb[k] = vnew;
    }
    __syncwarp();
  }

  float m[NH], l[NH];
  float2 o2[NH][NV / 2];  // head h, dims (2j, 2j+1) of this lane's NV
#pragma unroll
  for (int h = 0; h < NH; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int j = 0; j < NV / 2; ++j) o2[h][j] = make_float2(0.0f, 0.0f);
  }
  if (nvalid > 0) {
    // Scores, lane = key: heads in pairs (2q, 2q+1), two chains per packed FMA,
    // each in the order d = 0..D-1.
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    float2 s2[NP];
#pragma unroll
    for (int q = 0; q < NP; ++q) s2[q] = make_float2(0.0f, 0.0f);
    // Row `lane`, chunk c sits at byte ((c ^ (lane & 7)) << 4): one base per
    // value of c & 7, the rest compile-time offsets.
    const uint8_t *kr = k_w + lane * S::RB;
    const uint8_t *kb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) kb[j] = kr + ((j ^ (lane & 7)) << 4);
#pragma unroll
    for (int c4 = 0; c4 < D / 4; ++c4) {
      const int byte = c4 * 4 * S::ES, c = byte >> 4;
      const float4 k = load4<F32>(kb[c & 7] + (c & ~7) * 16 + (byte & 15));
      const float kd[4] = {k.x, k.y, k.z, k.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 kk = make_float2(kd[e], kd[e]);
        const float *qd = q_s + (c4 * 4 + e) * kMaxGroup;
        const float4 qa = *reinterpret_cast<const float4 *>(qd);
        s2[0] = fma2(make_float2(qa.x, qa.y), kk, s2[0]);
        if constexpr (NP > 1) s2[1] = fma2(make_float2(qa.z, qa.w), kk, s2[1]);
        if constexpr (NP > 2) {
          const float4 qb = *reinterpret_cast<const float4 *>(qd + 4);
          s2[2] = fma2(make_float2(qb.x, qb.y), kk, s2[2]);
          if constexpr (NP > 3) s2[3] = fma2(make_float2(qb.z, qb.w), kk, s2[3]);
        }
      }
    }
    __syncwarp();  // every lane is done with the K rows: P goes over them
    float2 *p_w = reinterpret_cast<float2 *>(k_w);  // [32 keys][8 heads] as (p, p)
    const bool valid = lane < nvalid;
    float pv[NH];
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      const float sg = (h & 1) ? s2[h >> 1].y : s2[h >> 1].x;
      const float sc = valid ? __fmul_rn(sg, scale) : -INFINITY;
      m[h] = warp_max(sc);
      pv[h] = expf(__fsub_rn(sc, m[h]));
      l[h] = warp_sum(pv[h]);
    }
#pragma unroll
    for (int h = 0; h < NH; h += 2)
      *reinterpret_cast<float4 *>(p_w + lane * kMaxGroup + h) =
          make_float4(pv[h], pv[h], pv[h + 1], pv[h + 1]);
    __syncwarp();
    // P.V, lane = dims NV*lane .. NV*lane+NV-1, keys in order: o[h][d] =
    // fmaf(p[key][h], v[key][d], o[h][d]), dims in packed pairs.
    auto pv_key = [&](int k, const typename VR::T &vx) {
      float v[NV];
      VR::to_f32(vx, v);
      const float4 *pk = reinterpret_cast<const float4 *>(p_w + k * kMaxGroup);
#pragma unroll
      for (int q = 0; q < NP; ++q) {
        const float4 pp = pk[q];  // (p_2q, p_2q, p_2q+1, p_2q+1)
#pragma unroll
        for (int j = 0; j < NV / 2; ++j) {
          const float2 vv = make_float2(v[2 * j], v[2 * j + 1]);
          o2[2 * q][j] = fma2(make_float2(pp.x, pp.y), vv, o2[2 * q][j]);
          o2[2 * q + 1][j] = fma2(make_float2(pp.z, pp.w), vv, o2[2 * q + 1][j]);
        }
      }
    };
#pragma unroll
    for (int k = 0; k < 16; ++k) pv_key(k, vb[k]);
    if constexpr (kEarlyV) {
      if (nvalid > 16) {
#pragma unroll
        for (int k = 16; k < 32; ++k) pv_key(k, vb[k]);
      }
    } else if (nvalid > 16) {
      if (ncache == kSub) {
#pragma unroll
        for (int k = 0; k < 16; ++k) vb[k] = VR::load(vg + (size_t)(16 + k) * rsb);
      } else {
        const int rn = has_new ? nvalid - 1 - 16 : -1;  // the new key's row in this half
#pragma unroll
        for (int k = 0; k < 16; ++k)
          vb[k] = 16 + k < ncache ? VR::load(vg + (size_t)(16 + k) * rsb)
                                  : (k == rn ? vnew : VR::zero());
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) pv_key(16 + k, vb[k]);
    }
  }
  // Merge the sub-tiles of this split in order (warp 0 first).
  __syncwarp();
  float *o_w = reinterpret_cast<float *>(k_w);  // [8][D], over this warp's P
#pragma unroll
  for (int h = 0; h < NH; ++h)
#pragma unroll
    for (int j = 0; j < NV / 2; ++j)
      *reinterpret_cast<float2 *>(o_w + h * D + lane * NV + 2 * j) = o2[h][j];
  if (lane == 0)
#pragma unroll
    for (int h = 0; h < NH; ++h) ml_s[warp * kMaxGroup + h] = make_float2(m[h], l[h]);
  __syncthreads();
  const int nsub = (L - split * kSplitKeys + kSub - 1) / kSub;  // valid sub-tiles, >= 1
  // The merge factors depend on the head only: one thread per head runs the
  // (max, sum) chain once; every output element then applies them.
  float2 *fab = reinterpret_cast<float2 *>(q_s);  // [G][4] (the queries are no longer read)
  __shared__ float2 mls[kMaxGroup];
  if (threadIdx.x < Gc) {
    const int g = threadIdx.x;
    float M = ml_s[g].x, Ls = ml_s[g].y;
    for (int w = 1; w < kSubPerSplit && w < nsub; ++w) {
      float fa, fb;
      merge_ml(M, Ls, ml_s[w * kMaxGroup + g].x, ml_s[w * kMaxGroup + g].y, fa, fb);
      fab[g * kSubPerSplit + w] = make_float2(fa, fb);
    }
    mls[g] = make_float2(M, Ls);
  }
  __syncthreads();
  constexpr int PER = kMaxGroup * D / (kSubPerSplit * 32);  // outputs per thread (8 or 4 x 2)
  const float *ob = reinterpret_cast<const float *>(smem + S::Q);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int idx = threadIdx.x + i * kSubPerSplit * 32;
    const int g = idx / D, d = idx % D;
    if (g < Gc) {
      const float M = mls[g].x, Ls = mls[g].y;
      float O = ob[g * D + d];
      for (int w = 1; w < kSubPerSplit && w < nsub; ++w) {
        const float2 f = fab[g * kSubPerSplit + w];
        O = merge_o(O, f.x, ob[w * (S::KW / 4) + g * D + d], f.y);
      }
      const int h = kvh * G + h0 + g;
      if (a.nsplit == 1) {  // no combine pass follows
        const size_t o = ((size_t)t * Hq + h) * D + d;
        const float y = __fdiv_rn(O, Ls);
        a.out[o] = y;
        if (a.q8_qs) {  // a warp holds 32 consecutive dims of one head: one Q8 block
          uint16_t d16;
          a.q8_qs[o] = q8_lane(y, d16);
          if ((d & 31) == 0) a.q8_d[o / 32] = d16;
        }
      } else {
        float *p = a.part + (((size_t)t * Hq + h) * a.nsplit + split) * (D + 2);
        if (d == 0) { p[0] = M; p[1] = Ls; }
        p[2 + d] = O;
      }
    }
  }
}

__global__ void k_attn_combine(const AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  const int h = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
  const int D = a.head_dim;
  const int S = splits_for(ctx_of(a, t));
  const float *p = a.part + ((size_t)t * a.n_q_heads + h) * a.nsplit * (D + 2);
  // Merge factors per split, the values of the sequential chain M' = max(M, m),
  // a = expf(M - M'), b = expf(m - M'), L = fmaf(L, a, l*b) (merge_ml): the
  // running maxima are a prefix max, so warp 0 computes every split's M, a and
  // b in parallel (a scan over 32 splits at a time); only the L chain stays
  // serial (thread 0).  Every d then applies (a, b) to its O chain in order.
  extern __shared__ float2 fs[];  // [S] (m, l); [S] = final (M, L); then [S] (a, b)
  float2 *fab = fs + S + 1;
  // The first 17 splits' outputs of this d, in flight while the factors are formed.
  const float *po = p + 2 + d;
  float O = po[0];
  float o1[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) o1[j] = 1 + j < S ? po[(size_t)(1 + j) * (D + 2)] : 0.0f;
  for (int s = d; s < S; s += blockDim.x)
    fs[s] = make_float2(p[(size_t)s * (D + 2)], p[(size_t)s * (D + 2) + 1]);
  __syncthreads();
  if (d < 32) {
    float run = -INFINITY;  // M after the splits before this batch of 32
    for (int base = 0; base < S; base += 32) {
      const int s = base + d;
      const float m = s < S ? fs[s].x : -INFINITY;
      float x = m;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if (d >= o) x = fmaxf(x, y);
      }
      const float Ms = fmaxf(run, x);  // M after split s
      float Mp = __shfl_up_sync(0xffffffffu, Ms, 1);
      if (d == 0) Mp = run;            // M before split s
      if (s < S && s > 0) fab[s] = make_float2(expf(__fsub_rn(Mp, Ms)), expf(__fsub_rn(m, Ms)));
      run = __shfl_sync(0xffffffffu, Ms, 31);
    }
    if (d == 0) fs[S].x = run;
  }
  __syncthreads();
  if (d == 0) {  // the normaliser chain, while the other warps merge their O chains
    float Ls = fs[0].y;
    for (int s = 1; s < S; ++s) Ls = fmaf(Ls, fab[s].x, __fmul_rn(fs[s].y, fab[s].y));
    fs[S].y = Ls;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j)
    if (1 + j < S) O = merge_o(O, fab[1 + j].x, o1[j], fab[1 + j].y);
  int s = 17;
  for (; s + 16 <= S; s += 16) {  // sixteen splits' loads in flight, merged in order
    float oo[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) oo[j] = p[(size_t)(s + j) * (D + 2) + 2 + d];
#pragma unroll
    for (int j = 0; j < 16; ++j) O = merge_o(O, fab[s + j].x, oo[j], fab[s + j].y);
  }
  for (; s < S; ++s) O = merge_o(O, fab[s].x, p[(size_t)s * (D + 2) + 2 + d], fab[s].y);
  __syncthreads();  // the normaliser
  const size_t o = ((size_t)t * a.n_q_heads + h) * D + d;
  const float y = __fdiv_rn(O, fs[S].y);
  a.out[o] = y;
  if (a.q8_qs) {  // warp w holds dims 32w .. 32w+31 of the head: one Q8 block
    uint16_t d16;
    a.q8_qs[o] = q8_lane(y, d16);
    if ((d & 31) == 0) a.q8_d[o / 32] = d16;
  }
}

// ---------------------------------------------------------------------------
// prefill: one CTA per (64 query rows, KV head), splits in order
// ---------------------------------------------------------------------------
template <int D, bool F32>
struct PfShape {
  static constexpr int ES = F32 ? 4 : 2;
  static constexpr int KS = D + 16 / ES;            // k row stride (elements), +16 B
  static constexpr int SS = kSplitKeys + 1;         // score row stride (floats)
  static constexpr int Q = D * kPrefillRows * 4;    // queries as [D][64 rows]
  static constexpr int K = kSplitKeys * KS * ES;
  static constexpr int V = kSplitKeys * D * ES;
  static constexpr int SC = kPrefillRows * SS * 4;
  // per row: running (M, L), sub-tile (m, l) x4, sub-tile factors (a, b) x4,
  // split factors (a, b)
  static constexpr int ROW = kPrefillRows * (2 + 8 + 8 + 2) * 4;
  static constexpr int bytes() { return Q + K + V + SC + ROW; }
};

template <int D, bool F32>
__global__ void __launch_bounds__(kPrefillThreads, 1) k_attn_prefill(const AttnArgs a) {
  using S = PfShape<D, F32>;
  constexpr int DG = D / 16;   // dims per thread in P.V (two float4 for D = 128)
  extern __shared__ __align__(16) uint8_t smem[];
  float *q_s = reinterpret_cast<float *>(smem);
  uint8_t *k_s = smem + S::Q;
  uint8_t *v_s = smem + S::Q + S::K;
  float *s_s = reinterpret_cast<float *>(smem + S::Q + S::K + S::V);
  float *rw = reinterpret_cast<float *>(smem + S::Q + S::K + S::V + S::SC);
  float *run_m = rw, *run_l = rw + kPrefillRows;
  float *sub_m = rw + 2 * kPrefillRows, *sub_l = sub_m + 4 * kPrefillRows;
  float *fa_s = sub_l + 4 * kPrefillRows, *fb_s = fa_s + 4 * kPrefillRows;
  float *sa_s = fb_s + 4 * kPrefillRows, *sb_s = sa_s + kPrefillRows;

  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hq = a.n_q_heads, Hkv = a.n_kv_heads, G = Hq / Hkv;
  const int TQ = kPrefillRows / G, R = TQ * G;
  const int tile = gridDim.x - 1 - blockIdx.x;  // longest contexts first
  const int kvh = blockIdx.y;
  const int t0 = tile * TQ;
  const int tlast = min(a.T, t0 + TQ) - 1;
  const int Lmax = min(a.ctx0 + tlast, a.max_ctx);
  const int nsplit = splits_for(Lmax);
  const size_t rowstride = (size_t)Hkv * D;
  const size_t base = (size_t)a.seq0 * a.max_ctx * rowstride + (size_t)kvh * D;
  const uint8_t *kg = static_cast<const uint8_t *>(a.kc) + base * S::ES;
  const uint8_t *vg = static_cast<const uint8_t *>(a.vc) + base * S::ES;
  auto row_ctx = [&](int r) {  // context of row r, 0 for padding rows
    const int t = t0 + r / G;
    return (r < R && t <= tlast) ? min(a.ctx0 + t, a.max_ctx) : 0;
  };

  // Queries transposed to [D][64 rows]: four rows of one dim are one float4.
  for (int i = tid; i < kPrefillRows * D; i += kPrefillThreads) {
    const int r = i % kPrefillRows, d = i / kPrefillRows;
    float v = 0.0f;
    if (row_ctx(r) > 0) {
      const int t = t0 + r / G, h = kvh * G + r % G;
      v = a.q[((size_t)t * Hq + h) * D + d];
    }
    q_s[d * kPrefillRows + r] = v;
  }

  // QK^T tiling: rows 4*rg .. 4*rg+3 (two packed pairs), keys kq + 16j (j < 8).
  const int rg = tid & 15, kq = tid >> 4;
  // P.V tiling: rows rg + 16i, dims dq*4 + 64*jj (jj < DG/4), packed in pairs.
  const int dq = tid >> 4;
  int Lr[4], Lq[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    Lr[i] = row_ctx(rg + 16 * i);
    Lq[i] = row_ctx(4 * rg + i);
  }
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
  float O[4][DG];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < DG; ++j) O[i][j] = 0.0f;

  for (int sp = 0; sp < nsplit; ++sp) {
    const int key0 = sp * kSplitKeys;
    const int nkeys = min(kSplitKeys, Lmax - key0);
    __syncthreads();  // previous split done with the tiles
    constexpr int CPR = D * S::ES / 16;
    for (int i = tid; i < kSplitKeys * CPR; i += kPrefillThreads) {
      const int r = i / CPR, c = i % CPR;
      const bool ok = r < nkeys;
      const size_t off = ((size_t)(ok ? key0 + r : 0) * rowstride) * S::ES + c * 16;
      cp_async16(smem_u32(k_s + r * S::KS * S::ES + c * 16), kg + off, ok ? 16 : 0);
      cp_async16(smem_u32(v_s + r * D * S::ES + c * 16), vg + off, ok ? 16 : 0);
    }
    cp_async_wait_all();
    __syncthreads();

    // Scores: row pairs (4rg, 4rg+1), (4rg+2, 4rg+3) as packed FMA chains.
    {
      float2 acc[2][8];
#pragma unroll
      for (int p2 = 0; p2 < 2; ++p2)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[p2][j] = make_float2(0.0f, 0.0f);
#pragma unroll 2
      for (int c4 = 0; c4 < D / 4; ++c4) {
        float4 q[4], k[8];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          q[e] = *reinterpret_cast<const float4 *>(q_s + (c4 * 4 + e) * kPrefillRows + 4 * rg);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          k[j] = load4<F32>(k_s + ((kq + 16 * j) * S::KS + c4 * 4) * S::ES);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 qa = make_float2(q[e].x, q[e].y), qb = make_float2(q[e].z, q[e].w);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float kv = e == 0 ? k[j].x : (e == 1 ? k[j].y : (e == 2 ? k[j].z : k[j].w));
            const float2 kk = make_float2(kv, kv);
            acc[0][j] = fma2(qa, kk, acc[0][j]);
            acc[1][j] = fma2(qb, kk, acc[1][j]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int key = kq + 16 * j;
          const float sv = (i & 1) ? acc[i >> 1][j].y : acc[i >> 1][j].x;
          s_s[(4 * rg + i) * S::SS + key] = key0 + key < Lq[i] ? __fmul_rn(sv, scale) : -INFINITY;
        }
    }
    __syncthreads();

    // Sub-tile softmax, lane = key: warp w takes rows 8w .. 8w+7, the four
    // sub-tiles of a row at once so their shuffle chains overlap.
#pragma unroll 1
    for (int rr = 0; rr < 8; ++rr) {
      const int r = warp * 8 + rr;
      const int Lrow = row_ctx(r);
      float *srow = s_s + r * S::SS;
      float sc[kSubPerSplit], mx[kSubPerSplit], p[kSubPerSplit], ls[kSubPerSplit];
#pragma unroll
      for (int u = 0; u < kSubPerSplit; ++u) mx[u] = sc[u] = srow[u * kSub + lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < kSubPerSplit; ++u)
          mx[u] = fmaxf(mx[u], __shfl_xor_sync(0xffffffffu, mx[u], o));
#pragma unroll
      for (int u = 0; u < kSubPerSplit; ++u) ls[u] = p[u] = expf(__fsub_rn(sc[u], mx[u]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < kSubPerSplit; ++u)
          ls[u] = __fadd_rn(ls[u], __shfl_xor_sync(0xffffffffu, ls[u], o));
#pragma unroll
      for (int u = 0; u < kSubPerSplit; ++u) {
        const bool live = key0 + u * kSub < Lrow;  // else the sub-tile is all masked
        srow[u * kSub + lane] = live ? p[u] : 0.0f;
        if (live && lane == 0) { sub_m[r * 4 + u] = mx[u]; sub_l[r * 4 + u] = ls[u]; }
      }
    }
    __syncthreads();
    // Merge factors per row: sub-tiles of this split, then the split itself.
    if (tid < kPrefillRows) {
      const int r = tid, Lrow = row_ctx(r);
      if (key0 < Lrow) {
        float M = sub_m[r * 4], Ls = sub_l[r * 4];
        for (int u = 1; u < kSubPerSplit && key0 + u * kSub < Lrow; ++u)
          merge_ml(M, Ls, sub_m[r * 4 + u], sub_l[r * 4 + u], fa_s[r * 4 + u], fb_s[r * 4 + u]);
        if (sp == 0) {
          run_m[r] = M;
          run_l[r] = Ls;
        } else {
          float rm = run_m[r], rl = run_l[r];
          merge_ml(rm, rl, M, Ls, sa_s[r], sb_s[r]);
          run_m[r] = rm;
          run_l[r] = rl;
        }
      }
    }
    __syncthreads();

    // P.V per sub-tile, merged into the split, then into the running output.
    float Os[4][DG];
    for (int u = 0; u < kSubPerSplit && key0 + u * kSub < Lmax; ++u) {
      float2 acc2[4][DG / 2];  // dim pairs as packed FMA chains
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < DG / 2; ++j) acc2[i][j] = make_float2(0.0f, 0.0f);
#pragma unroll 4
      for (int k = 0; k < kSub; ++k) {
        const int kk = u * kSub + k;
        float p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = s_s[(rg + 16 * i) * S::SS + kk];
#pragma unroll
        for (int jj = 0; jj < DG / 4; ++jj) {
          const float4 v = load4<F32>(v_s + (kk * D + dq * 4 + 64 * jj) * S::ES);
          const float2 va = make_float2(v.x, v.y), vb = make_float2(v.z, v.w);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 pp = make_float2(p[i], p[i]);
            acc2[i][jj * 2] = fma2(pp, va, acc2[i][jj * 2]);
            acc2[i][jj * 2 + 1] = fma2(pp, vb, acc2[i][jj * 2 + 1]);
          }
        }
      }
      float acc[4][DG];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < DG / 2; ++j) {
          acc[i][2 * j] = acc2[i][j].x;
          acc[i][2 * j + 1] = acc2[i][j].y;
        }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = rg + 16 * i;
        if (key0 + u * kSub < Lr[i]) {
          if (u == 0) {
#pragma unroll
            for (int j = 0; j < DG; ++j) Os[i][j] = acc[i][j];
          } else {
            const float fa = fa_s[r * 4 + u], fb = fb_s[r * 4 + u];
#pragma unroll
            for (int j = 0; j < DG; ++j) Os[i][j] = merge_o(Os[i][j], fa, acc[i][j], fb);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = rg + 16 * i;
      if (key0 < Lr[i]) {
        if (sp == 0) {
#pragma unroll
          for (int j = 0; j < DG; ++j) O[i][j] = Os[i][j];
        } else {
          const float fa = sa_s[r], fb = sb_s[r];
#pragma unroll
          for (int j = 0; j < DG; ++j) O[i][j] = merge_o(O[i][j], fa, Os[i][j], fb);
        }
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = rg + 16 * i;
    if (Lr[i] > 0) {
      const int t = t0 + r / G, h = kvh * G + r % G;
      const float Ls = run_l[r];
      float *out = a.out + ((size_t)t * Hq + h) * D;
#pragma unroll
      for (int jj = 0; jj < DG / 4; ++jj) {
        float4 y;
        y.x = __fdiv_rn(O[i][jj * 4 + 0], Ls);
        y.y = __fdiv_rn(O[i][jj * 4 + 1], Ls);
        y.z = __fdiv_rn(O[i][jj * 4 + 2], Ls);
        y.w = __fdiv_rn(O[i][jj * 4 + 3], Ls);
        *reinterpret_cast<float4 *>(out + dq * 4 + 64 * jj) = y;
      }
    }
  }
}

bool use_prefill(const AttnArgs &a) { return !a.tok_ctx && !a.tok_seq && a.T >= kPrefillMinTokens; }

template <class K>
cudaError_t with_smem(K kern, int bytes) {
  return bytes > 48 * 1024
             ? cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)
             : cudaSuccess;
}

template <int D, bool F32>
cudaError_t run(const AttnArgs &a, cudaStream_t s) {
  if (use_prefill(a)) {
    using P = PfShape<D, F32>;
    const int G = a.n_q_heads / a.n_kv_heads, TQ = kPrefillRows / G;
    cudaError_t e = with_smem(k_attn_prefill<D, F32>, P::bytes());
    if (e != cudaSuccess) return e;
    return launch_pdl(k_attn_prefill<D, F32>, dim3((a.T + TQ - 1) / TQ, a.n_kv_heads),
                      dim3(kPrefillThreads), P::bytes(), s, a);
  }
  using Sd = DecShape<D, F32>;
  const int G = a.n_q_heads / a.n_kv_heads;
  // Heads per CTA: the whole group, or chunks of 2 or 4 heads when the launch
  // is latency-bound -- at most 16 MB of K/V (each chunk's CTA reads the rows
  // again) and at most eight CTAs per SM.  Measured on B200 (graph replays):
  // 7B step at batch 1 61.4 -> 57.2 us, at batch 2 72.5 -> 67.8 us; the
  // TP = 8 shard at batch 8 (35 MB of fp32 K/V) 560 -> 576 us when chunked,
  // so it is not.
  int np = (G + 1) / 2;
  const double kv_bytes =
      (double)a.nsplit * kSplitKeys * a.n_kv_heads * a.T * Sd::RB * 2.0;
  if (kv_bytes <= 16e6) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long base = (long)a.nsplit * a.n_kv_heads * a.T;
    for (int c : {1, 2})
      if (c < np && base * ((G + 2 * c - 1) / (2 * c)) <= 8L * sms) {
        np = c;
        break;
      }
  }
  const int hs = (G + 2 * np - 1) / (2 * np);  // head chunks per group
  auto kern = np == 1 ? k_attn_dec<D, F32, 1>
              : np == 2 ? k_attn_dec<D, F32, 2>
              : np == 3 ? k_attn_dec<D, F32, 3> : k_attn_dec<D, F32, 4>;
  cudaError_t e = with_smem(kern, Sd::bytes());
  if (e != cudaSuccess) return e;
  e = launch_pdl(kern, dim3(a.nsplit, a.n_kv_heads * hs, a.T), dim3(kSubPerSplit * 32),
                 Sd::bytes(), s, a);
  if (e != cudaSuccess || a.nsplit == 1) return e;
  return launch_pdl(k_attn_combine, dim3(a.n_q_heads, a.T), dim3(D),
                    (size_t)(2 * a.nsplit + 1) * sizeof(float2), s, a);
}
}  // namespace

bool attn_decode_form(const AttnArgs &a) { return !use_prefill(a); }

size_t attn_part_floats(int T, int n_q_heads, int head_dim, int nsplit) {
  return nsplit > 1 ? (size_t)T * n_q_heads * nsplit * (head_dim + 2) : 0;
}

int attn_pick_splits(int T, bool decode_form, int max_len) {
  // The prefill kernel walks the splits itself; the decode kernel needs the
  // largest split count of the launch.
  if (!decode_form && T >= kPrefillMinTokens) return 1;
  return splits_for(max_len);
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t s) {
  if (a.T <= 0) return cudaSuccess;
  if (a.n_kv_heads <= 0 || a.n_q_heads % a.n_kv_heads ||
      a.n_q_heads / a.n_kv_heads > kMaxGroup)
    return cudaErrorInvalidValue;
  if (!use_prefill(a) && a.nsplit < splits_for(a.tok_ctx ? 1 : min(a.ctx0 + a.T - 1, a.max_ctx)))
    return cudaErrorInvalidValue;
  if (a.qkv ? (use_prefill(a) || !a.cos_tab || !a.sin_tab) : !a.q) return cudaErrorInvalidValue;
  if (a.head_dim == 128) return a.kv_f32 ? run<128, true>(a, s) : run<128, false>(a, s);
  if (a.head_dim == 64) return a.kv_f32 ? run<64, true>(a, s) : run<64, false>(a, s);
  return cudaErrorInvalidValue;
}

}  // namespace si
