// attention.cu -- GQA attention with online softmax over the KV cache.
//
// Reference: attention_flash (attention_kernels.h:80-164), one query token per
// call: per head h, group = h / (Hq/Hkv); score_t = (q . k_t) * (1/sqrtf(D)); an
// online max/normaliser; out = sum_t softmax_t * v_t.  The standard variant
// (attention_kernels.h:33-78) computes the same function with materialised scores.
//
// GPU form (flash-decoding): the context of each (query token, KV head) is split
// into nsplit chunks, one CTA per chunk.  A CTA holds the G = Hq/Hkv queries of
// its group in registers (lane = D/32 dims) and streams its chunk of K/V once:
// each K/V row is read once for all G heads.  Warps take tokens round-robin and
// keep their own (max, normaliser, accumulator) per head; the warps, then the
// chunks, are merged with the usual rescaling by exp(m_i - m).  Summation order
// differs from the reference's serial loop, so results agree to fp32 rounding
// (the reference's own standard-vs-flash check uses 1e-5 + 1e-4*|x|).
// The same kernel serves causal prefill: query token t of a prefill sees
// context prefix + t + 1 (prefill_weight_stationary.h:173-177).
#include "si_common.cuh"
#include "si_kernels.cuh"

namespace si {

namespace {
constexpr int kAttnWarps = 4;
constexpr int kMaxGroup = 8;

template <int D, bool KVF32>
struct KvRow;
template <int D>
struct KvRow<D, true> {
  static constexpr int N = D / 32;
  __device__ static void load(const void *base, size_t off, int lane, float (&v)[N]) {
    const float *p = static_cast<const float *>(base) + off + lane * N;
    if constexpr (N == 4) {
      float4 x = __ldg(reinterpret_cast<const float4 *>(p));
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else {
      float2 x = __ldg(reinterpret_cast<const float2 *>(p));
      v[0] = x.x; v[1] = x.y;
    }
  }
};
template <int D>
struct KvRow<D, false> {
  static constexpr int N = D / 32;
  __device__ static void load(const void *base, size_t off, int lane, float (&v)[N]) {
    const uint16_t *p = static_cast<const uint16_t *>(base) + off + lane * N;
    if constexpr (N == 4) {
      uint2 x = __ldg(reinterpret_cast<const uint2 *>(p));
      v[0] = f16_to_f32((uint16_t)x.x); v[1] = f16_to_f32((uint16_t)(x.x >> 16));
      v[2] = f16_to_f32((uint16_t)x.y); v[3] = f16_to_f32((uint16_t)(x.y >> 16));
    } else {
      uint32_t x = __ldg(reinterpret_cast<const uint32_t *>(p));
      v[0] = f16_to_f32((uint16_t)x); v[1] = f16_to_f32((uint16_t)(x >> 16));
    }
  }
};

// Splits of a token's context depend on its own length only (128 keys per
// split, at most 64 splits), never on how many tokens share the launch, so a
// token's attention is bit-identical in a prefill, a batched decode or a
// decode of its own.
constexpr int kSplitKeys = 128, kMaxSplits = 64;
__host__ __device__ __forceinline__ int splits_for(int L) {
  int s = (L + kSplitKeys - 1) / kSplitKeys;
  return s < 1 ? 1 : (s > kMaxSplits ? kMaxSplits : s);
}

template <int D, bool KVF32>
__global__ void __launch_bounds__(kAttnWarps * 32) k_attn_split(const AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  constexpr int N = D / 32;
  const int split = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Hq = a.n_q_heads, Hkv = a.n_kv_heads;
  const int G = Hq / Hkv;
  const int seq = a.tok_seq ? a.tok_seq[t] : a.seq0;
  int L = a.tok_ctx ? a.tok_ctx[t] : a.ctx0 + t;
  L = min(L, a.max_ctx);
  const int ns = splits_for(L);
  if (split >= ns) return;  // this token needs fewer splits than the grid has
  const int chunk = (max(L, 0) + ns - 1) / ns;
  const int j0 = split * chunk, j1 = min(max(L, 0), j0 + chunk);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));

  float q[kMaxGroup][N], o[kMaxGroup][N], m[kMaxGroup], l[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      o[g][i] = 0.0f;
      q[g][i] = g < G ? a.q[((size_t)t * Hq + kvh * G + g) * D + lane * N + i] : 0.0f;
    }
  }
  const size_t rowstride = (size_t)Hkv * D;
  const size_t base = ((size_t)seq * a.max_ctx) * rowstride + (size_t)kvh * D;
  for (int j = j0 + warp; j < j1; j += kAttnWarps) {
    float k[N], v[N];
    KvRow<D, KVF32>::load(a.kc, base + (size_t)j * rowstride, lane, k);
    KvRow<D, KVF32>::load(a.vc, base + (size_t)j * rowstride, lane, v);
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      if (g < G) {
        float p = 0.0f;
#pragma unroll
        for (int i = 0; i < N; ++i) p = fmaf(q[g][i], k[i], p);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) p += __shfl_xor_sync(0xffffffffu, p, off);
        float s = p * scale;
        float mn = fmaxf(m[g], s);
        float corr = expf(m[g] - mn);
        float e = expf(s - mn);
        l[g] = fmaf(l[g], corr, e);
#pragma unroll
        for (int i = 0; i < N; ++i) o[g][i] = fmaf(o[g][i], corr, e * v[i]);
        m[g] = mn;
      }
    }
  }
  // Merge the warps of this CTA.
  __shared__ float sm_m[kAttnWarps][kMaxGroup], sm_l[kAttnWarps][kMaxGroup];
  __shared__ float sm_o[kAttnWarps][kMaxGroup][D];
  if (lane == 0)
    for (int g = 0; g < G; ++g) { sm_m[warp][g] = m[g]; sm_l[warp][g] = l[g]; }
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g)
    if (g < G)
#pragma unroll
      for (int i = 0; i < N; ++i) sm_o[warp][g][lane * N + i] = o[g][i];
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    int g = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_m[w][g]);
    float Ls = 0.0f, Os = 0.0f;
    if (M != -INFINITY)
      for (int w = 0; w < kAttnWarps; ++w) {
        float f = expf(sm_m[w][g] - M);
        Ls = fmaf(sm_l[w][g], f, Ls);
        Os = fmaf(sm_o[w][g][d], f, Os);
      }
    const int h = kvh * G + g;
    if (a.nsplit == 1) {
      a.out[((size_t)t * Hq + h) * D + d] = Ls > 0.0f ? Os / Ls : 0.0f;
    } else {
      float *p = a.part + (((size_t)t * Hq + h) * a.nsplit + split) * (D + 2);
      if (d == 0) { p[0] = M; p[1] = Ls; }
      p[2 + d] = Os;
    }
  }
}

__global__ void k_attn_combine(const AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  const int h = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
  const int D = a.head_dim;
  const int L = min(a.tok_ctx ? a.tok_ctx[t] : a.ctx0 + t, a.max_ctx);
  const int S = splits_for(L);
  const float *p = a.part + ((size_t)t * a.n_q_heads + h) * a.nsplit * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, p[(size_t)s * (D + 2)]);
  float Ls = 0.0f, Os = 0.0f;
  if (M != -INFINITY)
    for (int s = 0; s < S; ++s) {
      const float *ps = p + (size_t)s * (D + 2);
      float f = expf(ps[0] - M);
      Ls = fmaf(ps[1], f, Ls);
      Os = fmaf(ps[2 + d], f, Os);
    }
  a.out[((size_t)t * a.n_q_heads + h) * D + d] = Ls > 0.0f ? Os / Ls : 0.0f;
}

template <int D, bool F32>
cudaError_t run(const AttnArgs &a, cudaStream_t s) {
  dim3 grid(a.nsplit, a.n_kv_heads, a.T);
  cudaError_t e = launch_pdl(k_attn_split<D, F32>, grid, dim3(kAttnWarps * 32), 0, s, a);
  if (e != cudaSuccess || a.nsplit == 1) return e;
  return launch_pdl(k_attn_combine, dim3(a.n_q_heads, a.T), dim3(D), 0, s, a);
}
}  // namespace

size_t attn_part_floats(int T, int n_q_heads, int head_dim, int nsplit) {
  return nsplit > 1 ? (size_t)T * n_q_heads * nsplit * (head_dim + 2) : 0;
}

int attn_pick_splits(int T, int n_kv_heads, int max_len) {
  (void)T;
  (void)n_kv_heads;
  return splits_for(max_len);
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t s) {
  if (a.T <= 0) return cudaSuccess;
  if (a.n_q_heads / a.n_kv_heads > kMaxGroup) return cudaErrorInvalidValue;
  if (a.head_dim == 128) return a.kv_f32 ? run<128, true>(a, s) : run<128, false>(a, s);
  if (a.head_dim == 64) return a.kv_f32 ? run<64, true>(a, s) : run<64, false>(a, s);
  return cudaErrorInvalidValue;
}

}  // namespace si
