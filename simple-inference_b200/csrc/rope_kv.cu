// rope_kv.cu -- RoPE (rotate_half, theta 1e6) on Q and K, and the KV-cache append.
//
// Reference: rope (qwen_one_layer.c:171-183) pairs d with d+D/2:
//   v[i] = a*c - b*s ; v[i+D/2] = b*c + a*s   (four separately rounded products)
// with c, s = cosf/sinf((float)pos / powf(theta, (float)(2i)/D)).  The angles
// are evaluated on the host with the same libm calls (the reference itself
// precomputes them for its register-fused path, register_fusion.h:364-369) and
// passed in as tables, so the rotation here is bit-identical.
// KV append (qwen_one_layer.c:262-266): the rotated K and the raw V of each
// token are stored at its slot as fp16 (round-to-nearest-even) or fp32.
#include "si_common.cuh"
#include "si_kernels.cuh"

namespace si {

// One thread per rotated pair: grid (T, ceil((Hq + Hkv) * D/2 / 256)); pairs
// [0, Hq*D/2) are query pairs, the rest key pairs (each also moves V's pair).
__global__ void __launch_bounds__(256) k_rope_kv(const RopeKvArgs a) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int D = a.head_dim, half = D / 2;
  const int Hq = a.n_q_heads, Hkv = a.n_kv_heads;
  const int QD = Hq * D, KVD = Hkv * D;
  const int idx = blockIdx.y * blockDim.x + threadIdx.x;
  if (idx >= (Hq + Hkv) * half) return;
  const int seq = a.tok_seq ? a.tok_seq[t] : a.seq0;
  const int pos = a.tok_pos ? a.tok_pos[t] : a.pos0 + t;
  const float *row = a.qkv + (size_t)t * (QD + 2 * KVD);
  // Positions are validated on the host; an out-of-table position is never
  // dereferenced (the row is left unrotated and nothing is appended).
  if (pos < 0 || pos >= a.max_positions) return;
  const int h = idx / half, i = idx % half;
  const float c = a.cos_tab[(size_t)pos * half + i], s = a.sin_tab[(size_t)pos * half + i];
  if (h < Hq) {  // rotated query
    const float x0 = row[h * D + i], x1 = row[h * D + i + half];
    float *q = a.q_out + (size_t)t * QD + h * D;
    q[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    q[i + half] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    return;
  }
  if (!a.kc || pos >= a.max_ctx) return;  // rotation only (reference rope()), or no cache slot
  const int kh = h - Hq;
  const float *k = row + QD + kh * D;
  const float *v = row + QD + KVD + kh * D;
  const float x0 = k[i], x1 = k[i + half];
  const float k0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  const float k1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
  const size_t o = ((size_t)seq * a.max_ctx + pos) * KVD + (size_t)kh * D + i;
  if (a.kv_f32) {
    float *kc = static_cast<float *>(a.kc), *vc = static_cast<float *>(a.vc);
    kc[o] = k0; kc[o + half] = k1;
    vc[o] = v[i]; vc[o + half] = v[i + half];
  } else {
    uint16_t *kc = static_cast<uint16_t *>(a.kc), *vc = static_cast<uint16_t *>(a.vc);
    kc[o] = f32_to_f16(k0); kc[o + half] = f32_to_f16(k1);
    vc[o] = f32_to_f16(v[i]); vc[o + half] = f32_to_f16(v[i + half]);
  }
}

// Per-token index arrays of a decode step, [seq T][pos T][ctx T], written from
// kernel parameters (no host staging buffer, no host synchronisation).
__global__ void k_set_idx(const IdxParams p, int *__restrict__ idx) {
  pdl_trigger();
  pdl_wait();
  for (int t = threadIdx.x; t < p.T; t += blockDim.x) {
    idx[t] = p.seq[t];
    idx[p.T + t] = p.ctx[t] - 1;
    idx[2 * p.T + t] = p.ctx[t];
  }
}

// One decode step later: every position and context length + 1.  A length that
// would pass max_ctx stays where it is and records SI_ERR_INVALID (1).
__global__ void k_advance_idx(int *__restrict__ idx, int T, int max_ctx, int *err) {
  pdl_trigger();
  pdl_wait();
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const int c = idx[2 * T + t];
    if (c + 1 > max_ctx) {
      raise_error(err, 1);
      continue;
    }
    idx[T + t] = c;
    idx[2 * T + t] = c + 1;
  }
}

cudaError_t launch_set_idx(const IdxParams &p, int *idx, cudaStream_t s) {
  if (p.T <= 0 || p.T > kIdxMaxByValue) return cudaErrorInvalidValue;
  return launch_pdl(k_set_idx, dim3(1), dim3(256), 0, s, p, idx);
}

cudaError_t launch_advance_idx(int *idx, int T, int max_ctx, int *err, cudaStream_t s) {
  return launch_pdl(k_advance_idx, dim3(1), dim3(256), 0, s, idx, T, max_ctx, err);
}

cudaError_t launch_rope_kv(const RopeKvArgs &a, cudaStream_t s) {
  if (a.T <= 0) return cudaSuccess;
  const int pairs = (a.n_q_heads + a.n_kv_heads) * (a.head_dim / 2);
  return launch_pdl(k_rope_kv, dim3(a.T, (pairs + 255) / 256), dim3(256), 0, s, a);
}

}  // namespace si
