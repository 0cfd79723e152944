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

__global__ void k_rope_kv(const RopeKvArgs a) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int D = a.head_dim, half = D / 2;
  const int Hq = a.n_q_heads, Hkv = a.n_kv_heads;
  const int QD = Hq * D, KVD = Hkv * D;
  const int seq = a.tok_seq ? a.tok_seq[t] : a.seq0;
  const int pos = a.tok_pos ? a.tok_pos[t] : a.pos0 + t;
  const float *row = a.qkv + (size_t)t * (QD + 2 * KVD);
  // Positions are validated on the host; an out-of-table position is never
  // dereferenced (the row is left unrotated and nothing is appended).
  if (pos < 0 || pos >= a.max_positions) return;
  const float *ct = a.cos_tab + (size_t)pos * half;
  const float *st = a.sin_tab + (size_t)pos * half;
  // Rotated queries.
  for (int idx = threadIdx.x; idx < Hq * half; idx += blockDim.x) {
    int h = idx / half, i = idx % half;
    float x0 = row[h * D + i], x1 = row[h * D + i + half];
    float c = ct[i], s = st[i];
    float *q = a.q_out + (size_t)t * QD + h * D;
    q[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    q[i + half] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
  }
  if (!a.kc || pos >= a.max_ctx) return;  // rotation only (reference rope()), or no cache slot
  const size_t slot = ((size_t)seq * a.max_ctx + pos) * KVD;
  for (int idx = threadIdx.x; idx < Hkv * half; idx += blockDim.x) {
    int h = idx / half, i = idx % half;
    const float *k = row + QD + h * D;
    const float *v = row + QD + KVD + h * D;
    float x0 = k[i], x1 = k[i + half];
    float c = ct[i], s = st[i];
    float k0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    float k1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    size_t o = slot + (size_t)h * D + i;
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
}

cudaError_t launch_rope_kv(const RopeKvArgs &a, cudaStream_t s) {
  if (a.T <= 0) return cudaSuccess;
  return launch_pdl(k_rope_kv, dim3(a.T), dim3(256), 0, s, a);
}

}  // namespace si
