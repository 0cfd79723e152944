// si_kernels.cuh -- internal launch interface between the C ABI (si_api.cu)
// and the kernel translation units.  Not installed; plain pointers only.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace si {

// Row-parallel tensor parallelism: where a GEMV's partial sums go instead of
// `out` -- every rank's receive slot.  Each rank holds one symmetric buffer
// whose receive slots [2 parities][world][slot] of 8-byte words start at
// kPeerData; a word is (float bits | epoch << 32), stored in one 8-byte
// write, so a reader that sees this call's epoch in a word has its value (no
// fence and no separate flag).  The 4 KB below kPeerData is control space.
constexpr int kPeerMaxWorld = 8;
constexpr size_t kPeerData = 4096;
struct PeerOut {
  char *base[kPeerMaxWorld];  // each rank's buffer as mapped in this process (own included)
  int world;                  // 0: no peer output
  int rank;
  int slot;                   // words per receive slot (>= M * N)
  unsigned long long epoch;   // this call's number (1, 2, ...), or its offset from
                              // *epoch_base; the parity picks the slot set
  const unsigned long long *epoch_base;  // device counter added to epoch, or null
};

// The call's effective epoch, read after griddepcontrol.wait (the counter is
// advanced by an earlier kernel of the stream).
__device__ __forceinline__ unsigned long long peer_epoch(const PeerOut &p) {
  return p.epoch + (p.epoch_base ? *p.epoch_base : 0ull);
}


// ---- layout.cu -------------------------------------------------------------
// GGUF Q4_0 rows [rows][KB] x 18 B  ->  row-tile SoA: nib [rows/32][KB][32][16]
// (each byte XOR 0x88) and scl [rows/32][KB][32] fp16.
cudaError_t launch_repack_gguf(const uint8_t *gguf, int rows, int KB, uint8_t *nib,
                               uint16_t *scl, cudaStream_t s);
cudaError_t launch_unpack_to_gguf(const uint8_t *nib, const uint16_t *scl, int rows, int KB,
                                  uint8_t *gguf, cudaStream_t s);
// Seeded synthetic Q4_0 rows [row0, row0+rows) x blocks [cb0, cb0+KB) of a
// matrix with full_KB blocks per row (0: full_KB = KB), written to a matrix of
// exactly `rows` x KB blocks.
cudaError_t launch_synth_q4(int rows, int KB, uint64_t seed, float std, uint8_t *nib,
                            uint16_t *scl, cudaStream_t s, int row0 = 0, int cb0 = 0,
                            int full_KB = 0);
// Elements [i0, i0+n) of a seeded N(mean, std) vector.
cudaError_t launch_synth_f32(float *dst, size_t n, uint64_t seed, float mean, float std,
                             cudaStream_t s, size_t i0 = 0);
cudaError_t launch_synth_kv(void *dst, size_t n, int f32, uint64_t seed, float std,
                            cudaStream_t s);
cudaError_t launch_q8_to_blocks(const int8_t *qs, const uint16_t *d, int M, int K,
                                uint8_t *blocks, cudaStream_t s);
cudaError_t launch_q8_from_blocks(const uint8_t *blocks, int M, int K, int8_t *qs, uint16_t *d,
                                  cudaStream_t s);

// Column-SoA tiles of repack_weights.py -> row-tile SoA rows [row0, row0+nrows)
// of a matrix with KB blocks per row.  kind 0 = Q pair tiles, 1 = K|V group
// tiles (destination: kv_rows K rows then kv_rows V rows), 2 = O pair x output
// subtiles of a model with `hidden` outputs.
cudaError_t launch_colsoa_to_rt(const uint8_t *tiles, int kind, int nrows, int row0, int KB,
                                int hidden, size_t tile_bytes, int kv_rows, uint8_t *nib,
                                uint16_t *scl, cudaStream_t s);
// fused_column_matvec on one column-SoA tile: out[256] (+)= blocks in order.
cudaError_t launch_colsoa_matvec(const uint8_t *tile, const uint8_t *x_blocks, int nblocks,
                                 const float *bias_lo, const float *bias_hi, float *out, int add,
                                 cudaStream_t s);

// ---- norm_q8.cu -------------------------------------------------------------
cudaError_t launch_q8_quantize(const float *x, int M, int K, int8_t *qs, uint16_t *d,
                               cudaStream_t s);
// With rp (tensor parallelism, decode): x is the residual and the row is
// first h = x + the sum over ranks (rank order) of the receive slots of
// rp->p.epoch (each word waited for, bounded); h is written to rp->h_out and
// normalised.
struct RmsPeer {
  PeerOut p;
  float *h_out;
  unsigned long long timeout_ns;
  int *err;
};
cudaError_t launch_rmsnorm_q8(const float *x, const float *w, int M, int n, float eps,
                              float *out, int8_t *qs, uint16_t *d, cudaStream_t s,
                              const RmsPeer *rp = nullptr);
// y = a + b elementwise (residual), fp32, round-to-nearest.
cudaError_t launch_add(const float *a, const float *b, float *y, size_t n, cudaStream_t s);

// ---- gemv.cu ----------------------------------------------------------------
struct GemvArgs {
  const uint8_t *nib;      // row-tile nibbles of the (first) matrix
  const uint16_t *scl;     // row-tile scales
  const uint8_t *nib2;     // second matrix (SwiGLU "up"), same shape
  const uint16_t *scl2;
  int N, K;                // rows, inputs
  const int8_t *xq;        // activations [M][K]
  const uint16_t *xd;      // [M][K/32] fp16 scales
  int M;
  const float *bias;       // [N] or null
  const float *resid;      // [M][N] added after the block sum, or null
  float *out;              // [M][N] fp32 (non-SwiGLU), or SwiGLU fp32 act (optional)
  int8_t *act_qs;          // SwiGLU: Q8 of silu(gate)*up, [M][N]
  uint16_t *act_d;         // [M][N/32]
  int32_t *isum_out;       // [M][N][K/32] block partial sums (parity), or null
  int *err;                // context device error word (bounded waits), or null
  float *scratch;          // tcgen05 GEMM: gemm_tc_scratch_bytes() of device memory
  int variant;             // GEMV form: kGemvAuto, kGemvDp4a or kGemvMma
  int fused_rescale;       // tcgen05 GEMM: acc = fma(round(isum*dw), dx, acc) (one rounding
                           // fewer per block; within 1e-5) instead of the exact two roundings
  PeerOut peer;            // tensor-core form only: partial sums to every rank's slot
};
enum { kGemvAuto = 0, kGemvDp4a = 1, kGemvMma = 2 };
cudaError_t launch_gemv(const GemvArgs &a, bool swiglu, cudaStream_t s);

// ---- gemv_gguf.cu (row-major GGUF Q4_0, no repack) ------------------------------
// out[M][N] = bias + blocks in order, from GGUF rows [N][K/32] x 18 B; K % 128,
// 1 <= M <= 8; w and xq 16-byte aligned.
bool gemv_gguf_supported(int N, int K, int M);
cudaError_t launch_gemv_gguf(const uint8_t *w, int N, int K, const int8_t *xq, const uint16_t *xd,
                             int M, const float *bias, float *out, cudaStream_t s);

// ---- gemm_tc.cu (tcgen05) ------------------------------------------------------
cudaError_t launch_gemm_tc(const GemvArgs &a, bool swiglu, cudaStream_t s);
bool gemm_tc_supported(int N, int K, int M);
// Activation scales fp16 [M][KB] -> fp32 [KB][round_up(M, 4)] (zero padded).
cudaError_t launch_scales_t(const uint16_t *xd, int M, int KB, float *dT, cudaStream_t s);

// ---- gemm_mma.cu (mma.sync, many tokens) ----------------------------------------
// Same results and scratch as the tcgen05 GEMM; N % 128 (SwiGLU: % 64), K % 32.
cudaError_t launch_gemm_mma(const GemvArgs &a, bool swiglu, cudaStream_t s);
bool gemm_mma_supported(int N, int K, int M, bool swiglu);
// Scratch the GEMM needs for its transposed fp32 activation scales.
size_t gemm_tc_scratch_bytes(int K, int M);

// ---- tc_peak.cu (int8 tensor-core throughput probe) ---------------------------
// One CTA per SM, `iters` x 4 tcgen05 kind::i8 MMAs of 128 x n x 32 each (n =
// 128 or 256); *ops = int8 operations per launch, *ctas = CTAs launched;
// sink needs one int per SM.
cudaError_t launch_tc_i8_peak(int n, int iters, int *err, int *sink, int *ctas, double *ops,
                              cudaStream_t s);

// ---- rope_kv.cu -------------------------------------------------------------
struct RopeKvArgs {
  const float *qkv;      // [T][QD + 2*KVD] projections (bias included)
  float *q_out;          // [T][QD] rotated queries
  void *kc, *vc;         // caches [B][max_ctx][Hkv][D]
  int kv_f32;
  int T, n_q_heads, n_kv_heads, head_dim, max_ctx;
  const int *tok_pos;    // [T] device positions (decode) or null
  const int *tok_seq;    // [T] device sequence ids (decode) or null
  int seq0, pos0;        // prefill: seq = seq0, pos = pos0 + t
  const float *cos_tab, *sin_tab;  // [max_positions][D/2]
  int max_positions;
};
cudaError_t launch_rope_kv(const RopeKvArgs &a, cudaStream_t s);
// Decode-step index arrays [seq T][pos T][ctx T] (pos = ctx - 1).
constexpr int kIdxMaxByValue = 256;
struct IdxParams {
  int T;
  int seq[kIdxMaxByValue];
  int ctx[kIdxMaxByValue];
};
cudaError_t launch_set_idx(const IdxParams &p, int *idx, cudaStream_t s);
// All positions / lengths + 1, bounded by max_ctx (SI_ERR_INVALID past it).
cudaError_t launch_advance_idx(int *idx, int T, int max_ctx, int *err, cudaStream_t s);

// ---- attention.cu -----------------------------------------------------------
struct AttnArgs {
  const float *q;        // [T][Hq][D] (after RoPE)
  const void *kc, *vc;   // [B][max_ctx][Hkv][D]
  int kv_f32;
  int T, n_q_heads, n_kv_heads, head_dim, max_ctx;
  const int *tok_seq;    // [T] device, or null (then seq0)
  const int *tok_ctx;    // [T] device context lengths, or null (then ctx0 + t)
  int seq0, ctx0;
  float *out;            // [T][Hq][D]
  float *part;           // split-K scratch, >= attn_part_floats() floats
  int nsplit;
  int *err;              // context device error word (bounded waits), or null
  // Decode form only: also the Q8_0 pair of out ([T][Hq*D] int8 and one fp16
  // scale per 32), written by the kernel that writes out; null: out only.
  int8_t *q8_qs;
  uint16_t *q8_d;
  // Decode form only, with distinct sequences per token: the raw projections
  // [T][QD + 2*KVD] instead of q.  The kernel then rotates the queries itself
  // and appends each token's rotated K and raw V at position ctx - 1 (the
  // RoPE of rope_kv.cu, the same tables), so no separate RoPE kernel runs.
  const float *qkv;
  const float *cos_tab, *sin_tab;  // [positions][D/2]
};
size_t attn_part_floats(int T, int n_q_heads, int head_dim, int nsplit);
// Splits the launch needs: 1 when the prefill kernel runs (contiguous tokens
// of one sequence, T >= 16), else ceil(max_len / 128).
int attn_pick_splits(int T, bool decode_form, int max_len);
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t s);
// True when launch_attention runs the decode form (per-token arrays, or
// fewer than 16 tokens): the only form that honours q8_qs / q8_d.
bool attn_decode_form(const AttnArgs &a);

// ---- attention_tc.cu (tcgen05 causal prefill, split fp16 operands) ------------
// The prefill form (no per-token arrays) at head_dim 128 and groups <= 8.
bool attn_tc_supported(const AttnArgs &a);
// Scratch for the operand splits (Q, K and V^T as fp16 hi / lo halves).
size_t attn_tc_scratch_bytes(const AttnArgs &a);
cudaError_t launch_attention_tc(const AttnArgs &a, void *scratch, size_t scratch_bytes,
                                cudaStream_t s);

// ---- tp_peer.cu --------------------------------------------------------------
// y[i] = resid[i] + sum over ranks (in rank order) of the receive slots of
// epoch `epoch`, each word waited for (bounded by timeout_ns) until it
// carries the epoch.
cudaError_t launch_tp_combine(const PeerOut &p, const float *resid, float *y, size_t n,
                              unsigned long long timeout_ns, int *err, cudaStream_t s);
// *counter += n: the exchanges of a finished step move the epoch base on.
cudaError_t launch_epoch_advance(unsigned long long *counter, unsigned n, cudaStream_t s);

}  // namespace si
