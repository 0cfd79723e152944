/*
 * si_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, single-threaded CPU restatement of the keyvan-dadash/simple-inference
 * block arithmetic for the Qwen decoder-layer hot path, generalised over the model
 * dimensions.  It is the checker that the CUDA path is compared against.  Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may
 * load it; the product library (libsi_b200.so) never links or calls it.
 *
 * Each function names the reference file:line whose expressions it restates, in
 * the same evaluation order, and is compiled with -ffp-contract=off exactly like
 * the reference (Makefile:7) so float rounding is identical.  At the reference's
 * compile-time 1.5B dims the restatement is checked bit-for-bit against the
 * reference translation unit itself (oracle/_ref, built by oracle/Makefile) and
 * against the golden vectors under tests/golden/.
 *
 * Parts with no reference implementation (SwiGLU MLP, residual adds, fp32 KV
 * cache, Q4_0 weight quantiser) follow the same conventions but their parity is
 * pinned only by this restatement.
 */
#ifndef SI_ORACLE_H
#define SI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OC_QK 32
#define OC_Q4_BYTES 18
#define OC_Q8_BYTES 34

/* Model dimensions; the reference fixes these at compile time (defines.h:16-25). */
typedef struct {
    int hidden;        /* H */
    int n_q_heads;     /* Hq */
    int n_kv_heads;    /* Hkv */
    int head_dim;      /* D */
    int intermediate;  /* I (SwiGLU), 0 = attention sublayer only */
    float rope_theta;  /* 1e6 */
    float rms_eps;     /* 1e-6 */
} oc_dims;

/* One decoder layer; Q4_0 matrices are GGUF row-major [rows][K/32] x 18 B.
 * Optional vectors may be NULL (identity norm / zero bias), as in
 * qwen_one_layer.c:216-219. */
typedef struct {
    const uint8_t *wq, *wk, *wv, *wo;
    const float *norm, *bq, *bk, *bv;
    const uint8_t *w_gate, *w_up, *w_down;  /* [I][H], [I][H], [H][I] */
    const float *norm2;
} oc_layer;

/* L1 numeric primitives -- qwen_one_layer.c:42-86 */
float oc_f16_to_f32(uint16_t h);
uint16_t oc_f32_to_f16(float x);

/* Q8_0 activation quantiser -- qwen_one_layer.c:98-116.  dst holds count/32
 * reference-layout blocks of 34 bytes (fp16 d, 32 x int8). Returns -1 if count%32. */
int oc_quantize_q8(const float *src, uint8_t *dst, int count);

/* GGUF Q4_0 x Q8_0 block dot -- qwen_one_layer.c:118-146 (portable branch). */
int32_t oc_dot_32_q4q8(const uint8_t *w_block, const int8_t *a);

/* Row-major GEMV -- qwen_one_layer.c:148-162. */
void oc_matvec_q4q8(const uint8_t *weights, const uint8_t *q8_input,
                    int inputs, int outputs, const float *bias, float *out);

/* The per-(row, block) int32 partial sums the GEMV combines: isum[row*KB + b]. */
void oc_block_isums(const uint8_t *weights, const uint8_t *q8_input,
                    int inputs, int outputs, int32_t *isum);

/* RMSNorm -- qwen_one_layer.c:164-169 (fp64 sum of squares). */
void oc_rmsnorm(const float *input, const float *weight, float *out, int n, float eps);

/* RoPE rotate_half -- qwen_one_layer.c:171-183. */
void oc_rope(float *heads, int nheads, int position, int head_dim, float theta);
/* cos/sin table rows [pos][head_dim/2] for positions [pos0, pos0+npos), the
 * expressions of qwen_one_layer.c:176-177 and register_fusion.h:364-369. */
void oc_rope_table(int pos0, int npos, int head_dim, float theta, float *cos_out, float *sin_out);

/* GQA decode attention over a KV cache laid out [pos][Hkv][D]; kv_f32 selects
 * fp32 (1) or fp16 (0) storage.  attention_kernels.h:80-164 (flash) and
 * attention_kernels.h:33-78 (standard; scores is Hq*context floats). */
void oc_attention_flash(const oc_dims *d, const float *q, const void *kc, const void *vc,
                        int kv_f32, int context, float *out);
void oc_attention_flash_heads(const oc_dims *dm, const float *q, const void *kc,
                              const void *vc, int kv_f32, int context, float *out, int h0,
                              int h1);
void oc_attention_standard(const oc_dims *d, const float *q, const void *kc, const void *vc,
                           int kv_f32, int context, float *out, float *scores);

/* Staged attention-sublayer decode for one token -- qwen_one_layer.c:237-281:
 * rmsnorm -> Q8 -> Wq/Wk/Wv(+bias) -> RoPE(q,k) -> KV append at slot context-1
 * -> attention -> Q8 -> Wo (no bias, no residual).  method 0 = standard,
 * 1 = flash.  Captures may be NULL.  q8_capture receives H/32 blocks. */
void oc_run_layer(const oc_dims *d, const oc_layer *l, const float *x,
                  void *kc, void *vc, int kv_f32, int context, float *out,
                  int method, float *scores, float *attn_capture, uint8_t *q8_capture);

/* SwiGLU MLP (not in the reference): rmsnorm(norm2) -> Q8 -> gate,up ->
 * silu(gate)*up -> Q8 -> down.  out = down projection only. */
void oc_mlp(const oc_dims *d, const oc_layer *l, const float *h, float *out,
            float *act_capture, uint8_t *q8_capture);

/* Full decoder layer for one token: h = x + attn(x); y = h + mlp(h). */
void oc_decoder_layer(const oc_dims *d, const oc_layer *l, const float *x,
                      void *kc, void *vc, int kv_f32, int context, float *y);

/* Causal prefill by sequential decode (bench_ai_dma_prefill.c:104-108): token t
 * uses context prefix+t+1.  full_layer 0 = attention sublayer (run_layer),
 * 1 = decoder layer.  x, y: [ntok][H]. */
void oc_prefill_sequential(const oc_dims *d, const oc_layer *l, const float *x, int ntok,
                           int prefix, void *kc, void *vc, int kv_f32, float *y, int full_layer);

/* Column-SoA tile GEMV -- fused_layer.h:169-245 (portable branch); tile format
 * of repack_weights.py:55-75 (per group: 32 x 128 B nibble columns + 256 fp32). */
void oc_fused_column_matvec(const uint8_t *tile, const uint8_t *q8_input, int nblocks,
                            const float *bias_lo, const float *bias_hi, float *output, int add);
/* Build one column-SoA tile exactly as repack_weights.py:55-75. */
void oc_pack_colsoa_tile(uint8_t *out, const uint8_t *low_src, const uint8_t *high_src,
                         int src_cols, int low_base, int high_base, int input_base, int nblocks);

/* Q4_0 weight quantiser for synthetic weights (ggml/GGUF rule): d = (signed
 * value of max|x|)/-8 stored fp16, q = min(15, (int)(x*(1/d) + 8.5)). */
void oc_quantize_q4_0(const float *w, uint8_t *dst, int rows, int k);

/* The reference's synthetic generator, qwen_one_layer.c:88-96. */
void oc_rng_seed(uint32_t s);
float oc_random_float(void);
/* dst[i] = oc_random_float() * scale + offset for i < n (same stream). */
void oc_random_fill(float *dst, size_t n, float scale, float offset);

#ifdef __cplusplus
}
#endif
#endif
