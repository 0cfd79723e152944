/*
 * ref_shim.c -- TEST INFRASTRUCTURE ONLY.
 *
 * Builds the UNMODIFIED reference translation unit (qwen_one_layer.c and the
 * headers it includes, read in place from the reference checkout given by -I)
 * with its portable C path (-DUSE_RVV=0) and exports thin non-static wrappers
 * so tests can call the reference's own static kernels through ctypes.  This
 * is the reference's own "include the TU, rename main" pattern
 * (verify_fused_projections.c:17-19).  Nothing from the reference is copied
 * into this repository; oracle/Makefile writes the result to oracle/_ref/.
 */
#define main si_reference_qwen_main_unused
#include "qwen_one_layer.c"
#undef main

#define REF_API __attribute__((visibility("default")))

REF_API void ref_dims(int *out) {
    out[0] = HIDDEN; out[1] = QHEADS; out[2] = KVHEADS; out[3] = HDIM; out[4] = QK;
}
REF_API float ref_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
REF_API uint16_t ref_f32_to_f16(float x) { return f32_to_f16(x); }
REF_API void ref_quantize_q8(const float *src, void *dst, int count) {
    quantize_q8(src, (block_q8_0 *)dst, count);
}
REF_API int32_t ref_dot_32_q4q8(const uint8_t *w, const int8_t *a) { return dot_32_q4q8(w, a); }
REF_API void ref_matvec_q4q8(const uint8_t *w, const void *x, int inputs, int outputs,
                             const float *bias, float *out) {
    matvec_q4q8(w, (const block_q8_0 *)x, inputs, outputs, bias, out);
}
REF_API void ref_rmsnorm(const float *in, const float *w, float *out) { rmsnorm(in, w, out); }
REF_API void ref_rope(float *heads, int nheads, int pos) { rope(heads, nheads, pos); }
REF_API void ref_attention_flash(const float *q, const uint16_t *kc, const uint16_t *vc,
                                 int context, float *out) {
    attention_flash(q, kc, vc, context, out);
}
REF_API void ref_attention_standard(const float *q, const uint16_t *kc, const uint16_t *vc,
                                    int context, float *out, float *scores) {
    attention_standard(q, kc, vc, context, out, scores);
}

static layer_t ref_make_layer(uint8_t *wq, uint8_t *wk, uint8_t *wv, uint8_t *wo,
                              float *norm, float *bq, float *bk, float *bv) {
    layer_t l;
    l.wq = wq; l.wk = wk; l.wv = wv; l.wo = wo;
    l.norm = norm; l.bq = bq; l.bk = bk; l.bv = bv;
    return l;
}

REF_API void ref_run_layer(uint8_t *wq, uint8_t *wk, uint8_t *wv, uint8_t *wo,
                           float *norm, float *bq, float *bk, float *bv,
                           const float *x, uint16_t *kc, uint16_t *vc, int context,
                           float *out, int method, float *scores,
                           float *attn_copy, void *q8_copy) {
    layer_t l = ref_make_layer(wq, wk, wv, wo, norm, bq, bk, bv);
    (void)run_layer(&l, x, kc, vc, context, out, (attention_method_t)method, scores,
                    attn_copy, (block_q8_0 *)q8_copy);
}

REF_API void ref_fused_column_matvec(const uint8_t *tile, const void *x, int nblocks,
                                     const float *blo, const float *bhi, float *out, int add) {
    fused_column_matvec(tile, (const block_q8_0 *)x, nblocks, blo, bhi, out, add);
}

REF_API void ref_fused_attention_pair(const float *qpair, const uint16_t *kc, const uint16_t *vc,
                                      int context, int group, float *opair) {
    fused_attention_pair(qpair, kc, vc, context, group, opair);
}

/* run_layer_fused falls back to run_layer_legacy_fused without RVV
 * (register_fusion.h:409-410); tcm_tile stays NULL so no device is touched. */
REF_API void ref_run_layer_fused(uint8_t *wq, uint8_t *wk, uint8_t *wv, uint8_t *wo,
                                 float *norm, float *bq, float *bk, float *bv,
                                 uint8_t *q_colsoa, uint8_t *kv_colsoa, uint8_t *o_colsoa,
                                 const float *x, uint16_t *kc, uint16_t *vc, int context,
                                 float *out, float *attn_capture, void *q8_capture) {
    layer_t l = ref_make_layer(wq, wk, wv, wo, norm, bq, bk, bv);
    fused_weights_t fw;
    memset(&fw, 0, sizeof(fw));
    fw.q = q_colsoa; fw.kv = kv_colsoa; fw.o = o_colsoa; fw.tcm_fd = -1;
    (void)run_layer_fused(&l, &fw, x, kc, vc, context, out, attn_capture,
                          (block_q8_0 *)q8_capture);
}

REF_API void ref_seed(uint32_t s) { rng_state = s; }
REF_API float ref_random_float(void) { return random_float(); }
REF_API void ref_fill_kv_history(uint16_t *kc, uint16_t *vc, int context) {
    fill_kv_history(kc, vc, context);
}
