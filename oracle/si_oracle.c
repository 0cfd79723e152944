/*
 * si_oracle.c -- TEST INFRASTRUCTURE ONLY (see si_oracle.h).
 *
 * CPU restatement of the reference's portable C hot path, dims-parametrised.
 * Build with -O2 -std=c11 -ffp-contract=off (as the reference, Makefile:7) so
 * that every float expression rounds exactly as the reference's does.
 */
#include "si_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static uint32_t oc_bits(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static float oc_float(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* qwen_one_layer.c:42-59: exact half -> float, subnormals normalised. */
float oc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exponent = (h >> 10) & 31u;
    uint32_t mant = h & 1023u;
    if (exponent == 0) {
        if (mant == 0) return oc_float(sign);
        int e = -14;
        while ((mant & 1024u) == 0) { mant <<= 1; --e; }
        mant &= 1023u;
        return oc_float(sign | ((uint32_t)(e + 127) << 23) | (mant << 13));
    }
    if (exponent == 31) return oc_float(sign | 0x7f800000u | (mant << 13));
    return oc_float(sign | ((exponent + 112u) << 23) | (mant << 13));
}

/* qwen_one_layer.c:61-86: round-to-nearest-even float -> half with subnormals,
 * overflow to infinity and quiet NaN. */
uint16_t oc_f32_to_f16(float x) {
    uint32_t b = oc_bits(x);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    uint32_t mant = b & 0x7fffffu;
    uint32_t biased = (b >> 23) & 255u;
    int e = (int)biased - 127 + 15;
    if (biased == 255u) return (uint16_t)(sign | (mant ? 0x7e00u : 0x7c00u));
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t m = mant | 0x800000u;
        int shift = 14 - e;
        uint32_t frac = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (frac & 1u))) ++frac;
        return (uint16_t)(sign | frac);
    }
    uint32_t r = mant + 0xfffu + ((mant >> 13) & 1u);
    if (r & 0x800000u) {
        ++e;
        r = 0;
        if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    }
    return (uint16_t)(sign | ((uint16_t)e << 10) | (r >> 13));
}

static uint16_t oc_rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void oc_wr16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* qwen_one_layer.c:98-116.  d is kept in fp32 for the reciprocal; only its
 * fp16 rounding is stored. */
int oc_quantize_q8(const float *src, uint8_t *dst, int count) {
    if (count % OC_QK) return -1;
    for (int b = 0; b < count / OC_QK; ++b) {
        const float *x = src + (size_t)b * OC_QK;
        uint8_t *blk = dst + (size_t)b * OC_Q8_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < OC_QK; ++j) {
            float a = fabsf(x[j]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        oc_wr16(blk, oc_f32_to_f16(d));
        float inv = d == 0.0f ? 0.0f : 1.0f / d;
        for (int j = 0; j < OC_QK; ++j) {
            long q = lrintf(x[j] * inv);
            if (q > 127) q = 127;
            if (q < -127) q = -127;
            blk[2 + j] = (uint8_t)(int8_t)q;
        }
    }
    return 0;
}

/* qwen_one_layer.c:137-144: low nibble of byte j is element j, high nibble
 * element j+16; both offset by 8. */
int32_t oc_dot_32_q4q8(const uint8_t *w_block, const int8_t *a) {
    int32_t acc = 0;
    for (int j = 0; j < 16; ++j) {
        uint8_t q = w_block[2 + j];
        acc += ((int32_t)(q & 15) - 8) * a[j];
        acc += ((int32_t)(q >> 4) - 8) * a[j + 16];
    }
    return acc;
}

/* qwen_one_layer.c:148-162: bias-initialised, blocks summed in order as
 * ((float)isum * dw) * dx. */
void oc_matvec_q4q8(const uint8_t *weights, const uint8_t *q8_input,
                    int inputs, int outputs, const float *bias, float *out) {
    int nb = inputs / OC_QK;
    for (int row = 0; row < outputs; ++row) {
        const uint8_t *wrow = weights + (size_t)row * nb * OC_Q4_BYTES;
        float acc = bias ? bias[row] : 0.0f;
        for (int b = 0; b < nb; ++b) {
            const uint8_t *wb = wrow + (size_t)b * OC_Q4_BYTES;
            const uint8_t *xb = q8_input + (size_t)b * OC_Q8_BYTES;
            int32_t isum = oc_dot_32_q4q8(wb, (const int8_t *)(xb + 2));
            acc += (float)isum * oc_f16_to_f32(oc_rd16(wb)) * oc_f16_to_f32(oc_rd16(xb));
        }
        out[row] = acc;
    }
}

void oc_block_isums(const uint8_t *weights, const uint8_t *q8_input,
                    int inputs, int outputs, int32_t *isum) {
    int nb = inputs / OC_QK;
    for (int row = 0; row < outputs; ++row)
        for (int b = 0; b < nb; ++b)
            isum[(size_t)row * nb + b] = oc_dot_32_q4q8(
                weights + ((size_t)row * nb + b) * OC_Q4_BYTES,
                (const int8_t *)(q8_input + (size_t)b * OC_Q8_BYTES + 2));
}

/* qwen_one_layer.c:164-169. */
void oc_rmsnorm(const float *input, const float *weight, float *out, int n, float eps) {
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += (double)input[i] * input[i];
    float inv = 1.0f / sqrtf((float)(ss / n) + eps);
    for (int i = 0; i < n; ++i) out[i] = input[i] * inv * (weight ? weight[i] : 1.0f);
}

/* qwen_one_layer.c:171-183. */
void oc_rope(float *heads, int nheads, int position, int head_dim, float theta) {
    int half = head_dim / 2;
    for (int h = 0; h < nheads; ++h) {
        float *v = heads + (size_t)h * head_dim;
        for (int i = 0; i < half; ++i) {
            float angle = (float)position / powf(theta, (float)(2 * i) / head_dim);
            float c = cosf(angle), s = sinf(angle);
            float a = v[i], b = v[i + half];
            v[i] = a * c - b * s;
            v[i + half] = b * c + a * s;
        }
    }
}

void oc_rope_table(int pos0, int npos, int head_dim, float theta, float *cos_out, float *sin_out) {
    int half = head_dim / 2;
    for (int p = 0; p < npos; ++p)
        for (int i = 0; i < half; ++i) {
            float angle = (float)(pos0 + p) / powf(theta, (float)(2 * i) / head_dim);
            cos_out[(size_t)p * half + i] = cosf(angle);
            sin_out[(size_t)p * half + i] = sinf(angle);
        }
}

static inline float oc_kv(const void *base, size_t idx, int kv_f32) {
    return kv_f32 ? ((const float *)base)[idx]
                  : oc_f16_to_f32(((const uint16_t *)base)[idx]);
}

/* attention_kernels.h:80-164: one exp per token, branch on a new maximum. */
void oc_attention_flash_heads(const oc_dims *dm, const float *q, const void *kc,
                              const void *vc, int kv_f32, int context, float *out, int h0,
                              int h1) {
    const int D = dm->head_dim, Hq = dm->n_q_heads, Hkv = dm->n_kv_heads;
    const float scale = 1.0f / sqrtf((float)D);
    const size_t stride = (size_t)Hkv * D;
    for (int h = h0; h < h1 && h < Hq; ++h) {
        const int group = h / (Hq / Hkv);
        const float *qh = q + (size_t)h * D;
        float *oh = out + (size_t)h * D;
        if (context <= 0) { memset(oh, 0, (size_t)D * sizeof(float)); continue; }
        size_t kb = (size_t)group * D;
        float score = 0.0f;
        for (int d = 0; d < D; ++d) score += qh[d] * oc_kv(kc, kb + d, kv_f32);
        float mx = score * scale;
        float norm = 1.0f;
        for (int d = 0; d < D; ++d) oh[d] = oc_kv(vc, kb + d, kv_f32);
        for (int t = 1; t < context; ++t) {
            kb += stride;
            score = 0.0f;
            for (int d = 0; d < D; ++d) score += qh[d] * oc_kv(kc, kb + d, kv_f32);
            score *= scale;
            if (score > mx) {
                const float alpha = expf(mx - score);
                norm = norm * alpha + 1.0f;
                for (int d = 0; d < D; ++d) oh[d] = oh[d] * alpha + oc_kv(vc, kb + d, kv_f32);
                mx = score;
            } else {
                const float beta = expf(score - mx);
                norm += beta;
                for (int d = 0; d < D; ++d) oh[d] += beta * oc_kv(vc, kb + d, kv_f32);
            }
        }
        const float inv = 1.0f / norm;
        for (int d = 0; d < D; ++d) oh[d] *= inv;
    }
}

/* The whole layer's heads; heads are independent, so the host baseline may
 * also call oc_attention_flash_heads on disjoint head ranges in parallel. */
void oc_attention_flash(const oc_dims *dm, const float *q, const void *kc, const void *vc,
                        int kv_f32, int context, float *out) {
    oc_attention_flash_heads(dm, q, kc, vc, kv_f32, context, out, 0, dm->n_q_heads);
}

/* attention_kernels.h:33-78: materialised scores, softmax, then P*V. */
void oc_attention_standard(const oc_dims *dm, const float *q, const void *kc, const void *vc,
                           int kv_f32, int context, float *out, float *scores) {
    const int D = dm->head_dim, Hq = dm->n_q_heads, Hkv = dm->n_kv_heads;
    const float inv_sqrt = 1.0f / sqrtf((float)D);
    for (int h = 0; h < Hq; ++h) {
        const int group = h / (Hq / Hkv);
        const float *qh = q + (size_t)h * D;
        float *row = scores + (size_t)h * context;
        for (int t = 0; t < context; ++t) {
            size_t kb = ((size_t)t * Hkv + group) * D;
            float dot = 0.0f;
            for (int d = 0; d < D; ++d) dot += qh[d] * oc_kv(kc, kb + d, kv_f32);
            row[t] = dot * inv_sqrt;
        }
    }
    for (int h = 0; h < Hq; ++h) {
        float *row = scores + (size_t)h * context;
        float m = -INFINITY;
        for (int t = 0; t < context; ++t) m = fmaxf(m, row[t]);
        float denom = 0.0f;
        for (int t = 0; t < context; ++t) { row[t] = expf(row[t] - m); denom += row[t]; }
        const float inv = 1.0f / denom;
        for (int t = 0; t < context; ++t) row[t] *= inv;
    }
    for (int h = 0; h < Hq; ++h) {
        const int group = h / (Hq / Hkv);
        const float *row = scores + (size_t)h * context;
        float *oh = out + (size_t)h * D;
        memset(oh, 0, (size_t)D * sizeof(float));
        for (int t = 0; t < context; ++t) {
            size_t vb = ((size_t)t * Hkv + group) * D;
            const float p = row[t];
            for (int d = 0; d < D; ++d) oh[d] += p * oc_kv(vc, vb + d, kv_f32);
        }
    }
}

static void oc_kv_store(void *base, size_t idx, float v, int kv_f32) {
    if (kv_f32) ((float *)base)[idx] = v;
    else ((uint16_t *)base)[idx] = oc_f32_to_f16(v);
}

/* qwen_one_layer.c:237-281. */
void oc_run_layer(const oc_dims *dm, const oc_layer *l, const float *x,
                  void *kc, void *vc, int kv_f32, int context, float *out,
                  int method, float *scores, float *attn_capture, uint8_t *q8_capture) {
    const int H = dm->hidden, D = dm->head_dim;
    const int QD = dm->n_q_heads * D, KVD = dm->n_kv_heads * D;
    float *normed = malloc((size_t)H * sizeof(float));
    float *q = malloc((size_t)QD * sizeof(float));
    float *k = malloc((size_t)KVD * sizeof(float));
    float *v = malloc((size_t)KVD * sizeof(float));
    float *attn = malloc((size_t)QD * sizeof(float));
    uint8_t *inq8 = malloc((size_t)H / OC_QK * OC_Q8_BYTES);
    uint8_t *attq8 = malloc((size_t)QD / OC_QK * OC_Q8_BYTES);
    float *own_scores = NULL;
    if (!method && !scores) scores = own_scores = malloc((size_t)dm->n_q_heads * context * sizeof(float));

    oc_rmsnorm(x, l->norm, normed, H, dm->rms_eps);
    oc_quantize_q8(normed, inq8, H);
    oc_matvec_q4q8(l->wq, inq8, H, QD, l->bq, q);
    oc_matvec_q4q8(l->wk, inq8, H, KVD, l->bk, k);
    oc_matvec_q4q8(l->wv, inq8, H, KVD, l->bv, v);
    oc_rope(q, dm->n_q_heads, context - 1, D, dm->rope_theta);
    oc_rope(k, dm->n_kv_heads, context - 1, D, dm->rope_theta);
    size_t slot = (size_t)(context - 1) * KVD;
    for (int i = 0; i < KVD; ++i) {
        oc_kv_store(kc, slot + i, k[i], kv_f32);
        oc_kv_store(vc, slot + i, v[i], kv_f32);
    }
    if (method) oc_attention_flash(dm, q, kc, vc, kv_f32, context, attn);
    else oc_attention_standard(dm, q, kc, vc, kv_f32, context, attn, scores);
    oc_quantize_q8(attn, attq8, QD);
    oc_matvec_q4q8(l->wo, attq8, QD, H, NULL, out);
    if (attn_capture) memcpy(attn_capture, attn, (size_t)QD * sizeof(float));
    if (q8_capture) memcpy(q8_capture, attq8, (size_t)QD / OC_QK * OC_Q8_BYTES);
    free(normed); free(q); free(k); free(v); free(attn); free(inq8); free(attq8); free(own_scores);
}

void oc_mlp(const oc_dims *dm, const oc_layer *l, const float *h, float *out,
            float *act_capture, uint8_t *q8_capture) {
    const int H = dm->hidden, I = dm->intermediate;
    float *normed = malloc((size_t)H * sizeof(float));
    float *gate = malloc((size_t)I * sizeof(float));
    float *up = malloc((size_t)I * sizeof(float));
    uint8_t *hq8 = malloc((size_t)H / OC_QK * OC_Q8_BYTES);
    uint8_t *aq8 = malloc((size_t)I / OC_QK * OC_Q8_BYTES);
    oc_rmsnorm(h, l->norm2, normed, H, dm->rms_eps);
    oc_quantize_q8(normed, hq8, H);
    oc_matvec_q4q8(l->w_gate, hq8, H, I, NULL, gate);
    oc_matvec_q4q8(l->w_up, hq8, H, I, NULL, up);
    for (int i = 0; i < I; ++i) {
        float g = gate[i];
        float s = g / (1.0f + expf(-g));
        gate[i] = s * up[i];
    }
    oc_quantize_q8(gate, aq8, I);
    oc_matvec_q4q8(l->w_down, aq8, I, H, NULL, out);
    if (act_capture) memcpy(act_capture, gate, (size_t)I * sizeof(float));
    if (q8_capture) memcpy(q8_capture, aq8, (size_t)I / OC_QK * OC_Q8_BYTES);
    free(normed); free(gate); free(up); free(hq8); free(aq8);
}

void oc_decoder_layer(const oc_dims *dm, const oc_layer *l, const float *x,
                      void *kc, void *vc, int kv_f32, int context, float *y) {
    const int H = dm->hidden;
    float *attn = malloc((size_t)H * sizeof(float));
    float *h = malloc((size_t)H * sizeof(float));
    float *mlp = malloc((size_t)H * sizeof(float));
    oc_run_layer(dm, l, x, kc, vc, kv_f32, context, attn, 1, NULL, NULL, NULL);
    for (int i = 0; i < H; ++i) h[i] = x[i] + attn[i];
    if (dm->intermediate > 0) {
        oc_mlp(dm, l, h, mlp, NULL, NULL);
        for (int i = 0; i < H; ++i) y[i] = h[i] + mlp[i];
    } else {
        memcpy(y, h, (size_t)H * sizeof(float));
    }
    free(attn); free(h); free(mlp);
}

void oc_prefill_sequential(const oc_dims *dm, const oc_layer *l, const float *x, int ntok,
                           int prefix, void *kc, void *vc, int kv_f32, float *y, int full_layer) {
    for (int t = 0; t < ntok; ++t) {
        const float *xt = x + (size_t)t * dm->hidden;
        float *yt = y + (size_t)t * dm->hidden;
        if (full_layer) oc_decoder_layer(dm, l, xt, kc, vc, kv_f32, prefix + t + 1, yt);
        else oc_run_layer(dm, l, xt, kc, vc, kv_f32, prefix + t + 1, yt, 1, NULL, NULL, NULL);
    }
}

/* fused_layer.h:220-244 (portable branch). */
void oc_fused_column_matvec(const uint8_t *tile, const uint8_t *q8_input, int nblocks,
                            const float *bias_lo, const float *bias_hi, float *output, int add) {
    if (!add)
        for (int j = 0; j < 128; ++j) {
            output[j] = bias_lo ? bias_lo[j] : 0.0f;
            output[j + 128] = bias_hi ? bias_hi[j] : 0.0f;
        }
    for (int b = 0; b < nblocks; ++b) {
        const uint8_t *group = tile + (size_t)b * 5120u;
        float scales[256];
        memcpy(scales, group + 4096, sizeof(scales));
        const uint8_t *xb = q8_input + (size_t)b * OC_Q8_BYTES;
        int32_t sums[256] = {0};
        for (int k = 0; k < OC_QK; ++k) {
            int xv = (int8_t)xb[2 + k];
            const uint8_t *col = group + (size_t)k * 128u;
            for (int j = 0; j < 128; ++j) {
                sums[j] += ((int)(col[j] & 15) - 8) * xv;
                sums[j + 128] += ((int)(col[j] >> 4) - 8) * xv;
            }
        }
        float dx = oc_f16_to_f32(oc_rd16(xb));
        for (int j = 0; j < 256; ++j) output[j] += ((float)sums[j] * scales[j]) * dx;
    }
}

/* repack_weights.py:43-75. */
static int oc_nibble(const uint8_t *src, int cols, int row, int col) {
    size_t pos = ((size_t)row * (cols / OC_QK) + col / OC_QK) * OC_Q4_BYTES;
    int k = col % OC_QK;
    uint8_t byte = src[pos + 2 + k % 16];
    return k < 16 ? (byte & 15) : (byte >> 4);
}

void oc_pack_colsoa_tile(uint8_t *out, const uint8_t *low_src, const uint8_t *high_src,
                         int src_cols, int low_base, int high_base, int input_base, int nblocks) {
    for (int b = 0; b < nblocks; ++b) {
        uint8_t *group = out + (size_t)b * 5120u;
        int in_block = input_base + b * OC_QK;
        for (int k = 0; k < OC_QK; ++k)
            for (int j = 0; j < 128; ++j)
                group[k * 128 + j] = (uint8_t)(oc_nibble(low_src, src_cols, low_base + j, in_block + k) |
                                               (oc_nibble(high_src, src_cols, high_base + j, in_block + k) << 4));
        for (int j = 0; j < 128; ++j) {
            size_t lo = ((size_t)(low_base + j) * (src_cols / OC_QK) + in_block / OC_QK) * OC_Q4_BYTES;
            size_t hi = ((size_t)(high_base + j) * (src_cols / OC_QK) + in_block / OC_QK) * OC_Q4_BYTES;
            float sl = oc_f16_to_f32(oc_rd16(low_src + lo));
            float sh = oc_f16_to_f32(oc_rd16(high_src + hi));
            memcpy(group + 4096 + 4 * j, &sl, 4);
            memcpy(group + 4096 + 4 * (j + 128), &sh, 4);
        }
    }
}

void oc_quantize_q4_0(const float *w, uint8_t *dst, int rows, int k) {
    int nb = k / OC_QK;
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < nb; ++b) {
            const float *x = w + (size_t)r * k + (size_t)b * OC_QK;
            uint8_t *blk = dst + ((size_t)r * nb + b) * OC_Q4_BYTES;
            float amax = 0.0f, signed_max = 0.0f;
            for (int j = 0; j < OC_QK; ++j)
                if (fabsf(x[j]) > amax) { amax = fabsf(x[j]); signed_max = x[j]; }
            float d = signed_max / -8.0f;
            float id = d != 0.0f ? 1.0f / d : 0.0f;
            oc_wr16(blk, oc_f32_to_f16(d));
            for (int j = 0; j < 16; ++j) {
                int lo = (int)(int8_t)(x[j] * id + 8.5f);
                int hi = (int)(int8_t)(x[j + 16] * id + 8.5f);
                if (lo > 15) lo = 15;
                if (hi > 15) hi = 15;
                blk[2 + j] = (uint8_t)(lo | (hi << 4));
            }
        }
}

/* qwen_one_layer.c:88-96. */
static uint32_t oc_rng = 0x5217ac8bu;
void oc_rng_seed(uint32_t s) { oc_rng = s; }
float oc_random_float(void) {
    uint32_t x = oc_rng;
    x ^= x << 13; x ^= x >> 17; x ^= x << 5;
    oc_rng = x;
    return (float)(x & 0xffffu) * (1.0f / 32767.5f) - 1.0f;
}

void oc_random_fill(float *dst, size_t n, float scale, float offset) {
    for (size_t i = 0; i < n; ++i) dst[i] = oc_random_float() * scale + offset;
}
