/*
 * si_qwen_one_layer.c -- the one-layer decode driver of simple-inference
 * (qwen_one_layer.c:596-740), running on libsi_b200.
 *
 *   si_qwen_one_layer <weights_dir> [context=256] [repeat=1]
 *                     [standard|flash|compare|fused|fused-compare|reference|
 *                      soa-staged|soa-fused]
 *
 * Same command line, inputs and result lines as the reference driver: the
 * input vector and the fp16 KV history come from the reference's xorshift32
 * stream (qwen_one_layer.c:88-96, 228-235), weights from q/k/v/o.q4_0 (+ the
 * optional norm and bias files) and, in the fused modes, q/kv/o.colsoa.  Every
 * layer call is a reference-shaped entry point of si_b200.h; phase times come
 * from CUDA events.  Only this file's reporting differs in layout.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "si_b200.h"

static void fail(const char *message) {
    fprintf(stderr, "error: %s\n", message);
    exit(1);
}

/* xorshift32 of qwen_one_layer.c:88-96: state 0x5217ac8b, x ^= x<<13, x>>17,
 * x<<5; a float is the low 16 bits mapped to [-1, 1). */
static uint32_t g_rng = 0x5217ac8bu;
static float next_float(void) {
    uint32_t x = g_rng;
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    g_rng = x;
    return (float)(x & 0xffffu) * (1.0f / 32767.5f) - 1.0f;
}

/* fp32 -> fp16, round to nearest even (the history is stored as the
 * reference stores it, qwen_one_layer.c:61-86). */
static uint16_t to_half(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t mag = u & 0x7fffffffu;
    if (mag >= 0x7f800000u) return (uint16_t)(sign | (mag > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (mag >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (mag < 0x38800000u) {                                   /* subnormal or zero */
        if (mag < 0x33000000u) return (uint16_t)sign;
        uint32_t m = (mag & 0x7fffffu) | 0x800000u;
        int shift = 126 - (int)(mag >> 23);                    /* 14..24 */
        uint32_t h = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((mag - 0x38000000u) >> 13);
    uint32_t rem = mag & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;
    return (uint16_t)(sign | h);
}

static void add_phase(phase_t *sum, const phase_t *p) {
    float *s = &sum->rms;
    const float *a = &p->rms;
    for (int i = 0; i < 9; ++i) s[i] += a[i];
}

static double phase_sum(const phase_t *p) {
    const float *a = &p->rms;
    double t = 0.0;
    for (int i = 0; i < 9; ++i) t += a[i];
    return t;
}

static double checksum(const float *y) {
    double s = 0.0;
    for (int i = 0; i < HIDDEN; ++i) {
        if (!isfinite(y[i])) fail("Non-finite projection output");
        s += (double)y[i];
    }
    return s;
}

static const char *const kPhases[9] = {
    "RMSNorm + input Q8", "Quantize input", "QKV projection (fused)", "K projection",
    "V projection", "RoPE + KV append", "GQA attention", "Quantize attention",
    "Output projection"};

static void print_phases(const char *title, const phase_t *p, int repeat) {
    const float *a = &p->rms;
    const double total = phase_sum(p);
    printf("%s\n", title);
    for (int i = 0; i < 9; ++i) {
        if (a[i] == 0.0f) continue; /* merged into the kernel that reports it */
        printf("  %-24s %10.4f ms/run %6.1f%%\n", kPhases[i], a[i] * 1e3 / repeat,
               total > 0 ? 100.0 * a[i] / total : 0.0);
    }
    printf("  %-24s %10.4f ms/run\n", "TOTAL (device, timed)", total * 1e3 / repeat);
}

static double max_abs_diff(const float *a, const float *b, int n) {
    double m = 0.0;
    for (int i = 0; i < n; ++i) {
        double d = fabs((double)a[i] - (double)b[i]);
        if (d > m) m = d;
    }
    return m;
}

static int q8_blocks_differ(const block_q8_0 *a, const block_q8_0 *b, int n) {
    int c = 0;
    for (int i = 0; i < n; ++i) c += memcmp(&a[i], &b[i], sizeof(block_q8_0)) != 0;
    return c;
}

int main(int argc, char **argv) {
    if (argc < 2 || argc > 5) {
        fprintf(stderr,
                "Usage: %s <weights_directory> [context=256] [repeat=1] "
                "[standard|flash|compare|fused|fused-compare|reference|soa-staged|soa-fused]\n",
                argv[0]);
        return 2;
    }
    char *end = NULL;
    long context = argc >= 3 ? strtol(argv[2], &end, 10) : 256;
    if (argc >= 3 && *end) fail("Invalid context argument");
    long repeat = argc >= 4 ? strtol(argv[3], &end, 10) : 1;
    if (argc >= 4 && *end) fail("Invalid repeat argument");
    if (context < 1 || context > 32768 || repeat < 1 || repeat > 100000)
        fail("Context must be 1..32768 and repeat 1..100000");
    const char *mode = argc >= 5 ? argv[4] : "compare";
    const int compare = !strcmp(mode, "compare");
    const int staged = !strcmp(mode, "soa-staged");
    const int fused_compare = !strcmp(mode, "fused-compare");
    const int fused = !strcmp(mode, "fused") || fused_compare || !strcmp(mode, "soa-fused") || staged;
    const int single = !strcmp(mode, "standard") || !strcmp(mode, "flash") ||
                       !strcmp(mode, "reference");
    if (!compare && !fused && !single)
        fail("Attention mode must be standard, flash, compare, fused, fused-compare, reference, "
             "soa-staged or soa-fused");
    const attention_method_t selected =
        !strcmp(mode, "standard") ? ATTENTION_STANDARD : ATTENTION_FLASH;

    layer_t l = load_layer(argv[1]);
    float *x = malloc(HIDDEN * sizeof(float));
    uint16_t *kc = malloc((size_t)context * KVDIM * sizeof(uint16_t));
    uint16_t *vc = malloc((size_t)context * KVDIM * sizeof(uint16_t));
    float *scores = malloc((size_t)QHEADS * (size_t)context * sizeof(float));
    float *y[2] = {malloc(HIDDEN * sizeof(float)), malloc(HIDDEN * sizeof(float))};
    float *att[2] = {malloc(HIDDEN * sizeof(float)), malloc(HIDDEN * sizeof(float))};
    block_q8_0 *q8[2] = {malloc((HIDDEN / QK) * sizeof(block_q8_0)),
                         malloc((HIDDEN / QK) * sizeof(block_q8_0))};
    if (!x || !kc || !vc || !scores || !y[0] || !y[1] || !att[0] || !att[1] || !q8[0] || !q8[1])
        fail("Out of memory creating synthetic inputs");
    for (int i = 0; i < HIDDEN; ++i) x[i] = next_float();
    for (size_t i = 0, n = (size_t)(context - 1) * KVDIM; i < n; ++i) {
        kc[i] = to_half(next_float() * 0.25f);
        vc[i] = to_half(next_float() * 0.25f);
    }

    printf("Qwen2.5 one attention sublayer (decode) on B200 | mode %s | context %ld | repeats %ld\n",
           mode, context, repeat);
    printf("Weights Q4_0 | activations Q8_0 | KV cache FP16 | times are CUDA-event device time\n");

    if (fused) {
        fused_weights_t fw = fused_weights_load(argv[1], 0, 0);
        fused_stats_t fs;
        memset(&fs, 0, sizeof(fs));
        for (long r = 0; r < repeat; ++r) {
            fused_stats_t p = staged ? run_layer_soa_staged(&l, &fw, x, kc, vc, (int)context,
                                                            y[1], NULL, NULL)
                                     : run_layer_fused(&l, &fw, x, kc, vc, (int)context, y[1],
                                                       NULL, NULL);
            add_phase(&fs.phase, &p.phase);
            fs.tcm_stage += p.tcm_stage;
        }
        if (fused_compare) {
            (void)run_layer(&l, x, kc, vc, (int)context, y[0], ATTENTION_FLASH, scores, att[0],
                            q8[0]);
            (void)run_layer_fused(&l, &fw, x, kc, vc, (int)context, y[1], att[1], q8[1]);
            printf("run_layer vs run_layer_fused: output max|diff| %.3g, attention max|diff| %.3g, "
                   "Q8 blocks differing %d/%d\n",
                   max_abs_diff(y[0], y[1], HIDDEN), max_abs_diff(att[0], att[1], HIDDEN),
                   q8_blocks_differ(q8[0], q8[1], HIDDEN / QK), HIDDEN / QK);
        }
        print_phases(staged ? "SOA STAGED one-token" : "REGISTER FUSED one-token", &fs.phase,
                     (int)repeat);
        printf("Compute %.3f ms/token, staging %.3f ms/token, all %.3f ms/token\n",
               (fused_total(&fs) - fs.tcm_stage) * 1e3 / repeat, fs.tcm_stage * 1e3 / repeat,
               fused_total(&fs) * 1e3 / repeat);
        printf("Output checksum %.10g | first four %.6g %.6g %.6g %.6g\n", checksum(y[1]), y[1][0],
               y[1][1], y[1][2], y[1][3]);
        fused_weights_free(&fw);
    } else if (compare) {
        phase_t sum[2];
        memset(sum, 0, sizeof(sum));
        for (long r = 0; r < repeat; ++r)
            for (int j = 0; j < 2; ++j) {
                int m = (r & 1) ? 1 - j : j;
                phase_t p = run_layer(&l, x, kc, vc, (int)context, y[m], (attention_method_t)m,
                                      scores, att[m], q8[m]);
                add_phase(&sum[m], &p);
            }
        print_phases("STANDARD", &sum[0], (int)repeat);
        print_phases("FLASH", &sum[1], (int)repeat);
        printf("standard vs flash: output max|diff| %.3g, attention max|diff| %.3g, Q8 blocks "
               "differing %d/%d\n",
               max_abs_diff(y[0], y[1], HIDDEN), max_abs_diff(att[0], att[1], HIDDEN),
               q8_blocks_differ(q8[0], q8[1], HIDDEN / QK), HIDDEN / QK);
        printf("Output checksum: %.9g  |  First 4: [%.6g, %.6g, %.6g, %.6g]\n", checksum(y[1]),
               y[1][0], y[1][1], y[1][2], y[1][3]);
    } else {
        phase_t sum;
        memset(&sum, 0, sizeof(sum));
        for (long r = 0; r < repeat; ++r) {
            phase_t p = run_layer(&l, x, kc, vc, (int)context, y[0], selected, scores, NULL, NULL);
            add_phase(&sum, &p);
        }
        print_phases(attention_name(selected), &sum, (int)repeat);
        printf("Output checksum: %.9g  |  First 4: [%.6g, %.6g, %.6g, %.6g]\n", checksum(y[0]),
               y[0][0], y[0][1], y[0][2], y[0][3]);
    }
    free(x);
    free(kc);
    free(vc);
    free(scores);
    for (int i = 0; i < 2; ++i) {
        free(y[i]);
        free(att[i]);
        free(q8[i]);
    }
    free_layer(&l);
    return 0;
}
