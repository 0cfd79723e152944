/*
 * si_b200.h -- C ABI of libsi_b200.so, the B200 (sm_100a) implementation of the
 * keyvan-dadash/simple-inference Qwen decoder-layer hot path.
 *
 * Two layers of entry points:
 *
 *  1. The handle API (si_*): a context owns one CUDA device and stream; weights
 *     are uploaded once as device matrices in the SoA Q4_0 layout; KV caches live
 *     on the device.  Everything the benchmarks and the reference-shaped calls do
 *     goes through these functions.  Plain pointers and sizes only.
 *
 *  2. Reference-shaped entry points with the reference's names and argument
 *     lists (quantize_q8, matvec_q4q8, rmsnorm, rope, attention_compute,
 *     run_layer, fused_column_matvec, run_layer_fused, pf_run_batch, ...), so a
 *     translation unit written against the reference's headers builds against
 *     this header instead.  They take HOST pointers, run on the GPU of an
 *     implicit per-process context, and copy results back.  The functions whose
 *     reference versions read compile-time dims (HIDDEN, QHEADS, ...) are static
 *     inline wrappers over dims-parametrised si_ref_* symbols; the dims macros
 *     default to the reference's defines.h values and can be overridden.
 *
 * Errors: every si_* function returns si_status.  The reference-shaped wrappers
 * keep the reference's contract (qwen_one_layer.c:26-28): on error they print
 * "error: <message>" to stderr and exit(1).  There is no CPU fallback: without
 * an sm_100 device every entry point fails with SI_ERR_NO_DEVICE.
 */
#ifndef SI_B200_H
#define SI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define SI_API
#else
#define SI_API __attribute__((visibility("default")))
#endif

/* ------------------------------------------------------------------------ */
/* Reference compile-time configuration (defines.h:16-25); overridable.      */
/* ------------------------------------------------------------------------ */
#ifndef HIDDEN
#define HIDDEN 1536
#endif
#ifndef QHEADS
#define QHEADS 12
#endif
#ifndef KVHEADS
#define KVHEADS 2
#endif
#ifndef HDIM
#define HDIM 128
#endif
#ifndef KVDIM
#define KVDIM (KVHEADS * HDIM)
#endif
#ifndef QK
#define QK 32
#endif
#ifndef Q4_BYTES
#define Q4_BYTES 18
#endif
#ifndef Q8_BYTES
#define Q8_BYTES 34
#endif
#ifndef ROPE_BASE
#define ROPE_BASE 1000000.0f
#endif
#ifndef RMS_EPS
#define RMS_EPS 1e-6f
#endif

/* ------------------------------------------------------------------------ */
/* Status                                                                    */
/* ------------------------------------------------------------------------ */
typedef enum {
    SI_OK = 0,
    SI_ERR_INVALID = 1,    /* bad argument, shape or handle */
    SI_ERR_CUDA = 2,       /* CUDA runtime error */
    SI_ERR_OOM = 3,        /* device allocation failed */
    SI_ERR_NO_DEVICE = 4,  /* no sm_100 device / CUDA unavailable */
    SI_ERR_DEVICE = 5,     /* a kernel set the device error word */
    SI_ERR_TIMEOUT = 6,    /* a bounded device wait expired */
    SI_ERR_IO = 7,         /* file missing or of the wrong size */
    SI_ERR_UNSUPPORTED = 8 /* configuration not implemented */
} si_status;

SI_API const char *si_status_str(si_status s);

/* ------------------------------------------------------------------------ */
/* Reference types, byte-identical (defines.h:27-37, attention_kernels.h:24). */
/* ------------------------------------------------------------------------ */
#ifndef SI_NO_REFERENCE_TYPES
typedef struct { uint16_t d; int8_t qs[32]; } block_q8_0;      /* defines.h:27-28 */
typedef struct {                                                /* defines.h:30-33 */
    uint8_t *wq, *wk, *wv, *wo;
    float *norm, *bq, *bk, *bv;
} layer_t;
typedef struct {                                                /* defines.h:35-37 */
    float rms, q8_input, q_proj, k_proj, v_proj, rope_cache, attention, q8_output, out_proj;
} phase_t;
typedef enum { ATTENTION_STANDARD = 0, ATTENTION_FLASH = 1 } attention_method_t;
/* Column-SoA tile geometry of repack_weights.py (fused_layer.h:33-36): one
 * 5120-byte group per Q4_0 block (32 columns x 128 bytes of nibble pairs for
 * 256 outputs, then 256 fp32 scales); a tile is 256 outputs over HIDDEN. */
#ifndef FUSED_COL_BYTES
#define FUSED_COL_BYTES 128u
#define FUSED_GROUP_BYTES 5120u
#define FUSED_TILE_BYTES ((unsigned)(HIDDEN / QK) * FUSED_GROUP_BYTES)
#define FUSED_WO_SUBTILE (8u * FUSED_GROUP_BYTES)
#endif
typedef struct {                                                /* fused_layer.h:59-66 */
    uint8_t *q, *kv, *o;
    int tcm_fd;
    uint8_t *tcm_map;
    uint8_t *tcm_tile;
    size_t tcm_map_bytes;
    int tcm_block;
} fused_weights_t;
typedef struct {                                                /* fused_layer.h:68-71 */
    phase_t phase;
    double tcm_stage;
} fused_stats_t;
typedef struct {                            /* prefill_weight_stationary.h:149-155 */
    block_q8_0 *xin;
    block_q8_0 *oq;
    float *acc;
    float *cv, *sv;
    int capacity;
} pf_workspace_t;
/* The reference's AI-DMA pipeline handle (ai_dma_pipeline.h:79-97).  Weight
 * staging happens inside the GPU kernels (TMA / cp.async), so here it is an
 * opaque type that pf_run_batch accepts and ignores; NULL is fine. */
typedef struct si_ai_pipeline rt_ai_pipeline_t;
#ifdef __cplusplus
static_assert(sizeof(block_q8_0) == 34, "block_q8_0 must be the reference's 34 bytes");
static_assert(sizeof(phase_t) == 9 * sizeof(float), "phase_t must be 9 floats");
#else
_Static_assert(sizeof(block_q8_0) == 34, "block_q8_0 must be the reference's 34 bytes");
_Static_assert(sizeof(phase_t) == 9 * sizeof(float), "phase_t must be 9 floats");
#endif
#endif

/* ------------------------------------------------------------------------ */
/* Handle API                                                                */
/* ------------------------------------------------------------------------ */
typedef struct si_ctx si_ctx;
typedef struct si_matrix si_matrix;
typedef struct si_layer si_layer;
typedef struct si_kv si_kv;

typedef struct {
    int hidden, n_q_heads, n_kv_heads, head_dim, intermediate; /* intermediate 0 = no MLP */
    float rope_theta, rms_eps;
} si_dims;

/* Host-side layer description.  Q4_0 matrices are GGUF row-major blocks
 * ([rows][cols/32] x 18 B: fp16 d + 16 nibble bytes); optional vectors may be
 * NULL (identity norm, zero bias) as in qwen_one_layer.c:216-219. */
typedef struct {
    const uint8_t *wq, *wk, *wv, *wo;       /* [Hq*D][H], [Hkv*D][H] x2, [H][Hq*D] */
    const uint8_t *w_gate, *w_up, *w_down;  /* [I][H], [I][H], [H][I]; NULL if intermediate==0 */
    const float *norm, *bq, *bk, *bv, *norm2;
} si_layer_host;

/* Layer run modes. */
#define SI_LAYER_ATTN 0  /* run_layer semantics: y = W_O(attn(rmsnorm(x))), no residual */
#define SI_LAYER_FULL 1  /* decoder layer: h = x + attn; y = h + down(silu(gate)*up) */

/* Context: one device, one stream, RoPE cos/sin tables for positions
 * [0, max_positions) computed on the host with the reference's expressions. */
SI_API si_status si_ctx_create(int device, int max_positions, float rope_theta, int head_dim,
                               si_ctx **out);
SI_API void si_ctx_destroy(si_ctx *ctx);
SI_API si_status si_ctx_synchronize(si_ctx *ctx);
/* Synchronises, then returns and clears the device error word. */
SI_API si_status si_ctx_status(si_ctx *ctx);
SI_API void *si_ctx_stream(si_ctx *ctx); /* the cudaStream_t all work is queued on */
/* Prefill attention kernel of this context (no reference counterpart: the
 * reference has one CPU loop).  0 (default): tcgen05 tensor cores on split
 * fp16 operands, within about 1e-6 relative of the fp32 kernel, for head_dim
 * 128; 1: the fp32 kernel, whose prefill tokens are bit-identical to the
 * same tokens' decode steps.  The reference-shaped pf_run_batch always uses
 * the fp32 kernel. */
SI_API si_status si_ctx_set_exact_attention(si_ctx *ctx, int exact);
/* Bytes of device memory the context currently holds in its on-demand
 * buffers (step arena, index arrays, GEMM activation-scale scratch); they grow
 * when a call needs more and are freed by si_ctx_destroy. */
SI_API size_t si_ctx_scratch_bytes(const si_ctx *ctx);
/* Kernels this library has queued so far, process-wide (all devices and
 * contexts); the difference across a region counts its kernel launches. */
SI_API unsigned long long si_kernel_launches(void);
SI_API const char *si_last_error(void);  /* message of the last failing call on this thread */

/* Weight matrices.  Upload GGUF Q4_0 rows and repack on the device into the
 * row-tile SoA layout (see si_matrix_layout). rows % 32 == 0, cols % 32 == 0. */
SI_API si_status si_matrix_upload(si_ctx *ctx, const uint8_t *gguf_host, int rows, int cols,
                                  si_matrix **out);
SI_API si_status si_matrix_upload_dev(si_ctx *ctx, const uint8_t *gguf_dev, int rows, int cols,
                                      si_matrix **out);
SI_API void si_matrix_free(si_matrix *m);
SI_API int si_matrix_rows(const si_matrix *m);
SI_API int si_matrix_cols(const si_matrix *m);
/* Device pointers of the layout: nibbles [rows/32][cols/32][32][16] bytes
 * (GGUF nibble order, each byte XOR 0x88) and scales [rows/32][cols/32][32] fp16. */
SI_API si_status si_matrix_layout(const si_matrix *m, void **nib_dev, void **scale_dev);
/* Fill a matrix with seeded synthetic Q4_0 weights on the device: element
 * values ~N(0, std) from a counter hash of (seed, row, col), quantised with the
 * GGUF rule.  Used for large benchmark configurations. */
SI_API si_status si_matrix_synth(si_ctx *ctx, int rows, int cols, uint64_t seed, float std,
                                 si_matrix **out);
/* Copy a matrix back as GGUF row-major Q4_0 bytes (host). */
SI_API si_status si_matrix_download(si_ctx *ctx, const si_matrix *m, uint8_t *gguf_host);

/* Activations on the device: Q8 tensors are two arrays, qs int8 [M][K] and
 * d fp16 [M][K/32] (block_q8_0 split for coalescing); the reference's 34-byte
 * blocks are produced by si_q8_to_blocks.  si_q8_quantize_dev needs x 16-byte
 * aligned and qs 4-byte aligned (SI_ERR_CUDA otherwise). */
SI_API si_status si_q8_quantize_dev(si_ctx *ctx, const float *x_dev, int M, int K,
                                    int8_t *qs_dev, uint16_t *d_dev);
SI_API si_status si_q8_to_blocks_dev(si_ctx *ctx, const int8_t *qs_dev, const uint16_t *d_dev,
                                     int M, int K, block_q8_0 *blocks_dev);
SI_API si_status si_q8_from_blocks_dev(si_ctx *ctx, const block_q8_0 *blocks_dev, int M, int K,
                                       int8_t *qs_dev, uint16_t *d_dev);
/* out[m][n] = bias[n] + sum_b ((float)isum * dw) * dx, blocks in order
 * (qwen_one_layer.c:148-162); picks the GEMV or the tensor-core GEMM by M. */
SI_API si_status si_matmul_dev(si_ctx *ctx, const si_matrix *w, const int8_t *qs_dev,
                               const uint16_t *d_dev, int M, const float *bias_dev,
                               float *out_dev);
/* Force a kernel: 0 = GEMV (its form picked by M), 1 = tcgen05 GEMM,
 * 2 = GEMV in its tensor-core (mma.sync s8) form, 3 = GEMV in its dp4a form,
 * 4 = mma.sync GEMM (rows % 128, cols % 32).  Kernels 0-4 return the same bits
 * (the reference's).  5 = tcgen05 GEMM in its fused-rescale mode: each block's
 * term is added with one FMA, acc = fma(round(isum*dw), dx, acc), one rounding
 * fewer than the reference's ((float)isum*dw)*dx then +=, so outputs differ
 * from the reference's by far less than the 1e-5 relative projection bar. */
SI_API si_status si_matmul_dev_kernel(si_ctx *ctx, const si_matrix *w, const int8_t *qs_dev,
                                      const uint16_t *d_dev, int M, const float *bias_dev,
                                      float *out_dev, int kernel);
/* matvec_q4q8 (qwen_one_layer.c:148-162) for M <= 8 tokens straight from
 * row-major GGUF Q4_0 blocks in device memory (rows x cols/32 blocks of 18
 * bytes, the reference's own layout), no repack: the same bits as the
 * repacked GEMV.  cols % 128 == 0; weights and qs 16-byte aligned. */
SI_API si_status si_matvec_gguf_dev(si_ctx *ctx, const uint8_t *w_gguf_dev, int rows, int cols,
                                    const int8_t *qs_dev, const uint16_t *d_dev, int M,
                                    const float *bias_dev, float *out_dev);
/* The tcgen05 GEMM of si_matmul_dev_kernel(..., 1) with the same results, but
 * allocating nothing: its scratch (the transposed fp32 activation scales,
 * (cols/32) * round_up(M, 4) * 4 bytes) is a fixed array of
 * SI_STATIC_GEMM_SCRATCH_BYTES inside the library, which every GPU that loads
 * the library holds until the process exits.  For callers that must not
 * allocate device memory while they run (an allocator that already owns the
 * free memory, or a loop that cannot take cudaMalloc's synchronisation).
 * Larger shapes fail with SI_ERR_INVALID.  The first call on each device looks
 * up the array's device address (cudaGetSymbolAddress) and should come before
 * any stream capture.  All calls on a device share the one array: calls that
 * overlap on the GPU (other streams, other contexts of the same device) race
 * and must be serialised by the caller.  This entry point has no counterpart
 * in the reference. */
#define SI_STATIC_GEMM_SCRATCH_BYTES (4 * 1024 * 1024)
SI_API si_status si_matmul_tc_static_dev(si_ctx *ctx, const si_matrix *w, const int8_t *qs_dev,
                                         const uint16_t *d_dev, int M, const float *bias_dev,
                                         float *out_dev);
/* Per-(row, block) int32 partial sums [M][rows][cols/32] (parity checks). */
/* Int8 tensor-core throughput probe (no reference counterpart: it measures
 * the prefill GEMM's roofline denominator).  Queues one launch on the
 * context's stream: one CTA per SM, each issuing iters x 4 tcgen05 kind::i8
 * MMAs of 128 x n x 32 (n = 128 or 256) from operands resident in shared
 * memory; *ops_per_launch receives the int8 operations the launch performs.
 * Time it with events on si_ctx_stream(). */
SI_API si_status si_tc_i8_peak_dev(si_ctx *ctx, int n, int iters, double *ops_per_launch);
SI_API si_status si_block_isums_dev(si_ctx *ctx, const si_matrix *w, const int8_t *qs_dev,
                                    int M, int32_t *isum_dev);
/* SwiGLU pair: act = silu(gate@x) * (up@x), quantised to Q8 in the epilogue. */
SI_API si_status si_gateup_q8_dev(si_ctx *ctx, const si_matrix *gate, const si_matrix *up,
                                  const int8_t *qs_dev, const uint16_t *d_dev, int M,
                                  int8_t *act_qs_dev, uint16_t *act_d_dev, float *act_f32_dev);
/* The same with a forced kernel (-1 = by M; otherwise as si_matmul_dev_kernel). */
SI_API si_status si_gateup_q8_dev_kernel(si_ctx *ctx, const si_matrix *gate, const si_matrix *up,
                                         const int8_t *qs_dev, const uint16_t *d_dev, int M,
                                         int8_t *act_qs_dev, uint16_t *act_d_dev,
                                         float *act_f32_dev, int kernel);
/* RMSNorm over rows of x [M][n] (qwen_one_layer.c:164-169) with optional fp32
 * output and fused Q8 output.  x, w and out 16-byte aligned, qs 4-byte aligned
 * (SI_ERR_CUDA otherwise). */
SI_API si_status si_rmsnorm_q8_dev(si_ctx *ctx, const float *x_dev, const float *w_dev, int M,
                                   int n, float eps, float *out_dev, int8_t *qs_dev,
                                   uint16_t *d_dev);

/* Layers and KV caches. */
SI_API si_status si_layer_upload(si_ctx *ctx, const si_dims *dims, const si_layer_host *host,
                                 si_layer **out);
/* Synthetic layer generated on the device (seeded); norms 1+N(0,0.02), biases N(0,0.02). */
SI_API si_status si_layer_synth(si_ctx *ctx, const si_dims *dims, uint64_t seed, si_layer **out);
SI_API void si_layer_free(si_layer *l);
SI_API si_status si_layer_matrix(si_layer *l, int which, si_matrix **out); /* 0 qkv,1 o,2 gate,3 up,4 down */
/* Copy the layer's norm, norm2 and fused Q|K|V bias to host arrays (NULL skips). */
SI_API si_status si_layer_vectors_download(si_ctx *ctx, const si_layer *l, float *norm,
                                           float *norm2, float *bias_qkv);

/* KV cache [batch][max_ctx][Hkv][D], fp16 (kv_f32=0, the reference's format,
 * attention_kernels.h:43-44) or fp32. */
SI_API si_status si_kv_create(si_ctx *ctx, const si_dims *dims, int batch, int max_ctx,
                              int kv_f32, si_kv **out);
SI_API void si_kv_free(si_kv *kv);
SI_API si_status si_kv_write(si_ctx *ctx, si_kv *kv, int seq, int pos0, int npos,
                             const void *k_host, const void *v_host);
SI_API si_status si_kv_read(si_ctx *ctx, si_kv *kv, int seq, int pos0, int npos, void *k_host,
                            void *v_host);
SI_API si_status si_kv_fill_synth(si_ctx *ctx, si_kv *kv, uint64_t seed, float std, int npos);
SI_API void *si_kv_device_ptr(si_kv *kv, int which); /* 0 = K, 1 = V */

/* Optional intermediate captures of a decode step (device or host pointers as
 * the calling function states; NULL = off). */
typedef struct {
    float *attn;        /* [B][Hq*D] attention output before W_O */
    block_q8_0 *attn_q8;/* [B][Hq*D/32] quantised attention output */
    float *qkv;         /* [B][Hq*D + 2*Hkv*D] projections before RoPE */
} si_captures;

/* One decode step for a batch: sequence b appends its token at slot
 * ctx_lens[b]-1 and attends over [0, ctx_lens[b]).  x and y are [B][H].
 * _dev variants take device pointers (ctx_lens stays a host array). */
SI_API si_status si_decode_step(si_ctx *ctx, si_layer *l, si_kv *kv, const float *x_host,
                                int batch, const int *ctx_lens, float *y_host, int mode,
                                const si_captures *cap_host);
SI_API si_status si_decode_step_dev(si_ctx *ctx, si_layer *l, si_kv *kv, const float *x_dev,
                                    int batch, const int *ctx_lens, float *y_dev, int mode,
                                    const si_captures *cap_dev);
/* Decode positions kept on the device (no reference counterpart: the
 * reference passes `context` per call, qwen_one_layer.c:237).  A decode step
 * given a state reads sequence b's context length from device memory instead
 * of a host array, so a whole multi-layer step -- the layers' calls and then
 * si_decode_state_advance -- can be captured once (si_graph_begin/end) and
 * replayed for step after step with no host work per step.  Sequence b is
 * batch entry b; 1 <= batch <= 256; lengths stay within [1, max_ctx] (the
 * advance that would pass max_ctx leaves the lengths and records
 * SI_ERR_INVALID in the context's error word). */
typedef struct si_decode_state si_decode_state;
SI_API si_status si_decode_state_create(si_ctx *ctx, int batch, const int *ctx_lens_host,
                                        int max_ctx, si_decode_state **out);
SI_API void si_decode_state_free(si_decode_state *st);
/* Queues "set the lengths to ctx_lens_host" (their values are taken now). */
SI_API si_status si_decode_state_set(si_ctx *ctx, si_decode_state *st, const int *ctx_lens_host);
/* Queues "every length + 1" on the context's stream. */
SI_API si_status si_decode_state_advance(si_ctx *ctx, si_decode_state *st);
/* Synchronises and copies the current lengths to the host. */
SI_API si_status si_decode_state_read(si_ctx *ctx, si_decode_state *st, int *ctx_lens_host);
/* si_decode_step_dev with the lengths of st (batch = st's batch; the KV cache's
 * max_ctx must equal st's). */
SI_API si_status si_decode_step_state_dev(si_ctx *ctx, si_layer *l, si_kv *kv, const float *x_dev,
                                          si_decode_state *st, float *y_dev, int mode);
/* Causal prefill of ntok tokens of sequence seq at positions [prefix,
 * prefix+ntok): token t attends over [0, prefix+t+1) (prefill_weight_stationary.h:173-186). */
SI_API si_status si_prefill(si_ctx *ctx, si_layer *l, si_kv *kv, int seq, const float *x_host,
                            int ntok, int prefix, float *y_host, int mode);
SI_API si_status si_prefill_dev(si_ctx *ctx, si_layer *l, si_kv *kv, int seq, const float *x_dev,
                                int ntok, int prefix, float *y_dev, int mode);

/* ------------------------------------------------------------------------ */
/* Tensor parallelism (multi-layer 72B configuration over 2/4/8 GPUs).       */
/* One process per GPU.  Q/K/V and gate/up are split by rows (whole heads;    */
/* 128-row units of the MLP, uneven by at most one unit), o and down by       */
/* columns, so each row-parallel projection leaves partial sums to be added  */
/* across the ranks.  Decode-sized steps (at most 16 tokens) fuse that       */
/* exchange into the projection: its GEMV stores the partial sums into every */
/* rank's receive slot over NVLink (CUDA IPC mappings of one buffer per rank, */
/* set up by the first such step, a collective call), each value in one      */
/* 8-byte word tagged with the call's epoch; the consuming kernel waits for   */
/* the tagged words (bounded; SI_ERR_TIMEOUT past the limit) and adds the     */
/* slots in rank order and the residual.  Larger steps use one NCCL           */
/* all-reduce on the context's stream, then the residual add.  Cross-rank     */
/* summation changes the fp32 order: layer outputs agree with one GPU to the  */
/* 1e-3 layer bar, not bit for bit; every rank holds identical outputs.       */
/* The context that creates a group must outlive it.  Not in the reference.   */
/* ------------------------------------------------------------------------ */
typedef struct si_tp si_tp;
/* Units [*first, *first + *count) of `units` owned by rank (host only). */
SI_API void si_tp_split(int units, int rank, int world, int *first, int *count);
/* ncclGetUniqueId into 128 bytes, to be shared with every rank. */
SI_API si_status si_tp_unique_id(void *id128);
SI_API si_status si_tp_create(si_ctx *ctx, const void *id128, int rank, int world, si_tp **out);
/* Collective when the group has fused buffers: every rank frees together. */
SI_API void si_tp_free(si_tp *tp);
/* fused = 0 sends every row-parallel projection through NCCL; timeout_ms
 * bounds the fused reduction's wait for the other ranks (default 5000). */
SI_API si_status si_tp_set_options(si_tp *tp, int fused, int timeout_ms);
/* Runs the fused reduction's bounded wait against words that nothing writes,
 * on this GPU alone: returns SI_ERR_TIMEOUT after about timeout_us and leaves
 * the context usable (a check of the failure path, no other rank needed). */
SI_API si_status si_tp_probe_wait(si_ctx *ctx, int timeout_us);
/* The shard's dims (heads / world, this rank's MLP rows) and the first MLP
 * row it owns.  Needs heads divisible by world and intermediate % 128 == 0. */
SI_API si_status si_tp_local_dims(const si_dims *full, int rank, int world, si_dims *local,
                                  int *mlp_first);
/* This rank's shard of si_layer_synth(full, seed): equal to the same slices
 * of the whole layer. */
SI_API si_status si_layer_tp_synth(si_ctx *ctx, const si_dims *full, uint64_t seed, int rank,
                                   int world, si_layer **out);
/* Steps on a shard (KV cache created with the local dims); x and y are the
 * full hidden vectors, identical on every rank. */
SI_API si_status si_decode_step_tp_dev(si_ctx *ctx, si_tp *tp, si_layer *l, si_kv *kv,
                                       const float *x_dev, int batch, const int *ctx_lens,
                                       float *y_dev, int mode);
/* si_decode_step_tp_dev with the lengths of a decode state.  The fused
 * exchanges' epochs are then counted from a device counter that
 * si_decode_state_advance moves on, so the whole multi-layer step (every
 * layer's call, then the advance) can be captured once and replayed. */
SI_API si_status si_decode_step_state_tp_dev(si_ctx *ctx, si_tp *tp, si_layer *l, si_kv *kv,
                                             const float *x_dev, si_decode_state *st,
                                             float *y_dev, int mode);
SI_API si_status si_prefill_tp_dev(si_ctx *ctx, si_tp *tp, si_layer *l, si_kv *kv, int seq,
                                   const float *x_dev, int ntok, int prefix, float *y_dev,
                                   int mode);

/* CUDA-graph capture of a sequence of calls on the context's stream (no host
 * synchronisation may happen between begin and end: the *_dev matrix/Q8 calls
 * qualify).  Replays run the captured kernels with no launch gaps. */
typedef struct si_graph si_graph;
SI_API si_status si_graph_begin(si_ctx *ctx);
SI_API si_status si_graph_end(si_ctx *ctx, si_graph **out);
SI_API si_status si_graph_launch(si_ctx *ctx, si_graph *g);
SI_API void si_graph_free(si_graph *g);
/* Number of kernel launches a replay performs (-1 on error). */
SI_API int si_graph_kernel_nodes(const si_graph *g);

/* Decode attention alone (parity): q [B][Hq][D] after RoPE. */
SI_API si_status si_attention_decode_dev(si_ctx *ctx, si_kv *kv, const si_dims *dims,
                                         const float *q_dev, int batch, const int *ctx_lens,
                                         float *out_dev);
/* Causal attention of a prefill on its own (no reference counterpart as an
 * entry point: the prefill attention inside pf_run_batch,
 * prefill_weight_stationary.h:245-287): q [ntok][Hq][D] (RoPE applied) of
 * tokens at positions prefix .. prefix+ntok-1 of sequence seq, attending the
 * cache's keys 0 .. position; out [ntok][Hq][D].  The kernel follows the
 * context's si_ctx_set_exact_attention setting; the tensor-core kernel needs
 * q 16-byte aligned. */
SI_API si_status si_attention_prefill_dev(si_ctx *ctx, si_kv *kv, const si_dims *d,
                                          const float *q_dev, int ntok, int seq, int prefix,
                                          float *out_dev);

/* ------------------------------------------------------------------------ */
/* Reference-shaped entry points (host pointers, implicit context).          */
/* ------------------------------------------------------------------------ */

/* qwen_one_layer.c:98 quantize_q8 */
SI_API void quantize_q8(const float *src, block_q8_0 *dst, int count);
/* qwen_one_layer.c:148 matvec_q4q8.  Device copies of `weights` are cached by
 * host address and size; call si_forget_host_weights() after changing them
 * (also for a layer's wq, and for column-SoA tiles or blobs of
 * fused_weights_load). */
SI_API void matvec_q4q8(const uint8_t *weights, const block_q8_0 *input, int inputs, int outputs,
                        const float *bias, float *out);
SI_API void si_forget_host_weights(const void *host_ptr);

/* Dims-parametrised symbols behind the inline wrappers below. */
SI_API void si_ref_rmsnorm(const float *input, const float *weight, float *out, int n, float eps);
SI_API void si_ref_rope(float *heads, int nheads, int position, int head_dim, float theta);
SI_API void si_ref_attention(int method, const float *q, const uint16_t *kc, const uint16_t *vc,
                             int context, float *out, float *scores, int n_q_heads,
                             int n_kv_heads, int head_dim);
SI_API phase_t si_ref_run_layer(const layer_t *l, const float *x, uint16_t *kc, uint16_t *vc,
                                int context, float *output, int method, float *scores,
                                float *attn_copy, block_q8_0 *q8_copy, int hidden, int n_q_heads,
                                int n_kv_heads, int head_dim, float theta, float eps);
SI_API layer_t si_ref_load_layer(const char *dir, int hidden, int kvdim);
SI_API void si_ref_free_layer(layer_t *l);

/* fused_layer.h:169 fused_column_matvec: output[0..255] = (add ? output :
 * bias) + sum over nblocks groups of one column-SoA tile, in block order.
 * The tile's device copy is cached by host address and size. */
SI_API void fused_column_matvec(const uint8_t *tile, const block_q8_0 *x, int nblocks,
                                const float *bias_lo, const float *bias_hi, float *output,
                                int add);
/* fused_layer.h:131 fused_weights_load / :141 fused_weights_free: the
 * q/kv/o.colsoa tiles.  use_tcm and block select the RISC-V TCM staging of the
 * reference; they are accepted and ignored (tcm_fd = -1, no TCM mapping). */
SI_API fused_weights_t si_ref_fused_weights_load(const char *dir, int use_tcm, int block,
                                                 int hidden, int n_q_heads, int n_kv_heads);
SI_API void fused_weights_free(fused_weights_t *fw);
/* register_fusion.h:344 run_layer_fused, fused_layer.h:397
 * run_layer_legacy_fused, soa_staged.h:18 run_layer_soa_staged: one decode
 * step whose Q/K/V/O weights come from the column-SoA tiles and norm/biases
 * from l.  The three schedules compute the same function (the reference's
 * portable build runs the legacy schedule for all three); here they share one
 * GPU schedule.  tcm_stage is 0. */
SI_API fused_stats_t si_ref_run_layer_fused(const layer_t *l, const fused_weights_t *fw,
                                            const float *x, uint16_t *kc, uint16_t *vc,
                                            int context, float *output, float *attn_capture,
                                            block_q8_0 *q8_capture, int hidden, int n_q_heads,
                                            int n_kv_heads, int head_dim, float theta,
                                            float eps);
/* prefill_weight_stationary.h:157-168 pf_workspace_open / close (host
 * buffers of the reference's layout; the GPU prefill keeps its own). */
SI_API void si_ref_pf_workspace_open(pf_workspace_t *p, int ntok, int hidden);
SI_API void pf_workspace_close(pf_workspace_t *p);
/* prefill_weight_stationary.h:183 pf_run_batch: causal prefill of ntok tokens
 * at positions [prefix, prefix+ntok) -- token t attends over prefix+t+1
 * positions -- appending their K/V to the caller's fp16 cache and writing
 * output[ntok][hidden]; equal to ntok sequential run_layer steps. */
SI_API void si_ref_pf_run_batch(const layer_t *l, const fused_weights_t *fw,
                                rt_ai_pipeline_t *a, pf_workspace_t *p, const float *x,
                                int ntok, int prefix, uint16_t *kc, uint16_t *vc,
                                float *output, int hidden, int n_q_heads, int n_kv_heads,
                                int head_dim, float theta, float eps);

/* qwen_one_layer.c:164 rmsnorm */
static inline void rmsnorm(const float *input, const float *weight, float *out) {
    si_ref_rmsnorm(input, weight, out, HIDDEN, RMS_EPS);
}
/* qwen_one_layer.c:172 rope */
static inline void rope(float *heads, int nheads, int position) {
    si_ref_rope(heads, nheads, position, HDIM, ROPE_BASE);
}
/* attention_kernels.h:166 attention_compute (flash: :80, standard: :33) */
static inline void attention_compute(attention_method_t method, const float *q,
                                     const uint16_t *kc, const uint16_t *vc, int context,
                                     float *out, float *score_workspace) {
    si_ref_attention((int)method, q, kc, vc, context, out, score_workspace, QHEADS, KVHEADS, HDIM);
}
static inline void attention_flash(const float *q, const uint16_t *kc, const uint16_t *vc,
                                   int context, float *out) {
    si_ref_attention(1, q, kc, vc, context, out, NULL, QHEADS, KVHEADS, HDIM);
}
static inline void attention_standard(const float *q, const uint16_t *kc, const uint16_t *vc,
                                      int context, float *out, float *scores) {
    si_ref_attention(0, q, kc, vc, context, out, scores, QHEADS, KVHEADS, HDIM);
}
/* qwen_one_layer.c:237 run_layer (phase_t filled from CUDA events) */
static inline phase_t run_layer(const layer_t *l, const float *x, uint16_t *kc, uint16_t *vc,
                                int context, float *output, attention_method_t method,
                                float *scores, float *attn_copy, block_q8_0 *q8_copy) {
    return si_ref_run_layer(l, x, kc, vc, context, output, (int)method, scores, attn_copy,
                            q8_copy, HIDDEN, QHEADS, KVHEADS, HDIM, ROPE_BASE, RMS_EPS);
}
/* attention_kernels.h:29 attention_name */
static inline const char *attention_name(attention_method_t method) {
    return method == ATTENTION_FLASH ? "flash" : "standard";
}
static inline fused_weights_t fused_weights_load(const char *dir, int use_tcm, int block) {
    return si_ref_fused_weights_load(dir, use_tcm, block, HIDDEN, QHEADS, KVHEADS);
}
static inline fused_stats_t run_layer_fused(const layer_t *l, const fused_weights_t *fw,
                                            const float *x, uint16_t *kc, uint16_t *vc,
                                            int context, float *output, float *attn_capture,
                                            block_q8_0 *q8_capture) {
    return si_ref_run_layer_fused(l, fw, x, kc, vc, context, output, attn_capture, q8_capture,
                                  HIDDEN, QHEADS, KVHEADS, HDIM, ROPE_BASE, RMS_EPS);
}
static inline fused_stats_t run_layer_legacy_fused(const layer_t *l, const fused_weights_t *fw,
                                                   const float *x, uint16_t *kc, uint16_t *vc,
                                                   int context, float *output,
                                                   float *attn_capture, block_q8_0 *q8_capture) {
    return run_layer_fused(l, fw, x, kc, vc, context, output, attn_capture, q8_capture);
}
static inline fused_stats_t run_layer_soa_staged(const layer_t *l, const fused_weights_t *fw,
                                                 const float *x, uint16_t *kc, uint16_t *vc,
                                                 int context, float *out, float *attn_copy,
                                                 block_q8_0 *q8_copy) {
    return run_layer_fused(l, fw, x, kc, vc, context, out, attn_copy, q8_copy);
}
/* fused_layer.h:457 fused_total: all phase times plus TCM staging. */
static inline double fused_total(const fused_stats_t *p) {
    const phase_t *t = &p->phase;
    return (double)t->rms + t->q8_input + t->q_proj + t->k_proj + t->v_proj + t->rope_cache +
           t->attention + t->q8_output + t->out_proj + p->tcm_stage;
}
static inline void pf_workspace_open(pf_workspace_t *p, int ntok) {
    si_ref_pf_workspace_open(p, ntok, HIDDEN);
}
static inline void pf_run_batch(const layer_t *l, const fused_weights_t *fw,
                                rt_ai_pipeline_t *a, pf_workspace_t *p, const float *x,
                                int ntok, int prefix, uint16_t *kc, uint16_t *vc,
                                float *output) {
    si_ref_pf_run_batch(l, fw, a, p, x, ntok, prefix, kc, vc, output, HIDDEN, QHEADS, KVHEADS,
                        HDIM, ROPE_BASE, RMS_EPS);
}
/* qwen_one_layer.c:210 load_layer / :223 free_layer */
static inline layer_t load_layer(const char *dir) { return si_ref_load_layer(dir, HIDDEN, KVDIM); }
static inline void free_layer(layer_t *l) { si_ref_free_layer(l); }

#ifdef __cplusplus
}
#endif
#endif /* SI_B200_H */
