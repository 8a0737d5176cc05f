/*
 * cfi_glue.h -- element-wise helpers of libcfi_b200.so for the synthetic decode driver.
 *
 * No counterpart in cuda-for-intel: in a real deployment ggml runs its own get_rows, add, cpy, glu
 * and argmax kernels between the substituted ones.  These let a whole token step run on this
 * library's kernels (and be captured as one CUDA graph): positions and token ids are read from
 * device memory.  All pointers are device pointers; `stream` is a cudaStream_t; each returns 0 or
 * a CUDA error code.
 */
#ifndef CFI_GLUE_H
#define CFI_GLUE_H
#include <stdint.h>

#ifndef CFI_API
#define CFI_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* out[0..ncols) = row ids[0] of a row-major Q8_0 matrix, dequantised to f32 */
CFI_API int cfi_glue_get_rows_q8_0(const void *table, const int32_t *ids, float *out, int ncols, void *stream);
/* q += bq, k += bk, v += bv (nq and nkv values) */
CFI_API int cfi_glue_qkv_bias(float *q, float *k, float *v, const float *bq, const float *bk, const float *bv, int nq,
                              int nkv, void *stream);
/* K cache [kv head][pos][dim] and V cache [kv head][dim][pos] (f16, n_ctx positions) at pos[0];
 * q16 = f16(q).  A position outside [0, n_ctx) stores nothing in the caches (here and in the
 * fused cache stores below). */
CFI_API int cfi_glue_kv_store(const float *q, const float *k, const float *v, void *q16, void *kc, void *vc,
                              const int32_t *pos, int nq, int nkv, int head_dim, int n_ctx, void *stream);
/* mask[j] = 0 for j <= pos[0], -inf after */
CFI_API int cfi_glue_causal_mask(float *mask, const int32_t *pos, int n_ctx, void *stream);
/* y = f16(x) */
CFI_API int cfi_glue_to_f16(const float *x, void *y, int n, void *stream);
/* x += y */
CFI_API int cfi_glue_add(float *x, const float *y, int n, void *stream);
/* out = silu(g) * u */
CFI_API int cfi_glue_swiglu(const float *g, const float *u, float *out, int n, void *stream);
/* token[0] = first index of max(logits[0..n)); pos[0] += 1 (partials in the calling stream's own
 * scratch: calls on different streams may overlap) */
CFI_API int cfi_glue_argmax_next(const float *logits, int n, int32_t *token, int32_t *pos, void *stream);

/* Row-shard assembly after an all-gather (the multi-GPU split of the weight rows): src holds
 * `world` rank slices, slice r at src + r * src_rank_stride floats (0: ncols * rows_padded, the
 * slices back to back), each ncols columns of rows_padded = ceil(nrows / world) fp32 values
 * (rank r's rows first, padding after); dst gets ggml's column-major ncols x nrows output.  Rank
 * r owns rows [r*base + min(r, extra), ... + base + (r < extra)) with base = nrows / world,
 * extra = nrows % world (the split of shard.row_split).  A non-zero stride lets one all-gather
 * carry several products' slices (each rank's slices of a group back to back). */
CFI_API int cfi_glue_gather_row_shards(const float *src, float *dst, int nrows, int ncols, int world,
                                       long long src_rank_stride, void *stream);

/* Up to 4 mul_mat_q products that read the same q8_1_mmq activations y (K values, K % 256 == 0,
 * ncols <= 64 columns, y's block rows ncols_y >= ncols columns wide) in one launch of the skinny
 * kernel that the native mul_mat_q uses at <= 64 columns: product i writes dst[i][c *
 * stride_col_dst[i] + r] = sum_k W_i[r][k] y[c][k] for its nrows[i] rows, W_i in `type` blocks
 * (Q4_K = 12 or Q8_0 = 8; 16-byte aligned; stride_row_x[i] blocks per row, a multiple of 8 for
 * Q8_0).  The int32 block dots are exact; the fp32 sums agree with the separate products to
 * reassociation (the launch's shape is planned for all tiles together).  Batched decode: the q, k
 * and v products, or gate and up, in one launch instead of three or two. */
CFI_API int cfi_mmq_skinny_group(uint32_t type, int n, const void *const *x, const void *y, float *const *dst,
                                 const uint32_t *nrows, const uint32_t *stride_row_x, const uint32_t *stride_col_dst,
                                 uint32_t K, uint32_t ncols, uint32_t ncols_y, void *stream);

/*
 * Fused decode steps (one launch each where the ggml graph has two to five).  Results equal the
 * unfused chain where stated; n, nq, nkv multiples of 32.
 */
/* x += y (y may be NULL), then q8_1 blocks of rms_norm(x) * w: equal to cfi_glue_add, the native
 * rms_norm (with the weight multiply) and quantize_q8_1 in sequence, bit for bit.  n <= 8192. */
CFI_API int cfi_fused_add_rmsnorm_q8_1(float *x, const float *y, const float *w, void *out_q8_1, int n, float eps,
                                       void *stream);
/* qkv = [q | k | v] (nq + 2 nkv floats, the output of one GEMV over the stacked Q/K/V weights):
 * add the stacked biases, rope (NeoX, base theta, all head_dim dims) q into q_out and k, store k
 * and v (f16) at pos[0] in the caches of cfi_glue_kv_store's layout. */
CFI_API int cfi_fused_qkv_rope_store(const float *qkv, const float *bias, float *q_out, void *kc, void *vc,
                                     const int32_t *pos, int nq, int nkv, int head_dim, int n_ctx, float theta,
                                     void *stream);
/* Single-token attention over cache positions 0..pos[0]: per query head h (kv head h / (n_head /
 * n_kv_head)) softmax(scale K q) V in fp32 from the f16 caches, written as q8_1 blocks (head_dim
 * 64 or 128; n_head <= 64; n_ctx a multiple of 8, at most 8192; caches 16-byte aligned).  Split
 * over position ranges, the partials in the calling stream's own scratch. */
CFI_API int cfi_fused_attention_q8_1(const float *q, const void *kc, const void *vc, const int32_t *pos,
                                     void *out_q8_1, int n_head, int n_kv_head, int head_dim, int n_ctx, float scale,
                                     void *stream);
/* q8_1 blocks of silu(gu[i]) * gu[n + i], i < n: equal to cfi_glue_swiglu then quantize_q8_1. */
CFI_API int cfi_fused_swiglu_q8_1(const float *gu, void *out_q8_1, int n, void *stream);

/*
 * GEMV + fused step in one launch: y = W xq (W: rows x k Q8_0, row-major; xq: q8_1 blocks of one
 * column) through the streaming GEMV, whose last CTA to finish then runs the step on y.  Results
 * equal the GEMV followed by the standalone step, bit for bit.  The last-CTA counters are the
 * calling stream's own.
 */
/* ... then cfi_fused_add_rmsnorm_q8_1(x, y, norm_w, out, rows, eps); rows <= 8192 */
CFI_API int cfi_fused_mmvq_add_rmsnorm_q8_1(const void *w, const void *xq, float *y, int rows, int k, float *x,
                                            const float *norm_w, void *out_q8_1, float eps, void *stream);
/* ... then cfi_fused_swiglu_q8_1(y, out, rows / 2) */
CFI_API int cfi_fused_mmvq_swiglu_q8_1(const void *w, const void *xq, float *y, int rows, int k, void *out_q8_1,
                                       void *stream);
/* ... then cfi_fused_qkv_rope_store(y, ...) (rows = nq + 2 nkv) */
CFI_API int cfi_fused_mmvq_qkv_rope_store(const void *w, const void *xq, float *y, int k, const float *bias,
                                          float *q_out, void *kc, void *vc, const int32_t *pos, int nq, int nkv,
                                          int head_dim, int n_ctx, float theta, void *stream);

/*
 * One whole decode token step of a Q8_0 Qwen2-architecture model in a single persistent launch
 * (one CTA per SM, cooperative, grid-wide barriers between the phases): the op sequence of the
 * fused glue chain -- get_rows of token[0], per layer add_rmsnorm_q8_1 (x += dn), the stacked QKV
 * GEMV, qkv_rope_store, the split attention, the O GEMV, add_rmsnorm_q8_1 (x += o), the stacked
 * gate/up GEMV, swiglu_q8_1, the down GEMV; then add_rmsnorm_q8_1 with out_norm, the head GEMV and
 * argmax_next -- with the same results bit for bit (logits, token, pos, the caches, and x, hq,
 * qkv, qr, aq, o, gu, gq, dn as the chain leaves them).  hidden <= 1536 and a multiple of 64; ffn
 * a multiple of 64, ffn / 32 <= 384; head_dim 64 or 128; n_ctx a multiple of 8, at most 8192.
 * layers_dev: n_layers CfiDecodeLayer in device memory.  Returns a CUDA error code; a barrier
 * that times out (2 s) aborts the launch and records a code for cfi_decode_step_error().
 */
typedef struct {
    const void *wqkv;  /* (n_head + 2 n_kv_head) head_dim x hidden Q8_0: q, k, v rows stacked */
    const float *bqkv; /* the stacked biases */
    const void *wo;    /* hidden x n_head head_dim */
    const void *wgu;   /* 2 ffn x hidden: the gate rows, then the up rows */
    const void *wd;    /* hidden x ffn */
    const float *attn_norm, *ffn_norm;
    void *kc, *vc;     /* f16 K cache [kv head][pos][dim], V cache [kv head][dim][pos] */
} CfiDecodeLayer;
typedef struct {
    int hidden, n_head, n_kv_head, head_dim, ffn, vocab, n_ctx, n_layers;
    float eps, theta;
    const void *embd;     /* vocab x hidden Q8_0 token embedding */
    const void *head;     /* vocab x hidden Q8_0 output matrix */
    const float *out_norm;
    float *x, *qkv, *qr, *o, *gu, *dn, *logits;
    void *hq, *aq, *gq;   /* q8_1 buffers: hidden, n_head head_dim and ffn values */
    int32_t *token, *pos;
} CfiDecodeStep;
CFI_API int cfi_decode_step_q8_0(const CfiDecodeStep *s, const CfiDecodeLayer *layers_dev, void *stream);
/* Reads and clears the persistent decode step's error word (0: no barrier gave up). */
CFI_API unsigned int cfi_decode_step_error(void);

#ifdef __cplusplus
}
#endif
#endif
