/*
 * cfi_oracle.h -- CPU oracle for the ggml kernel-substitution hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a scalar C restatement of the host reference math of
 * cuda-for-intel's substitution layer (src/subst/refs.rs, src/subst/probe.rs,
 * src/ptx/ggml_ref.rs, crates/cublas_shim/src/plan.rs and the inline CPU references of
 * tests/gpu/{ggml_rms_norm,ggml_rope,soft_max_generic}.rs).  Only the test suite, the smoke
 * check and the CPU-baseline leg of bench.py may load it; the product library never links it.
 *
 * Parity status: numeric parity is UNPINNED against reference outputs -- the reference ships
 * no golden vectors for this path and its Rust toolchain is absent here.  The restatement is
 * cross-checked against the reference's own second opinion (the f64 block decoder of
 * src/ptx/ggml_ref.rs, restated below as cfo_dot_ref_f64) and against the invariants its tests
 * assert (stock-order vs decode-fast mmvq nmse < 1e-10, src/subst/tests.rs:566-582).
 *
 * Every function names the reference file:line it follows.  Float expressions keep the exact
 * operation structure of the reference (build with -ffp-contract=off; fmaf only where the
 * reference calls mul_add).
 */
#ifndef CFI_ORACLE_H
#define CFI_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { CFO_Q4_0 = 2, CFO_Q5_0 = 6, CFO_Q8_0 = 8, CFO_Q4_K = 12, CFO_Q5_K = 13, CFO_Q6_K = 14 };

/* refs.rs:35-80 */
float cfo_f16_to_f32(uint16_t h);
uint16_t cfo_f32_to_f16(float x);
/* refs.rs:83-100 */
void cfo_fastdiv_values(uint32_t d, uint32_t out[3]);
uint32_t cfo_fastdiv(uint32_t n, const uint32_t v[3]);
uint32_t cfo_fastmodulo(uint32_t n, const uint32_t v[3]);
/* refs.rs:149-155 */
int32_t cfo_dp4a(uint32_t a, uint32_t b, int32_t c);

/* refs.rs:501-515 (xorshift64*) */
uint64_t cfo_rng_next(uint64_t *s);
uint32_t cfo_rng_u32(uint64_t *s);
float cfo_rng_unit(uint64_t *s);
/* refs.rs:518-538 */
size_t cfo_block_bytes(uint32_t ty);
void cfo_random_blocks(uint32_t ty, size_t nblocks, uint64_t *rng, uint8_t *out);
/* refs.rs:540-547 */
double cfo_nmse(const float *got, const float *want, size_t n);

/* refs.rs:119-147: quantize n (multiple of 32) floats into n/32 q8_1 blocks of 36 bytes */
void cfo_quantize_q8_1(const float *x, size_t n, uint8_t *out);

/* refs.rs:169-259: per-thread vec_dot of one x block against the aligned q8_1 block(s) */
float cfo_vec_dot(uint32_t ty, const uint8_t *xb, const uint8_t *yb, size_t kqs, float acc);
/* refs.rs:386-433: wide per-lane dot of 32-value group g */
float cfo_vec_dot_wide(uint32_t ty, const uint8_t *xb, const uint8_t *yb, size_t g, float acc);

/* refs.rs:261-283 */
typedef struct cfo_mmvq {
    uint32_t ty, ncols_dst, nwarps, nrows_x, ncols_x, nchannels_dst, nsamples_dst;
    uint32_t channel_ratio, sample_ratio, nchannels_y, use_ids;
    uint32_t stride_row_x, stride_col_y, stride_col_dst;
    uint32_t stride_channel_x, stride_channel_y, stride_channel_dst;
    uint32_t stride_sample_x, stride_sample_y, stride_sample_dst;
} cfo_mmvq;

/* refs.rs:304-382: stock thread-order mul_mat_vec_q (dst updated in place) */
void cfo_mmvq_run(const cfo_mmvq *p, const uint8_t *x, const uint8_t *y, const int32_t *ids, float *dst);
/* refs.rs:438-497: decode-fast variant (ncols_dst 1) */
void cfo_mmvq_fast(const cfo_mmvq *p, const uint8_t *x, const uint8_t *y, const int32_t *ids, float *dst,
                   uint32_t warps, uint32_t unroll, int wide);

/* probe.rs:33-78: the reference's mmvq known-answer case.  With the *_sizes call first, the
 * caller learns the buffer sizes; the fill call writes p, x (weights), y (q8_1) and ids. */
void cfo_mmvq_case_sizes(uint32_t ty, uint32_t ncols_dst, uint32_t nrows, uint32_t ncols_x, uint32_t nch,
                         uint32_t ratio, uint32_t nsamples, int use_ids, size_t *x_bytes, size_t *y_bytes,
                         size_t *nids, size_t *dst_len);
void cfo_mmvq_case(uint32_t ty, uint32_t ncols_dst, uint32_t nrows, uint32_t ncols_x, uint32_t nch,
                   uint32_t ratio, uint32_t nsamples, int use_ids, uint64_t seed, cfo_mmvq *p, uint8_t *x,
                   uint8_t *y, int32_t *ids);

/* probe.rs:182-204: quantize known-answer case (x: ne00*ne1*ne2*ne3 floats) and its reference */
void cfo_quantize_case_x(size_t ne00, size_t ne1, size_t ne2, size_t ne3, uint64_t seed, float *x);
void cfo_quantize_case_reference(const float *x, size_t ne00, size_t ne0, size_t rows, uint8_t *out);

/* refs.rs:556-575, 744-769: block_q8_1_mmq layout (144 B per 128 values per column) */
int cfo_mmq_ds4(uint32_t ty);
size_t cfo_mmq_groups(uint32_t ty);
void cfo_quantize_mmq(uint32_t ty, const float *x, size_t ne0, size_t ncols, uint8_t *out);

/* refs.rs:577-595 */
typedef struct cfo_mmq {
    uint32_t ncols_x, nrows_x, ncols_dst, nchannels_y, nsamples_y, channel_ratio, sample_ratio;
    uint32_t stride_row_x, ncols_y, stride_col_dst, stride_channel_x, stride_channel_y, stride_channel_dst;
    uint32_t stride_sample_x, stride_sample_y, stride_sample_dst;
} cfo_mmq;
/* refs.rs:773-834 */
void cfo_mmq_ref(uint32_t ty, const cfo_mmq *p, const uint8_t *x, const uint8_t *y, float *dst);
/* probe.rs:249-279 */
void cfo_mmq_case_sizes(uint32_t ty, uint32_t ncols_x, uint32_t nrows, uint32_t ncols, uint32_t nch,
                        uint32_t ratio, uint32_t nsamples, size_t *x_bytes, size_t *y_bytes, size_t *dst_len);
void cfo_mmq_case(uint32_t ty, uint32_t ncols_x, uint32_t nrows, uint32_t ncols, uint32_t nch, uint32_t ratio,
                  uint32_t nsamples, uint64_t seed, cfo_mmq *p, uint8_t *x, uint8_t *y);

/* src/ptx/ggml_ref.rs:169-446: f64 dequantised dot of one quantized row against q8_1 blocks
 * (the reference's independent second opinion).  Returns the total; *abs gets sum |terms|. */
double cfo_dot_ref_f64(uint32_t ty, const uint8_t *row, size_t nblocks, const uint8_t *y, double *abs_sum);

/* crates/cublas_shim/src/plan.rs:160-215 -- 0 ok, 7 INVALID_VALUE, 15 NOT_SUPPORTED */
int cfo_gemm_validate(int transa, int transb, int m, int n, int k, int lda, int ldb, int ldc, int a_type,
                      int b_type, int c_type, int compute_type);
/* plan.rs:346-362: literal column-major reference GEMM (a_type/c_type are cudaDataType ids) */
void cfo_reference_gemm(int transa, int transb, int m, int n, int k, float alpha, const void *a, int a_type,
                        int lda, const void *b, int ldb, float beta, void *c, int c_type, int ldc);

/* tests/gpu/ggml_rms_norm.rs:43-55 (+ weight multiply): rows x ncols contiguous */
void cfo_rms_norm(const float *x, const float *w, float *dst, size_t rows, size_t ncols, float eps);
/* NeoX rotate-half rope over rows of ne0 with n_dims rotated; pos per channel (row / ne1) */
void cfo_rope_neox(const float *x, float *dst, size_t ne0, size_t ne1, size_t nch, size_t n_dims,
                   const int32_t *pos, float freq_base, float freq_scale, float attn_factor, const float *ff);
/* tests/gpu/soft_max_generic.rs:73-92 (+ ALiBi slope and sinks): rows of ncols, row r uses
 * mask row (r % ne01) and head (r / ne01) % nheads. mask may be NULL. */
void cfo_soft_max(const float *x, const float *mask, const float *sinks, float *dst, size_t ncols, size_t ne01,
                  size_t nheads, size_t rows, float scale, float max_bias);

/* cpu_baseline.c: one host decode step (quantize + row-parallel GEMV); returns threads used */
/* ---- FlashAttention case and exact reference (src/subst/probe.rs:405-489) ----
 * Q [ns][nh][nq][d] f32, K/V [ns][nh_kv][nkv][d] f16, mask [ns][nq_pad][nkv] f16 (or none),
 * dst [ns][nq][nh][d] f32; nq_pad = nq rounded up to 16. */
void cfo_fattn_case(uint32_t d, uint32_t nq, uint32_t nh, uint32_t nh_kv, uint32_t nkv, uint32_t ns, int causal,
                    uint64_t seed, float *q, uint16_t *k, uint16_t *v, uint16_t *mask);
void cfo_fattn_reference(uint32_t d, uint32_t nq, uint32_t nh, uint32_t nh_kv, uint32_t nkv, uint32_t ns,
                         const float *q, const uint16_t *k, const uint16_t *v, const uint16_t *mask, float scale,
                         float *dst);

int cfo_cpu_decode_step(uint32_t ty, const uint8_t *w, size_t rows, size_t ncols_x, const float *x,
                        size_t ncols_dst, uint8_t *yq, float *dst, int threads);

#ifdef __cplusplus
}
#endif
#endif
