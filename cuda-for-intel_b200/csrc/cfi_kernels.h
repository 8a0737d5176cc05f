// cfi_kernels.h -- host-side handles of the native sm_100a kernels (internal to the library).
//
// Every native kernel takes the caller's ggml parameter list unchanged (plus, where stated,
// trailing words the router appends), so a launch forwards the caller's kernelParams array.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

// k_quantize.cu
const void* cfi_native_quantize_q8_1();
const void* cfi_native_quantize_mmq(int ds4);

// k_mmvq.cu: mul_mat_vec_q<ty, ncols> with three trailing u32 words appended by the router:
// `nrows`, `chunk_rows` and `nstages` (rows per shared-memory stage and stage count of the
// streaming kernel, ncols <= 2; ignored by the row kernel of ncols >= 3).  Returns nullptr for an unsupported (ty, ncols);
// `stream` false selects the row kernel for ncols <= 2 as well.
const void* cfi_native_mmvq(uint32_t ty, uint32_t ncols, bool stream);
bool cfi_mmvq_streams(uint32_t ncols);
bool cfi_mmvq_stream_only(uint32_t ty);  // types without the row kernel (Q6_K, Q4_0)
// streaming kernel: rows per shared-memory stage and dynamic shared memory of a launch whose grid
// holds ctas_per_sm CTAs per SM
void cfi_mmvq_stream_layout(uint32_t ty, uint32_t ncols, uint32_t ncols_x, uint32_t nrows, uint32_t grid_x,
                            uint32_t stride_row_x, uint32_t chunk_target, uint32_t stage_budget, uint32_t max_stages,
                            uint32_t ctas_per_sm, uint32_t* chunk_rows, uint32_t* nstages, size_t* smem);
// direct-fill kernel (cfi_native_mmvq_direct, `nstages` 0): plain global loads into two
// register-fed stages of at most 16 KB.  False when the rows are strided or one row is larger than a stage.
bool cfi_mmvq_direct_layout(uint32_t ty, uint32_t ncols, uint32_t ncols_x, uint32_t nrows, uint32_t grid_x,
                            uint32_t stride_row_x, uint32_t* chunk_rows, size_t* smem);
// row kernel (ncols >= 3): dynamic shared memory of a launch
size_t cfi_mmvq_smem_bytes(uint32_t ty, uint32_t ncols, uint32_t ncols_x);
// Rows a warp of the row kernel computes at once (all loads of an iteration issued together).
inline uint32_t cfi_mmvq_rows_per_warp(uint32_t ty, uint32_t ncols) {
    return ty == 12 ? (ncols == 1 ? 2 : 1) : (ncols <= 2 ? 2 : 1);
}
// A deferred quantize_q8_1 absorbed by the streaming GEMV (the router's CFI_CTX_DEFER_Q8_1 mode):
// the fp32 activations x (column c at x + c * s01, ne00 real values), the q8_1 buffer the quantize
// would have written (nbq = ne0 / 32 blocks per column, columns contiguous) and nothing else.  The
// GEMV quantizes x in its prologue with the quantizer's own arithmetic and its CTAs together store
// every block of vy, so memory ends up as after quantize_q8_1 + mul_mat_vec_q.  Passed by value
// after the three trailing words.
struct CfiFuseQ {
    const float* x;
    uint8_t* vy;
    int64_t ne00, s01;
    uint32_t nbq, pad;
};
// the GEMV with the quantize in its prologue, on the direct-fill or the bulk-copy layout (the
// same trailing words as that layout's kernel, then the CfiFuseQ); nullptr above 4 columns
const void* cfi_native_mmvq_q81(uint32_t ty, uint32_t ncols, bool direct);
// tensor-core Q4_K GEMV for 3..8 columns (exact int32 block dots, fp32 scales reassociated):
// same parameters and trailing words as the streaming kernel; false when the layout does not fit
const void* cfi_native_mmvq_mma(uint32_t ty, uint32_t ncols);
bool cfi_mmvq_mma_layout(uint32_t ncols_x, uint32_t nrows, uint32_t grid_x, uint32_t ctas_per_sm, uint32_t chunk_target,
                         uint32_t stage_budget, uint32_t max_stages, uint32_t* chunk_rows, uint32_t* nstages,
                         size_t* smem);
const void* cfi_native_mmvq_direct(uint32_t ty, uint32_t ncols);  // the direct-fill kernel (nstages 0)
int cfi_mmvq_max_smem_bytes();
unsigned int cfi_mmvq_error_take();
constexpr int CFI_MMVQ_THREADS = 256;
constexpr int CFI_MMVQ_WARPS = CFI_MMVQ_THREADS / 32;

// k_rowops.cu
const void* cfi_native_rms_norm(int do_multiply, int do_add);  // ggml rms_norm_f32<*, mul, add>
const void* cfi_native_rms_norm_block(int do_multiply, int do_add);  // the same, one CTA per row (small launches)
const void* cfi_native_rms_norm_plain();                        // rms_norm_f32<32> (iiilllf ABI)
const void* cfi_native_rope_neox(int forward, int has_ff);     // rope_neox<fwd, ff, float>
const void* cfi_native_soft_max(int mask_f16);                  // soft_max_f32<*, *, *, T>
// warp-per-row soft_max (ncols % 4 == 0, <= cfi_soft_max_rows_max_cols(), aligned rows); trailing u32 ne01
const void* cfi_native_soft_max_rows(int mask_f16);
int cfi_soft_max_rows_max_cols();
int cfi_rope_rows_per_warp(uint32_t nrows);  // rope_neox rows per warp for a launch of nrows rows (1: small)
const void* cfi_native_rope_neox_pairs(int forward, int has_ff);  // thread per pair, for small launches
int cfi_rope_max_ne0();       // longest row rope_neox takes (pairs per lane kept in registers)
constexpr int CFI_ROWOP_THREADS = 256;

// k_gemm_sm100.cu: tcgen05 GEMM on K-major fp16/bf16 operands, fp32 accumulation:
//   C[plane][col][row] = alpha * sum_k A[aplane][row][k] * B[plane][col][k] (+ beta * C)
// Output plane p: channel p % nch, sample p / nch; its A plane (sample / smr) * (nch / chr) +
// channel / chr.  Strides in elements.  Returns 0 when launched, -1 when the operands cannot be
// described by tensor maps (alignment), or a CUDA error code.
struct TcGemm {
    const void* a;
    const void* b;
    void* c;
    int fmt;  // 0 f16, 1 bf16
    uint32_t m, n, k;
    uint64_t lda, ldb, a_plane, b_plane;
    uint32_t a_planes, nch, nsamples, chr, smr;
    int c_type;  // CFI_R_32F / 16F / 16BF
    uint64_t ldc;
    long long c_zstride, c_wstride;
    float alpha, beta;
    const void* alpha_ptr;
    const void* beta_ptr;
    int scalar_f16;
};
int cfi_tc_gemm(const TcGemm& d, cudaStream_t stream);

// Split-K support of k_gemm_sm100.cu shared with the quantized GEMM: a per-device fp32 workspace
// (grown outside stream capture; nullptr when it cannot be; replaced buffers stay allocated) and
// the ordered reduction C[plane][col][row] = sum over splits of ws[split][plane][col][row] (f32 C,
// alpha 1, beta 0; plane p: channel p % nch, sample p / nch).
float* cfi_splitk_workspace(size_t bytes, cudaStream_t stream);
int cfi_splitk_reduce_f32(const float* ws, uint32_t ld_ws, uint32_t m, uint32_t n, uint32_t planes, uint32_t splits,
                          float* c, long long ldc, long long c_zstride, long long c_wstride, uint32_t nch,
                          cudaStream_t stream, bool pdl);

// ---- per-(device, stream) scratch (stream_state.cpp) ----
constexpr int CFI_AMAX_CTAS = 148;                                  // argmax_next CTAs
constexpr int CFI_ATT_MAX_HEADS = 64, CFI_ATT_MAX_SPLIT = 64;        // split attention partials
struct CfiGlueSlot {
    unsigned int* amax_count;  // 1
    unsigned int* att_count;   // CFI_ATT_MAX_HEADS
    unsigned int* epi_count;   // 4 (GEMVs with a fused decode step, one per step kind)
    float* amax_val;           // CFI_AMAX_CTAS
    int* amax_idx;             // CFI_AMAX_CTAS
    float* att_part;           // CFI_ATT_MAX_HEADS x CFI_ATT_MAX_SPLIT x (2 + 128)
};
// The glue slot of the current device and `stream` (0 or a CUDA error code).
int cfi_glue_slot(cudaStream_t stream, CfiGlueSlot* out);
// A buffer of at least `bytes` for (current device, stream, kind), grown outside stream capture
// only (*err = cudaErrorStreamCaptureUnsupported when it would have to grow under capture).
// (CFI_BUF_COUNTERS buffers are zeroed when allocated; their kernels leave them at zero)
enum { CFI_BUF_SPLITK = 1, CFI_BUF_MMQ_SCRATCH = 2, CFI_BUF_SKINNY_WS = 3, CFI_BUF_COUNTERS = 4, CFI_BUF_DECODE_SYNC = 5 };
void* cfi_stream_buffer(int kind, size_t bytes, cudaStream_t stream, int* err);

// The library's device error word (k_mmq_sm100.cu; read and cleared by cfi_device_error).
unsigned int* cfi_device_error_word();

// ---- k_mmq_skinny.cu: mul_mat_q for at most 64 columns (Q4_K / Q8_0, one plane, K % 256 == 0) ----
bool cfi_mmq_skinny_applies(uint32_t ty, const void* x, const void* y, uint32_t K, uint32_t ncols_dst,
                            uint32_t stride_row_x, uint32_t planes);
// A rank's group for the all-gather over peer memory, as the kernels take it (cfi_peer.h's
// CfiPeerSet, checked, plus the wait bound): with world == 1 a launch stores only locally.
constexpr int CFI_MAX_RANKS = 8;
struct CfiPeerDev {
    int rank, world;
    long long delta[CFI_MAX_RANKS];            // byte offset to rank r's copy (0 for this rank)
    unsigned int* sig_remote[CFI_MAX_RANKS];  // rank r's slot for this rank
    unsigned int* sig_local;                  // this rank's slots, one per rank
    unsigned int* expect;                     // this rank's wait counts, one per rank
    unsigned long long limit_ns;              // bound of each wait for a peer
};
struct CfiPeerSet;
// Checks a CfiPeerSet and fills `out` (k_peer.cu); 0 or cudaErrorInvalidValue.
int cfi_peer_dev(const CfiPeerSet* in, CfiPeerDev* out);
// n <= 4 products over the same activations in one launch (their tiles back to back)
int cfi_mmq_skinny_group_launch(uint32_t ty, int n, const void* const* x, const void* y, float* const* dst,
                                const uint32_t* nrows, const uint32_t* stride_row_x, const uint32_t* stride_col_dst,
                                uint32_t K, uint32_t ncols_dst, uint32_t ncols_y, unsigned int* err, cudaStream_t stream,
                                bool pdl, const CfiPeerDev* peers = nullptr);
int cfi_mmq_skinny_launch(uint32_t ty, const void* x, const void* y, float* dst, uint32_t K, uint32_t nrows,
                          uint32_t ncols_dst, uint32_t ncols_y, uint32_t stride_row_x, uint32_t stride_col_dst,
                          unsigned int* err, cudaStream_t stream, bool pdl);
