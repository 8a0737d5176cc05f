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

// k_mmvq.cu: mul_mat_vec_q<ty, ncols> with one trailing u32 `nrows`.  Returns nullptr for an
// unsupported (ty, ncols).  Dynamic shared memory for a launch: cfi_mmvq_smem_bytes.
const void* cfi_native_mmvq(uint32_t ty, uint32_t ncols);
size_t cfi_mmvq_smem_bytes(uint32_t ty, uint32_t ncols, uint32_t ncols_x);
// Rows a warp computes at once (all loads of an iteration for those rows are issued together).
inline uint32_t cfi_mmvq_rows_per_warp(uint32_t ty, uint32_t ncols) {
    return ty == 12 ? (ncols == 1 ? 2 : 1) : (ncols <= 2 ? 2 : 1);
}
int cfi_mmvq_max_smem_bytes();
constexpr int CFI_MMVQ_THREADS = 256;
constexpr int CFI_MMVQ_WARPS = CFI_MMVQ_THREADS / 32;

// k_rowops.cu
const void* cfi_native_rms_norm(int do_multiply, int do_add);  // ggml rms_norm_f32<*, mul, add>
const void* cfi_native_rms_norm_plain();                        // rms_norm_f32<32> (iiilllf ABI)
const void* cfi_native_rope_neox(int forward, int has_ff);     // rope_neox<fwd, ff, float>
const void* cfi_native_soft_max(int mask_f16);                  // soft_max_f32<*, *, *, T>
constexpr int CFI_ROWOP_THREADS = 256;

// k_gemm_sm100.cu: tcgen05 GEMMs (own launch code; see cfi_gemm.h)
