// k_mmq_sm100.cu -- prefill quantized GEMM on the 5th-generation tensor cores (sm_100a).
#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "subst_host.hpp"

static __device__ unsigned int g_cfi_device_error;

namespace cfi {
int mmq_tile_n(uint32_t ncols_dst) { return ncols_dst > 128 ? 256 : 128; }
int mmq_threads() { return 192; }
bool mmq_type_ok(uint32_t) { return false; }
int mmq_launch(const cfi_plan&, void**, void*) { return (int)cudaErrorNotSupported; }
}  // namespace cfi

extern "C" unsigned int cfi_device_error(void) {
    unsigned int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_cfi_device_error, sizeof v) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaMemcpyToSymbol(g_cfi_device_error, &z, sizeof z);
    return v;
}
