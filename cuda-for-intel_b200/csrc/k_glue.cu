// k_glue.cu -- the small element-wise steps a decode step needs between the substituted kernels
// (ggml runs its own get_rows / add / cpy / glu / argmax kernels there).  They let the synthetic
// decode driver run a whole token step on this library's kernels alone; they are not part of the
// substitution table.  Each takes device pointers and a stream; positions and token ids are read
// from device memory so a captured step graph can be replayed token after token.
#include <cuda_fp16.h>
#include <math.h>

#include "../../include/cfi_glue.h"
#include "cfi_common.cuh"
#include "sm100_ptx.cuh"

#include <stdlib.h>
#include <string.h>

namespace {

// out[c] = d * q of row ids[0] of a Q8_0 matrix (ncols values, ncols % 32 == 0).
__global__ void get_rows_q8_0(const uint8_t* __restrict__ table, const int32_t* __restrict__ ids, float* __restrict__ out,
                              int ncols) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= ncols) return;
    const uint8_t* blk = table + ((size_t)ids[0] * (ncols / 32) + c / 32) * Q8_0_BYTES;
    const float d = h2f_bits((uint16_t)(blk[0] | (blk[1] << 8)));
    out[c] = d * (float)(int8_t)blk[2 + c % 32];
}

// q += bq, k += bk, v += bv; then K cache row pos (f16, [kv head][pos][dim]), V cache column pos
// (f16, [kv head][dim][pos]) and q as f16.
__global__ void qkv_store(float* __restrict__ q, float* __restrict__ k, float* __restrict__ v, const float* __restrict__ bq,
                          const float* __restrict__ bk, const float* __restrict__ bv, __half* __restrict__ q16,
                          __half* __restrict__ kc, __half* __restrict__ vc, const int32_t* __restrict__ pos, int nq,
                          int nkv, int head_dim, int n_ctx, int stage) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (stage == 0) {  // biases (before rope)
        if (i < nq) q[i] += bq[i];
        if (i < nkv) {
            k[i] += bk[i];
            v[i] += bv[i];
        }
        return;
    }
    const int p = pos[0];
    if (i < nq) q16[i] = __float2half_rn(q[i]);
    if (i < nkv) {
        const int h = i / head_dim, dd = i - h * head_dim;
        kc[((size_t)h * n_ctx + p) * head_dim + dd] = __float2half_rn(k[i]);
        vc[((size_t)h * head_dim + dd) * n_ctx + p] = __float2half_rn(v[i]);
    }
}

__global__ void causal_mask(float* __restrict__ mask, const int32_t* __restrict__ pos, int n_ctx) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j < n_ctx) mask[j] = j <= pos[0] ? 0.0f : -INFINITY;
}

__global__ void to_f16(const float* __restrict__ x, __half* __restrict__ y, int n) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __float2half_rn(x[i]);
}

__global__ void add_inplace(float* __restrict__ x, const float* __restrict__ y, int n) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] += y[i];
}

// out = silu(g) * u
__global__ void swiglu(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ out, int n) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float a = g[i];
        out[i] = a / (1.0f + expf(-a)) * u[i];
    }
}

// token[0] = argmax(logits) (first index of the maximum), pos[0] += 1.  One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) argmax_next(const float* __restrict__ logits, int n, int32_t* __restrict__ token,
                                                    int32_t* __restrict__ pos) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    __shared__ float bv[32];
    __shared__ int bi[32];
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = logits[i];
        if (v > best || (v == best && i < idx)) {
            best = v;
            idx = i;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) {
            best = ov;
            idx = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        bv[threadIdx.x >> 5] = best;
        bi[threadIdx.x >> 5] = idx;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        best = threadIdx.x < (blockDim.x >> 5) ? bv[threadIdx.x] : -INFINITY;
        idx = threadIdx.x < (blockDim.x >> 5) ? bi[threadIdx.x] : 0x7fffffff;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (ov > best || (ov == best && oi < idx)) {
                best = ov;
                idx = oi;
            }
        }
        if (threadIdx.x == 0) {
            token[0] = idx;
            pos[0] += 1;
        }
    }
}

inline dim3 g1(int n) { return dim3((unsigned)((n + 255) / 256)); }

// Launch with programmatic dependent launch unless CFI_PDL=0 (each kernel waits for its predecessor
// before reading anything).
template <typename... K, typename... A>
int launch(void (*k)(K...), dim3 grid, unsigned threads, void* stream, A... args) {
    static const bool pdl = [] {
        const char* e = getenv("CFI_PDL");
        return !(e && strcmp(e, "0") == 0);
    }();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, k, ((K)args)...);
}

}  // namespace

extern "C" int cfi_glue_get_rows_q8_0(const void* table, const int32_t* ids, float* out, int ncols, void* stream) {
    return launch(get_rows_q8_0, g1(ncols), 256, stream, (const uint8_t*)table, ids, out, ncols);
}
extern "C" int cfi_glue_qkv_bias(float* q, float* k, float* v, const float* bq, const float* bk, const float* bv, int nq,
                              int nkv, void* stream) {
    return launch(qkv_store, g1(nq > nkv ? nq : nkv), 256, stream, q, k, v, bq, bk, bv, (__half*)nullptr, (__half*)nullptr,
                  (__half*)nullptr, (const int32_t*)nullptr, nq, nkv, 1, 1, 0);
}
extern "C" int cfi_glue_kv_store(const float* q, const float* k, const float* v, void* q16, void* kc, void* vc,
                              const int32_t* pos, int nq, int nkv, int head_dim, int n_ctx, void* stream) {
    return launch(qkv_store, g1(nq > nkv ? nq : nkv), 256, stream, const_cast<float*>(q), const_cast<float*>(k),
                  const_cast<float*>(v), (const float*)nullptr, (const float*)nullptr, (const float*)nullptr, (__half*)q16,
                  (__half*)kc, (__half*)vc, pos, nq, nkv, head_dim, n_ctx, 1);
}
extern "C" int cfi_glue_causal_mask(float* mask, const int32_t* pos, int n_ctx, void* stream) {
    return launch(causal_mask, g1(n_ctx), 256, stream, mask, pos, n_ctx);
}
extern "C" int cfi_glue_to_f16(const float* x, void* y, int n, void* stream) {
    return launch(to_f16, g1(n), 256, stream, x, (__half*)y, n);
}
extern "C" int cfi_glue_add(float* x, const float* y, int n, void* stream) {
    return launch(add_inplace, g1(n), 256, stream, x, y, n);
}
extern "C" int cfi_glue_swiglu(const float* g, const float* u, float* out, int n, void* stream) {
    return launch(swiglu, g1(n), 256, stream, g, u, out, n);
}
extern "C" int cfi_glue_argmax_next(const float* logits, int n, int32_t* token, int32_t* pos, void* stream) {
    return launch(argmax_next, dim3(1), 1024, stream, logits, n, token, pos);
}
