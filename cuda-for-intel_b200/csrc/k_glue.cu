// k_glue.cu -- the small element-wise steps a decode step needs between the substituted kernels
// (ggml runs its own get_rows / add / cpy / glu / argmax kernels there).  They let the synthetic
// decode driver run a whole token step on this library's kernels alone; they are not part of the
// substitution table.  Each takes device pointers and a stream; positions and token ids are read
// from device memory so a captured step graph can be replayed token after token.
#include <cuda_fp16.h>
#include <math.h>

#include "../../include/cfi_glue.h"
#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "sm100_ptx.cuh"
#include "decode_epi.cuh"

#include <stdlib.h>
#include <algorithm>
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
    if (i < nkv && p >= 0 && p < n_ctx) {  // a position outside the cache stores nothing
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

// token[0] = argmax(logits) (first index of the maximum), pos[0] += 1.  AMAX_CTAS CTAs reduce
// contiguous ranges; the last CTA to finish (the slot's counter) reduces their results in CTA
// order and resets the counter.  The partials live in the calling stream's glue slot.
constexpr int AMAX_CTAS = CFI_AMAX_CTAS;

CFI_DEV void amax_pair_reduce(float& best, int& idx) {
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) {
            best = ov;
            idx = oi;
        }
    }
}

__global__ void __launch_bounds__(512) argmax_next(const float* __restrict__ logits, int n, int32_t* __restrict__ token,
                                                   int32_t* __restrict__ pos, float* __restrict__ amax_val,
                                                   int* __restrict__ amax_idx, unsigned int* __restrict__ amax_count) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    __shared__ float bv[16];
    __shared__ int bi[16];
    __shared__ int last;
    const int chunk = (n + (int)gridDim.x - 1) / (int)gridDim.x;
    const int lo = blockIdx.x * chunk, hi = min(n, lo + chunk);
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = lo + (int)threadIdx.x; i < hi; i += blockDim.x) {
        const float v = logits[i];
        if (v > best || (v == best && i < idx)) {
            best = v;
            idx = i;
        }
    }
    amax_pair_reduce(best, idx);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        bv[warp] = best;
        bi[warp] = idx;
    }
    __syncthreads();
    if (warp == 0) {
        best = lane < (int)(blockDim.x >> 5) ? bv[lane] : -INFINITY;
        idx = lane < (int)(blockDim.x >> 5) ? bi[lane] : 0x7fffffff;
        amax_pair_reduce(best, idx);
        if (lane == 0) {
            amax_val[blockIdx.x] = best;
            amax_idx[blockIdx.x] = idx;
            __threadfence();
            last = atomicAdd(amax_count, 1u) == gridDim.x - 1;
        }
    }
    __syncthreads();
    if (!last || warp != 0) return;
    __threadfence();
    best = -INFINITY;
    idx = 0x7fffffff;
    for (int b = lane; b < (int)gridDim.x; b += 32) {
        const float v = __ldcg(&amax_val[b]);
        const int i = __ldcg(&amax_idx[b]);
        if (v > best || (v == best && i < idx)) {
            best = v;
            idx = i;
        }
    }
    amax_pair_reduce(best, idx);
    if (lane == 0) {
        token[0] = idx;
        pos[0] += 1;
        *amax_count = 0;
    }
}

// ---- fused decode steps (block-level bodies in decode_epi.cuh) ----

// Block sum over 256 threads in the order of the native rms_norm (thread-strided partials, warp
// butterfly, then the 8 warp sums by a second butterfly).
CFI_DEV float block_sum256(float v, float* red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
    return warp_sum(t);
}

__global__ void __launch_bounds__(1024) add_rmsnorm_q81(float* __restrict__ x, const float* __restrict__ y,
                                                        const float* __restrict__ w, uint8_t* __restrict__ out, int n,
                                                        float eps) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    extern __shared__ float hbuf[];
    epi_add_rmsnorm_q81(x, y, w, out, n, eps, hbuf);
}

__global__ void __launch_bounds__(256) qkv_rope_store(const float* __restrict__ qkv, const float* __restrict__ bias,
                                                      float* __restrict__ q_out, __half* __restrict__ kc,
                                                      __half* __restrict__ vc, const int32_t* __restrict__ pos, int nq,
                                                      int nkv, int head_dim, int n_ctx, float theta_scale) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    epi_qkv_rope_store(qkv, bias, q_out, kc, vc, pos, nq, nkv, head_dim, n_ctx, theta_scale,
                       blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
}

// Split over positions (flash-decoding): CTA (h, s) of grid (n_head, nsplit) takes the positions
// [s chunk, (s + 1) chunk) that are <= pos[0] for query head h: scores (thread t: position t of the
// range, the K row read whole with 16-byte loads), the range's max m_s, e_j = exp(score_j - m_s),
// l_s = sum e_j and o_s[d] = sum e_j V[d][j] (256 / head_dim threads per dim over 8-position runs
// of the V^T row).  The partials go to the slot; the last CTA of the head (the slot's counter)
// combines them in split order, out[d] = sum_s o_s[d] e^(m_s - M) / sum_s l_s e^(m_s - M), writes
// the head_dim / 32 q8_1 blocks and resets the counter.  The partials and counters live in the
// calling stream's glue slot.
constexpr int ATT_MAX_CTX = 8192, ATT_MAX_HEADS = CFI_ATT_MAX_HEADS, ATT_MAX_SPLIT = CFI_ATT_MAX_SPLIT, ATT_CHUNK = 128;

__global__ void __launch_bounds__(256) attention_q81(const float* __restrict__ q, const __half* __restrict__ kc,
                                                    const __half* __restrict__ vc, const int32_t* __restrict__ pos,
                                                    uint8_t* __restrict__ out, int n_head, int n_kv_head, int head_dim,
                                                    int n_ctx, float scale, int chunk, float* __restrict__ att_part,
                                                    unsigned int* __restrict__ att_count) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    __shared__ float sc[ATT_CHUNK * 2];
    __shared__ float red[32];
    __shared__ __align__(16) float qs[128];
    __shared__ float o[128];
    __shared__ int last;
    const int h = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y, kvh = h / (n_head / n_kv_head);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int npos = min(pos[0] + 1, n_ctx);
    const int j0 = split * chunk, j1 = min(npos, j0 + chunk);  // j1 <= j0: empty range
    const __half* K = kc + (size_t)kvh * n_ctx * head_dim;
    const __half* V = vc + (size_t)kvh * head_dim * n_ctx;
    if (tid < head_dim) qs[tid] = q[(size_t)h * head_dim + tid];
    __syncthreads();
    // ---- scores of the range ----
    float mx = -INFINITY;
    const int nv = head_dim / 8;
    for (int jj = tid; j0 + jj < j1; jj += 256) {
        const uint4* kr = reinterpret_cast<const uint4*>(K + (size_t)(j0 + jj) * head_dim);
        uint4 kv[16];
#pragma unroll
        for (int e = 0; e < 16; e++)
            if (e < nv) kv[e] = __ldg(kr + e);
        float acc = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; e++) {
            if (e < nv) {
                const __half2* hp = reinterpret_cast<const __half2*>(&kv[e]);
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const float2 f = __half22float2(hp[t]);
                    acc = __fmaf_rn(qs[8 * e + 2 * t], f.x, acc);
                    acc = __fmaf_rn(qs[8 * e + 2 * t + 1], f.y, acc);
                }
            }
        }
        const float sj = acc * scale;
        sc[jj] = sj;
        mx = fmaxf(mx, sj);
    }
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = warp_max(lane < 8 ? red[lane] : -INFINITY);
    __syncthreads();
    float sum = 0.0f;
    const int cnt = max(0, j1 - j0), cpad = (cnt + 7) & ~7;
    for (int jj = tid; jj < cpad; jj += 256) {
        const float e = jj < cnt ? expf(sc[jj] - mx) : 0.0f;
        sc[jj] = e;
        sum += e;
    }
    sum = block_sum256(sum, red);
    __syncthreads();
    // ---- unnormalised output of the range ----
    const int tpd = 256 / head_dim, d = tid / tpd, part = tid % tpd;
    const uint4* vr = reinterpret_cast<const uint4*>(V + (size_t)d * n_ctx + j0);
    const int nrun = cpad / 8;
    float acc = 0.0f;
    for (int r0 = part; r0 < nrun; r0 += 4 * tpd) {
        uint4 vv[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int r = r0 + u * tpd;
            vv[u] = r < nrun ? __ldg(vr + r) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int r = r0 + u * tpd;
            if (r < nrun) {
                const __half2* hp = reinterpret_cast<const __half2*>(&vv[u]);
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const float2 f = __half22float2(hp[t]);
                    acc = __fmaf_rn(sc[8 * r + 2 * t], f.x, acc);
                    acc = __fmaf_rn(sc[8 * r + 2 * t + 1], f.y, acc);
                }
            }
        }
    }
    for (int off = tpd / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    float* pp = att_part + ((size_t)h * ATT_MAX_SPLIT + split) * (2 + 128);
    if (part == 0) pp[2 + d] = acc;
    if (tid == 0) {
        pp[0] = mx;
        pp[1] = sum;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&att_count[h], 1u) == (unsigned)nsplit - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    // ---- combine the splits in order ----
    const float* hp0 = att_part + (size_t)h * ATT_MAX_SPLIT * (2 + 128);
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; sp++) M = fmaxf(M, __ldcg(hp0 + sp * (2 + 128)));
    if (tid < head_dim) {
        float num = 0.0f, den = 0.0f;
        for (int sp = 0; sp < nsplit; sp++) {
            const float* ps = hp0 + sp * (2 + 128);
            const float ms = __ldcg(ps);
            if (ms == -INFINITY) continue;  // empty range
            const float f = expf(ms - M);
            num = __fmaf_rn(__ldcg(ps + 2 + tid), f, num);
            den = __fmaf_rn(__ldcg(ps + 1), f, den);
        }
        o[tid] = num / den;
    }
    __syncthreads();
    for (int b = warp; b < head_dim / 32; b += 8)
        q8_1_store_lane(o[32 * b + lane], out + ((size_t)h * (head_dim / 32) + b) * Q8_1_BYTES, lane);
    if (tid == 0) att_count[h] = 0;
}

// One warp per q8_1 block.
__global__ void __launch_bounds__(256) swiglu_q81(const float* __restrict__ gu, uint8_t* __restrict__ out, int n) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    epi_swiglu_q81(gu, out, n, blockIdx.x * 8 + (threadIdx.x >> 5), gridDim.x * 8);
}

// Row-shard assembly after an all-gather of column-major slices: src holds `world` slices (slice r
// at src + r * rank_stride) of ncols columns x rows_padded values (rank r's rows first, padding
// after), dst ggml's column-major ncols x nrows output; rank r owns rows
// [r*base + min(r, extra), +base + (r < extra)).
__global__ void __launch_bounds__(256) gather_row_shards(const float* __restrict__ src, float* __restrict__ dst,
                                                         uint32_t nrows, uint32_t ncols, uint32_t world,
                                                         uint64_t rank_stride) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const uint32_t base = nrows / world, extra = nrows - base * world, rp = base + (extra ? 1u : 0u);
    const uint64_t total = (uint64_t)nrows * ncols;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t c = (uint32_t)(i / nrows), row = (uint32_t)(i - (uint64_t)c * nrows);
        // rank of `row`: the first `extra` ranks hold base + 1 rows
        const uint32_t big = extra * (base + 1u);
        const uint32_t r = row < big ? row / (base + 1u) : extra + (row - big) / base;
        const uint32_t row0 = r * base + min(r, extra);
        dst[i] = src[(uint64_t)r * rank_stride + (uint64_t)c * rp + (row - row0)];
    }
}

inline dim3 g1(int n) { return dim3((unsigned)((n + 255) / 256)); }

// Launch with programmatic dependent launch unless CFI_PDL=0 (each kernel waits for its predecessor
// before reading anything).
template <typename... K, typename... A>
int launch_smem(void (*k)(K...), dim3 grid, unsigned threads, size_t smem, void* stream, A... args) {
    static const bool pdl = [] {
        const char* e = getenv("CFI_PDL");
        return !(e && strcmp(e, "0") == 0);
    }();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, k, ((K)args)...);
}

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
    CfiGlueSlot sl;
    const int rc = cfi_glue_slot(static_cast<cudaStream_t>(stream), &sl);
    if (rc) return rc;
    return launch(argmax_next, dim3(AMAX_CTAS), 512, stream, logits, n, token, pos, sl.amax_val, sl.amax_idx, sl.amax_count);
}

extern "C" int cfi_glue_gather_row_shards(const float* src, float* dst, int nrows, int ncols, int world,
                                          long long src_rank_stride, void* stream) {
    if (nrows <= 0 || ncols <= 0 || world <= 0 || world > nrows || src_rank_stride < 0) return (int)cudaErrorInvalidValue;
    const uint64_t rp = (uint64_t)(nrows / world + (nrows % world ? 1 : 0));
    const uint64_t rs = src_rank_stride ? (uint64_t)src_rank_stride : rp * (uint64_t)ncols;
    if (rs < rp * (uint64_t)ncols) return (int)cudaErrorInvalidValue;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t total = (uint64_t)nrows * (uint64_t)ncols;
    const unsigned grid = (unsigned)std::max<uint64_t>(1, std::min<uint64_t>((total + 255) / 256, (uint64_t)sms * 8));
    return launch(gather_row_shards, dim3(grid), 256, stream, src, dst, (uint32_t)nrows, (uint32_t)ncols, (uint32_t)world, rs);
}

extern "C" int cfi_fused_add_rmsnorm_q8_1(float* x, const float* y, const float* w, void* out, int n, float eps,
                                          void* stream) {
    if (n <= 0 || n % 32 || n > 8192) return (int)cudaErrorInvalidValue;
    const size_t smem = (size_t)n * 4;
    if (smem > 48 * 1024) cudaFuncSetAttribute(add_rmsnorm_q81, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const unsigned threads = (unsigned)std::max(256, std::min(1024, n));  // n is a multiple of 32
    return launch_smem(add_rmsnorm_q81, dim3(1), threads, smem, stream, x, y, w, (uint8_t*)out, n, eps);
}
extern "C" int cfi_fused_qkv_rope_store(const float* qkv, const float* bias, float* q_out, void* kc, void* vc,
                                        const int32_t* pos, int nq, int nkv, int head_dim, int n_ctx, float theta,
                                        void* stream) {
    if (head_dim <= 0 || head_dim % 2 || nq % head_dim || nkv % head_dim) return (int)cudaErrorInvalidValue;
    // theta_scale = theta^(-2 / n_dims), computed on the host as the rope_neox caller does
    const float theta_scale = powf(theta, -2.0f / (float)head_dim);
    return launch(qkv_rope_store, g1((nq + nkv) / 2 + nkv), 256, stream, qkv, bias, q_out, (__half*)kc, (__half*)vc,
                  pos, nq, nkv, head_dim, n_ctx, theta_scale);
}
extern "C" int cfi_fused_attention_q8_1(const float* q, const void* kc, const void* vc, const int32_t* pos, void* out,
                                        int n_head, int n_kv_head, int head_dim, int n_ctx, float scale, void* stream) {
    if ((head_dim != 64 && head_dim != 128) || n_kv_head <= 0 || n_head % n_kv_head || n_head > ATT_MAX_HEADS ||
        n_ctx <= 0 || n_ctx % 8 || n_ctx > ATT_MAX_CTX || (reinterpret_cast<uintptr_t>(kc) & 15) ||
        (reinterpret_cast<uintptr_t>(vc) & 15))
        return (int)cudaErrorInvalidValue;
    // position ranges of at most ATT_CHUNK (a multiple of 8, so V^T runs stay 16-byte aligned)
    const int nsplit = (n_ctx + ATT_CHUNK - 1) / ATT_CHUNK;
    const int chunk = ((n_ctx + nsplit - 1) / nsplit + 7) / 8 * 8;
    CfiGlueSlot sl;
    const int rc = cfi_glue_slot(static_cast<cudaStream_t>(stream), &sl);
    if (rc) return rc;
    return launch(attention_q81, dim3(n_head, nsplit), 256, stream, q, (const __half*)kc, (const __half*)vc, pos,
                  (uint8_t*)out, n_head, n_kv_head, head_dim, n_ctx, scale, chunk, sl.att_part, sl.att_count);
}
extern "C" int cfi_fused_swiglu_q8_1(const float* gu, void* out, int n, void* stream) {
    if (n <= 0 || n % 32) return (int)cudaErrorInvalidValue;
    return launch(swiglu_q81, dim3((unsigned)((n / 32 + 7) / 8)), 256, stream, gu, (uint8_t*)out, n);
}
