// decode_epi.cuh -- the fused decode steps as block-level device functions, shared by the
// standalone kernels of k_glue.cu and the GEMV epilogues of k_mmvq.cu (the last CTA of a GEMV
// runs one of them on the GEMV's output), so both forms compute the same bits.
#pragma once
#include <cuda_fp16.h>
#include <math.h>

#include "cfi_common.cuh"

// q8_1 block of 32 values, one value per lane (the reference's lane form: refs.rs:103-147):
// amax and sum by the xor butterfly 16..1, d = amax / 127, q = roundf(v / d).
CFI_DEV void q8_1_store_lane(float v, uint8_t* blk, int lane) {
    float a = fabsf(v), sm = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        sm += __shfl_xor_sync(0xffffffffu, sm, o);
    }
    const float d = __fdiv_rn(a, 127.0f);
    const int8_t q = a == 0.0f ? (int8_t)0 : (int8_t)(int32_t)roundf(__fdiv_rn(v, d));
    blk[4 + lane] = (uint8_t)q;
    if (lane == 0) *reinterpret_cast<uint32_t*>(blk) = (uint32_t)f2h_bits(d) | ((uint32_t)f2h_bits(sm) << 16);
}

// The sum-of-squares order of the warp-per-row rms_norm (vector path): lane l adds the squares of
// its 16-byte pieces l, l + 32, ... in order, four fma each, then the xor butterfly 16..1.
CFI_DEV float rms_fma4(float4 v, float ss) {
    ss = __fmaf_rn(v.x, v.x, ss);
    ss = __fmaf_rn(v.y, v.y, ss);
    ss = __fmaf_rn(v.z, v.z, ss);
    return __fmaf_rn(v.w, v.w, ss);
}

// x += y (y may be null), then q8_1 blocks of rms_norm(x) * w, by the whole block (>= 256
// threads, a multiple of 32).  The sum of squares is formed as the native rms_norm forms it for a
// decode step (cfi_rms_norm_block: 256 thread-strided fma chains, then the two-level butterfly),
// so the two agree bit for bit; hbuf: n floats of shared memory.
// y is read through L2 (it may have been written by other CTAs of this grid).
CFI_DEV void epi_add_rmsnorm_q81(float* __restrict__ x, const float* __restrict__ y, const float* __restrict__ w,
                                 uint8_t* __restrict__ out, int n, float eps, float* hbuf) {
    __shared__ float red[32];
    __shared__ float s_scale;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = blockDim.x;
    for (int c = tid; c < n; c += nt) {
        float v = x[c];
        if (y) {
            v += __ldcg(y + c);
            x[c] = v;
        }
        hbuf[c] = v;
    }
    __syncthreads();
    if (warp < 8) {
        float ss = 0.0f;
        for (int c = tid; c < n; c += 256) ss = __fmaf_rn(hbuf[c], hbuf[c], ss);
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
    }
    __syncthreads();
    if (warp == 0) {
        const float t = warp_sum(lane < 8 ? red[lane] : 0.0f);
        if (lane == 0) s_scale = rsqrtf(t / (float)n + eps);
    }
    __syncthreads();
    const float scale = s_scale;
    for (int c = tid; c < n; c += nt) {
        float v = scale * hbuf[c];
        v = v * w[c];
        q8_1_store_lane(v, out + (size_t)(c / 32) * Q8_1_BYTES, lane);
    }
}

// q8_1 blocks of silu(gu[i]) * gu[n + i]: warp `w0` of `nw` warps takes blocks w0, w0 + nw, ...
CFI_DEV void epi_swiglu_q81(const float* __restrict__ gu, uint8_t* __restrict__ out, int n, int w0, int nw) {
    const int lane = threadIdx.x & 31;
    for (int b = w0; b < n / 32; b += nw) {
        const int i = 32 * b + lane;
        const float a = __ldcg(gu + i);
        const float v = a / (1.0f + expf(-a)) * __ldcg(gu + n + i);
        q8_1_store_lane(v, out + (size_t)b * Q8_1_BYTES, lane);
    }
}

// qkv = [q | k | v]: + bias, NeoX rope on q (into q_out) and k, f16 K row / V column at pos[0] of
// the caches ([kv head][pos][dim], [kv head][dim][pos]).  Thread i0 of nt: items i0, i0 + nt, ...
// (one per rotation pair of q and k, then one per v value).
CFI_DEV void epi_qkv_rope_store(const float* __restrict__ qkv, const float* __restrict__ bias, float* __restrict__ q_out,
                                __half* __restrict__ kc, __half* __restrict__ vc, const int32_t* __restrict__ pos,
                                int nq, int nkv, int head_dim, int n_ctx, float theta_scale, int i0, int nt) {
    const int half = head_dim / 2, p = pos[0];
    const bool in_cache = p >= 0 && p < n_ctx;  // a position outside the cache stores nothing
    const int npairs = (nq + nkv) / 2;
    for (int i = i0; i < npairs + nkv; i += nt) {
        if (i < npairs) {
            const int head = i / half, j = i - head * half;
            const int base = head * head_dim;  // in [q | k]
            const float x0 = __ldcg(qkv + base + j) + bias[base + j];
            const float x1 = __ldcg(qkv + base + j + half) + bias[base + j + half];
            // rope_neox with freq_scale 1, no extrapolation, attn_factor 1: theta = pos * theta_scale^j
            const float theta = __fmul_rn((float)p, powf(theta_scale, (float)(2 * j) / 2.0f));
            float sn, cs;
            sincosf(theta, &sn, &cs);
            const float y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
            if (base < nq) {
                q_out[base + j] = y0;
                q_out[base + j + half] = y1;
            } else if (in_cache) {
                const int kh = (base - nq) / head_dim;
                __half* kr = kc + ((size_t)kh * n_ctx + p) * head_dim;
                kr[j] = __float2half_rn(y0);
                kr[j + half] = __float2half_rn(y1);
            }
        } else if (in_cache) {
            const int e = i - npairs, kh = e / head_dim, dd = e - kh * head_dim;
            const float v = __ldcg(qkv + nq + nkv + e) + bias[nq + nkv + e];
            vc[((size_t)kh * head_dim + dd) * n_ctx + p] = __float2half_rn(v);
        }
    }
}

// The fused step a GEMV's last CTA runs on the GEMV output y.
enum { EPI_ADD_RMSNORM_Q81 = 1, EPI_SWIGLU_Q81 = 2, EPI_QKV_ROPE_STORE = 3 };
struct DecodeEpi {
    float* x;              // add_rmsnorm: residual (x += y)
    const float* w;        // add_rmsnorm: norm weight
    uint8_t* q;            // q8_1 output (add_rmsnorm, swiglu)
    int n;                 // add_rmsnorm: length; swiglu: half the GEMV rows
    float eps;
    const float* bias;     // qkv: stacked biases
    float* q_out;
    __half* kc;
    __half* vc;
    const int32_t* pos;
    int nq, nkv, head_dim, n_ctx;
    float theta_scale;
    unsigned int* counter; // CTAs of the GEMV done (the last one runs the step and resets it)
};
