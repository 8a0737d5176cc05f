// k_rowops.cu -- fp32 row kernels of the decode/prefill path (sm_100a): rms_norm (optionally
// fused with the weight multiply and an add), rope_neox and soft_max.
//
// Each kernel takes the parameter list of the ggml-cuda kernel it replaces, so the caller's
// kernelParams are forwarded unchanged (rope_neox gets one trailing word, the row count).  The
// arithmetic follows the published ggml definitions that the reference's GPU tests check against
// (cuda-for-intel tests/gpu/ggml_rms_norm.rs:43-55, tests/gpu/ggml_rope.rs:38-53,
// tests/gpu/soft_max_generic.rs:73-92); fp32 results agree with those host references to well
// inside 1e-3 relative L2 (rsqrtf/expf/sincosf are CUDA's, not bit-identical to libm).
#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "sm100_ptx.cuh"

namespace {

// Block-wide sum over CFI_ROWOP_THREADS threads (8 warps).
CFI_DEV float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();  // red may still be read by a previous reduction
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
    return warp_sum(t);
}
CFI_DEV float block_max(float v, float* red) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
    return warp_max(t);
}

// rms_norm_f32<block, do_multiply, do_add> of ggml-cuda (v0.12.6 parameter list):
// x, dst, int ncols, i64 stride_row/channel/sample, f32 eps, mul, i64 mul strides, uint3 packed
// mul ncols/nrows/nchannels/nsamples, add, i64 add strides, uint3 packed add dims.
// Grid (nrows, nchannels, nsamples); dst rows are contiguous.
template <int DO_MUL, int DO_ADD>
__global__ void __launch_bounds__(CFI_ROWOP_THREADS)
    cfi_rms_norm(const float* __restrict__ x, float* __restrict__ dst, int ncols, int64_t stride_row,
                 int64_t stride_channel, int64_t stride_sample, float eps, const float* __restrict__ mul,
                 int64_t mul_stride_row, int64_t mul_stride_channel, int64_t mul_stride_sample, uint3 mul_ncols,
                 uint3 mul_nrows, uint3 mul_nchannels, uint3 mul_nsamples, const float* __restrict__ add,
                 int64_t add_stride_row, int64_t add_stride_channel, int64_t add_stride_sample, uint3 add_ncols,
                 uint3 add_nrows, uint3 add_nchannels, uint3 add_nsamples) {
    __shared__ float red[32];
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const uint32_t row = blockIdx.x, channel = blockIdx.y, sample = blockIdx.z;
    const uint32_t nrows = gridDim.x, nchannels = gridDim.y;
    x += sample * stride_sample + channel * stride_channel + row * stride_row;
    dst += (((int64_t)sample * nchannels + channel) * nrows + row) * ncols;
    if (DO_MUL)
        mul += fastmodulo(sample, mul_nsamples) * mul_stride_sample + fastmodulo(channel, mul_nchannels) * mul_stride_channel +
               fastmodulo(row, mul_nrows) * mul_stride_row;
    if (DO_ADD)
        add += fastmodulo(sample, add_nsamples) * add_stride_sample + fastmodulo(channel, add_nchannels) * add_stride_channel +
               fastmodulo(row, add_nrows) * add_stride_row;
    float ss = 0.0f;
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) ss = __fmaf_rn(x[c], x[c], ss);
    ss = block_sum(ss, red);
    const float scale = rsqrtf(ss / (float)ncols + eps);
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) {
        float v = scale * x[c];
        if (DO_MUL) v = v * mul[fastmodulo((uint32_t)c, mul_ncols)];
        if (DO_ADD) v = v + add[fastmodulo((uint32_t)c, add_ncols)];
        dst[c] = v;
    }
}

// rms_norm_f32<32> with the (x, dst, int ncols, int nchannels, int nsamples, i64 stride_row,
// stride_channel, stride_sample, f32 eps) parameter list the reference's GPU test launches
// (tests/gpu/ggml_rms_norm.rs:63-80); grid x = rows.
__global__ void __launch_bounds__(CFI_ROWOP_THREADS)
    cfi_rms_norm_plain(const float* __restrict__ x, float* __restrict__ dst, int ncols, int nchannels, int nsamples,
                       int64_t stride_row, int64_t stride_channel, int64_t stride_sample, float eps) {
    __shared__ float red[32];
    (void)nsamples;
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const uint32_t row = blockIdx.x, channel = blockIdx.y, sample = blockIdx.z, nrows = gridDim.x;
    x += sample * stride_sample + channel * stride_channel + row * stride_row;
    dst += (((int64_t)sample * nchannels + channel) * nrows + row) * ncols;
    float ss = 0.0f;
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) ss = __fmaf_rn(x[c], x[c], ss);
    ss = block_sum(ss, red);
    const float scale = rsqrtf(ss / (float)ncols + eps);
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) dst[c] = scale * x[c];
}

struct rope_corr_dims {
    float v[2];
};

// rope_neox<forward, has_ff, float>: x, dst, int ne0, ne1, s1, s2, n_dims, const int* pos,
// f32 freq_scale, ext_factor, attn_factor, rope_corr_dims, f32 theta_scale, const f32*
// freq_factors, then the router's trailing u32 nrows.  One thread per (row, pair): pair p < n_dims/2
// rotates elements (p, p + n_dims/2) by pos*theta_scale^p (yarn ramp when ext_factor != 0);
// pairs at or past n_dims/2 copy elements 2p, 2p+1 unchanged.
template <int FORWARD, int HAS_FF>
__global__ void __launch_bounds__(CFI_ROWOP_THREADS)
    cfi_rope_neox(const float* __restrict__ x, float* __restrict__ dst, int ne0, int ne1, int s1, int s2, int n_dims,
                  const int32_t* __restrict__ pos, float freq_scale, float ext_factor, float attn_factor,
                  rope_corr_dims corr_dims, float theta_scale, const float* __restrict__ freq_factors,
                  uint32_t nrows) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const uint32_t half = (uint32_t)ne0 / 2;
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t row_dst = (uint32_t)(gid / half);
    if (row_dst >= nrows) return;
    const uint32_t p = (uint32_t)(gid - (uint64_t)row_dst * half);
    const int i0 = 2 * (int)p;
    const int row_x = (int)(row_dst % (uint32_t)ne1);
    const int channel_x = (int)(row_dst / (uint32_t)ne1);
    const int64_t idst = (int64_t)row_dst * ne0 + p;
    const int64_t ix = (int64_t)channel_x * s2 + (int64_t)row_x * s1 + p;
    if (i0 >= n_dims) {
        dst[idst + p + 0] = x[ix + p + 0];
        dst[idst + p + 1] = x[ix + p + 1];
        return;
    }
    const float theta_base = __fmul_rn((float)pos[channel_x], powf(theta_scale, (float)i0 / 2.0f));
    const float ff = HAS_FF ? freq_factors[p] : 1.0f;
    const float theta_extrap = theta_base / ff;
    float theta = freq_scale * theta_extrap;
    float mscale = attn_factor;
    if (ext_factor != 0.0f) {
        const float y = ((float)(i0 / 2) - corr_dims.v[0]) / fmaxf(0.001f, corr_dims.v[1] - corr_dims.v[0]);
        const float ramp_mix = (1.0f - fminf(1.0f, fmaxf(0.0f, y))) * ext_factor;
        theta = theta * (1.0f - ramp_mix) + theta_extrap * ramp_mix;
        mscale *= 1.0f + 0.1f * logf(1.0f / freq_scale);
    }
    float sn, cs;
    sincosf(theta, &sn, &cs);
    cs *= mscale;
    sn *= mscale;
    if (!FORWARD) sn = -sn;
    const float x0 = x[ix + 0], x1 = x[ix + n_dims / 2];
    // rounded products, then the sum (no fused multiply-add: the fused decode kernel matches it)
    dst[idst + 0] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
    dst[idst + n_dims / 2] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
}

// ggml's soft_max_params (128 bytes, tests/gpu/soft_max_generic.rs:10-31).
struct soft_max_params {
    int64_t nheads;
    uint32_t n_head_log2;
    uint32_t pad_;
    int64_t ncols, nrows_x, nrows_y, ne00, ne01, ne02, ne03, nb11, nb12, nb13, ne12, ne13;
    float scale, max_bias, m0, m1;
};
static_assert(sizeof(soft_max_params) == 128, "soft_max_params layout");

template <typename T> CFI_DEV float to_f32(T v);
template <> CFI_DEV float to_f32<float>(float v) { return v; }
template <> CFI_DEV float to_f32<__half>(__half v) { return __half2float(v); }

// soft_max_f32<*, *, *, T>: x, mask (T), sinks, dst, soft_max_params.  Grid (ne01, ne02, ne03);
// one CTA per row; the scaled, masked logits are kept in dynamic shared memory (ncols floats).
template <typename T>
__global__ void __launch_bounds__(CFI_ROWOP_THREADS)
    cfi_soft_max(const float* __restrict__ x, const T* __restrict__ mask, const float* __restrict__ sinks,
                 float* __restrict__ dst, const soft_max_params p) {
    extern __shared__ float vals[];
    __shared__ float red[32];
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int64_t i03 = blockIdx.z, i02 = blockIdx.y, i01 = blockIdx.x;
    const int64_t rowx = blockIdx.x + (int64_t)blockIdx.y * gridDim.x + (int64_t)blockIdx.z * gridDim.x * gridDim.y;
    const int64_t i11 = i01, i12 = i02 % p.ne12, i13 = i03 % p.ne13;
    x += rowx * p.ncols;
    dst += rowx * p.ncols;
    if (mask) mask += (i11 * p.nb11 + i12 * p.nb12 + i13 * p.nb13) / (int64_t)sizeof(T);
    float slope = 1.0f;
    if (p.max_bias > 0.0f) {
        const uint32_t h = (uint32_t)i02;
        const float base = h < p.n_head_log2 ? p.m0 : p.m1;
        const int exph = h < p.n_head_log2 ? (int)h + 1 : 2 * (int)(h - p.n_head_log2) + 1;
        slope = powf(base, (float)exph);
    }
    const int ncols = (int)p.ncols;
    float mx = -INFINITY;
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) {
        const float v = x[c] * p.scale + (mask ? slope * to_f32<T>(mask[c]) : 0.0f);
        vals[c] = v;
        mx = fmaxf(mx, v);
    }
    mx = block_max(mx, red);
    if (sinks) mx = fmaxf(mx, sinks[i02]);
    float s = 0.0f;
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) {
        const float e = expf(vals[c] - mx);
        vals[c] = e;
        s += e;
    }
    s = block_sum(s, red);
    if (sinks) s += expf(sinks[i02] - mx);
    const float inv = 1.0f / s;
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) dst[c] = vals[c] * inv;
}

}  // namespace

const void* cfi_native_rms_norm(int do_multiply, int do_add) {
    if (do_multiply && do_add) return reinterpret_cast<const void*>(&cfi_rms_norm<1, 1>);
    if (do_multiply) return reinterpret_cast<const void*>(&cfi_rms_norm<1, 0>);
    if (do_add) return reinterpret_cast<const void*>(&cfi_rms_norm<0, 1>);
    return reinterpret_cast<const void*>(&cfi_rms_norm<0, 0>);
}
const void* cfi_native_rms_norm_plain() { return reinterpret_cast<const void*>(&cfi_rms_norm_plain); }
const void* cfi_native_rope_neox(int forward, int has_ff) {
    if (forward) return has_ff ? reinterpret_cast<const void*>(&cfi_rope_neox<1, 1>) : reinterpret_cast<const void*>(&cfi_rope_neox<1, 0>);
    return has_ff ? reinterpret_cast<const void*>(&cfi_rope_neox<0, 1>) : reinterpret_cast<const void*>(&cfi_rope_neox<0, 0>);
}
const void* cfi_native_soft_max(int mask_f16) {
    return mask_f16 ? reinterpret_cast<const void*>(&cfi_soft_max<__half>) : reinterpret_cast<const void*>(&cfi_soft_max<float>);
}
