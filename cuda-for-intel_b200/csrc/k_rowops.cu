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
#include "decode_epi.cuh"

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
// mul ncols/nrows/nchannels/nsamples, add, i64 add strides, uint3 packed add dims; then the
// router's trailing u32 nrows.  One warp per row (8 rows per CTA), grid (ceil(nrows / 8),
// nchannels, nsamples), for launches of at least 1024 rows (cfi_rms_norm_block below takes the
// smaller ones); dst rows are contiguous.
//   * vector path (ncols % 4 == 0, x / dst / the row strides 16-byte aligned): lane l reads the
//     16-byte pieces l, l + 32, ... of its row, keeping up to 16 of them in registers for the
//     second pass; the sum of squares is the fma chain over the lane's pieces in order (4 values
//     each), then the xor butterfly 16..1 (rms_sumsq_vec4 in decode_epi.cuh, shared with the fused
//     decode step);
//   * otherwise lane l takes columns l, l + 32, ... one value at a time, in the same two passes.
template <int DO_MUL, int DO_ADD>
__global__ void __launch_bounds__(CFI_ROWOP_THREADS)
    cfi_rms_norm(const float* __restrict__ x, float* __restrict__ dst, int ncols, int64_t stride_row,
                 int64_t stride_channel, int64_t stride_sample, float eps, const float* __restrict__ mul,
                 int64_t mul_stride_row, int64_t mul_stride_channel, int64_t mul_stride_sample, uint3 mul_ncols,
                 uint3 mul_nrows, uint3 mul_nchannels, uint3 mul_nsamples, const float* __restrict__ add,
                 int64_t add_stride_row, int64_t add_stride_channel, int64_t add_stride_sample, uint3 add_ncols,
                 uint3 add_nrows, uint3 add_nchannels, uint3 add_nsamples, uint32_t nrows) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const uint32_t lane = threadIdx.x & 31, row = blockIdx.x * (CFI_ROWOP_THREADS / 32) + (threadIdx.x >> 5);
    const uint32_t channel = blockIdx.y, sample = blockIdx.z, nchannels = gridDim.y;
    if (row >= nrows) return;
    x += sample * stride_sample + channel * stride_channel + row * stride_row;
    dst += (((int64_t)sample * nchannels + channel) * nrows + row) * ncols;
    if (DO_MUL)
        mul += fastmodulo(sample, mul_nsamples) * mul_stride_sample + fastmodulo(channel, mul_nchannels) * mul_stride_channel +
               fastmodulo(row, mul_nrows) * mul_stride_row;
    if (DO_ADD)
        add += fastmodulo(sample, add_nsamples) * add_stride_sample + fastmodulo(channel, add_nchannels) * add_stride_channel +
               fastmodulo(row, add_nrows) * add_stride_row;
    const bool vec = (ncols & 3) == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
    if (vec) {
        constexpr int KEEP = 16;
        const int n4 = ncols / 4;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        float4 r[KEEP];
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < KEEP; i++)
            if ((int)lane + 32 * i < n4) r[i] = __ldg(x4 + lane + 32 * i);
#pragma unroll
        for (int i = 0; i < KEEP; i++)
            if ((int)lane + 32 * i < n4) ss = rms_fma4(r[i], ss);
        for (int i = KEEP; (int)lane + 32 * i < n4; i++) ss = rms_fma4(__ldg(x4 + lane + 32 * i), ss);
        ss = warp_sum(ss);
        const float scale = rsqrtf(ss / (float)ncols + eps);
        const bool wvec = (!DO_MUL || (mul_ncols.z == (uint32_t)ncols && (reinterpret_cast<uintptr_t>(mul) & 15) == 0)) &&
                          (!DO_ADD || (add_ncols.z == (uint32_t)ncols && (reinterpret_cast<uintptr_t>(add) & 15) == 0));
        float4* d4 = reinterpret_cast<float4*>(dst);
        auto emit = [&](int i, float4 v) {
            const int c = 4 * ((int)lane + 32 * i);
            float e[4] = {scale * v.x, scale * v.y, scale * v.z, scale * v.w};
            if (DO_MUL) {
                if (wvec) {
                    const float4 m = __ldg(reinterpret_cast<const float4*>(mul) + lane + 32 * i);
                    e[0] = e[0] * m.x, e[1] = e[1] * m.y, e[2] = e[2] * m.z, e[3] = e[3] * m.w;
                } else {
#pragma unroll
                    for (int k = 0; k < 4; k++) e[k] = e[k] * mul[fastmodulo((uint32_t)(c + k), mul_ncols)];
                }
            }
            if (DO_ADD) {
                if (wvec) {
                    const float4 a = __ldg(reinterpret_cast<const float4*>(add) + lane + 32 * i);
                    e[0] = e[0] + a.x, e[1] = e[1] + a.y, e[2] = e[2] + a.z, e[3] = e[3] + a.w;
                } else {
#pragma unroll
                    for (int k = 0; k < 4; k++) e[k] = e[k] + add[fastmodulo((uint32_t)(c + k), add_ncols)];
                }
            }
            d4[lane + 32 * i] = make_float4(e[0], e[1], e[2], e[3]);
        };
#pragma unroll
        for (int i = 0; i < KEEP; i++)
            if ((int)lane + 32 * i < n4) emit(i, r[i]);
        for (int i = KEEP; (int)lane + 32 * i < n4; i++) emit(i, __ldg(x4 + lane + 32 * i));
        return;
    }
    float ss = 0.0f;
    for (int c = lane; c < ncols; c += 32) ss = __fmaf_rn(x[c], x[c], ss);
    ss = warp_sum(ss);
    const float scale = rsqrtf(ss / (float)ncols + eps);
    for (int c = lane; c < ncols; c += 32) {
        float v = scale * x[c];
        if (DO_MUL) v = v * mul[fastmodulo((uint32_t)c, mul_ncols)];
        if (DO_ADD) v = v + add[fastmodulo((uint32_t)c, add_ncols)];
        dst[c] = v;
    }
}

// The same rms_norm_f32 with one CTA per row, for launches of few rows (a decode step: the
// shorter chain over 256 threads): grid (nrows, nchannels, nsamples).  Sum of squares: 256
// thread-strided fma chains, then the two-level butterfly (block_sum) -- the order the fused
// add + rms_norm + quantize step of the decode driver reproduces.
template <int DO_MUL, int DO_ADD>
__global__ void __launch_bounds__(CFI_ROWOP_THREADS)
    cfi_rms_norm_block(const float* __restrict__ x, float* __restrict__ dst, int ncols, int64_t stride_row,
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
// freq_factors, then the router's trailing u32 nrows and rows per warp.  Pair p < n_dims/2 of a
// row rotates elements (p, p + n_dims/2) by pos*theta_scale^p (yarn ramp when ext_factor != 0);
// pairs at or past n_dims/2 copy elements 2p, 2p+1 unchanged.  One warp per `rpw` consecutive
// rows, lane l taking pairs l, l + 32, ...: the loads of all the warp's rows are issued first, and
// theta_scale^p (powf) is formed once per pair for the warp's rows.  The router gives
// large launches ROPE_ROWS rows per warp; small ones (a decode step's heads) take
// cfi_rope_neox_pairs below, one thread per pair.
constexpr int ROPE_ROWS = 4;      // rows per warp of a large launch
constexpr int ROPE_MAXP = 4;      // pairs per lane kept in registers (ne0 <= 256)

template <int FORWARD, int HAS_FF>
__global__ void __launch_bounds__(CFI_ROWOP_THREADS)
    cfi_rope_neox(const float* __restrict__ x, float* __restrict__ dst, int ne0, int ne1, int s1, int s2, int n_dims,
                  const int32_t* __restrict__ pos, float freq_scale, float ext_factor, float attn_factor,
                  rope_corr_dims corr_dims, float theta_scale, const float* __restrict__ freq_factors,
                  uint32_t nrows, uint32_t /*rows per warp: ROPE_ROWS*/) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int lane = threadIdx.x & 31;
    const uint32_t row0 = (blockIdx.x * (CFI_ROWOP_THREADS / 32) + (threadIdx.x >> 5)) * ROPE_ROWS;
    const int half = ne0 / 2, nd2 = n_dims / 2;
    // every load of the warp's rows first (positions, then both elements of each pair), then the math
    float fpos[ROPE_ROWS];
    const float* xr[ROPE_ROWS];
    float* dr[ROPE_ROWS];
    bool live[ROPE_ROWS];
#pragma unroll
    for (int rr = 0; rr < ROPE_ROWS; rr++) {
        const uint32_t row_dst = row0 + rr;
        live[rr] = row_dst < nrows;
        const uint32_t rd = live[rr] ? row_dst : 0u;
        const int row_x = (int)(rd % (uint32_t)ne1), channel_x = (int)(rd / (uint32_t)ne1);
        fpos[rr] = (float)pos[channel_x];
        xr[rr] = x + (int64_t)channel_x * s2 + (int64_t)row_x * s1;
        dr[rr] = dst + (int64_t)rd * ne0;
    }
#pragma unroll
    for (int k = 0; k < ROPE_MAXP; k++) {
        const int p = lane + 32 * k;
        const int i0 = 2 * p;
        if (p >= half) continue;
        if (i0 >= n_dims) {
#pragma unroll
            for (int rr = 0; rr < ROPE_ROWS; rr++)
                if (live[rr]) {
                    dr[rr][2 * p] = xr[rr][2 * p];
                    dr[rr][2 * p + 1] = xr[rr][2 * p + 1];
                }
            continue;
        }
        float x0[ROPE_ROWS], x1[ROPE_ROWS];
#pragma unroll
        for (int rr = 0; rr < ROPE_ROWS; rr++) {
            x0[rr] = live[rr] ? xr[rr][p] : 0.0f;
            x1[rr] = live[rr] ? xr[rr][p + nd2] : 0.0f;
        }
        const float tp = powf(theta_scale, (float)i0 / 2.0f);
        const float ff = HAS_FF ? freq_factors[p] : 1.0f;
#pragma unroll
        for (int rr = 0; rr < ROPE_ROWS; rr++) {
            const float theta_base = __fmul_rn(fpos[rr], tp);
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
            // rounded products, then the sum (no fused multiply-add: the fused decode kernel matches it)
            if (live[rr]) {
                dr[rr][p] = __fsub_rn(__fmul_rn(x0[rr], cs), __fmul_rn(x1[rr], sn));
                dr[rr][p + nd2] = __fadd_rn(__fmul_rn(x0[rr], sn), __fmul_rn(x1[rr], cs));
            }
        }
    }
}

// rope_neox<forward, has_ff, float>: x, dst, int ne0, ne1, s1, s2, n_dims, const int* pos,
// f32 freq_scale, ext_factor, attn_factor, rope_corr_dims, f32 theta_scale, const f32*
// freq_factors, then the router's trailing u32 nrows.  The thread-per-(row, pair) form, for
// launches of few rows (a decode step's heads), with the arithmetic of cfi_rope_neox above.
template <int FORWARD, int HAS_FF>
__global__ void __launch_bounds__(CFI_ROWOP_THREADS)
    cfi_rope_neox_pairs(const float* __restrict__ x, float* __restrict__ dst, int ne0, int ne1, int s1, int s2, int n_dims,
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

// soft_max_f32 as above, one warp per row (8 rows per CTA; grid (ceil(ne01 / 8), ne02, ne03)) for
// rows of at most SMW_MAX columns with ncols % 4 == 0 and 16-byte aligned x / dst / mask rows (8-byte
// for an f16 mask): lane l keeps its 16-byte pieces l, l + 32, ... of the scaled, masked row in
// registers; row max and sum by the xor butterfly; trailing u32: ne01.
constexpr int SMW_KEEP = 8;                  // 16-byte pieces per lane
constexpr int SMW_MAX = 4 * 32 * SMW_KEEP;  // 1024 columns

template <typename T> CFI_DEV float4 mask4(const T* m, int i);
template <> CFI_DEV float4 mask4<float>(const float* m, int i) { return __ldg(reinterpret_cast<const float4*>(m) + i); }
template <> CFI_DEV float4 mask4<__half>(const __half* m, int i) {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(m) + i);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x)), b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

template <typename T>
__global__ void __launch_bounds__(CFI_ROWOP_THREADS)
    cfi_soft_max_rows(const float* __restrict__ x, const T* __restrict__ mask, const float* __restrict__ sinks,
                      float* __restrict__ dst, const soft_max_params p, uint32_t ne01) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t i01 = (int64_t)blockIdx.x * (CFI_ROWOP_THREADS / 32) + (threadIdx.x >> 5);
    if (i01 >= (int64_t)ne01) return;
    const int64_t i03 = blockIdx.z, i02 = blockIdx.y;
    const int64_t rowx = i01 + i02 * (int64_t)ne01 + i03 * (int64_t)ne01 * gridDim.y;
    const int64_t i12 = i02 % p.ne12, i13 = i03 % p.ne13;
    x += rowx * p.ncols;
    dst += rowx * p.ncols;
    if (mask) mask += (i01 * p.nb11 + i12 * p.nb12 + i13 * p.nb13) / (int64_t)sizeof(T);
    float slope = 1.0f;
    if (p.max_bias > 0.0f) {
        const uint32_t h = (uint32_t)i02;
        const float base = h < p.n_head_log2 ? p.m0 : p.m1;
        const int exph = h < p.n_head_log2 ? (int)h + 1 : 2 * (int)(h - p.n_head_log2) + 1;
        slope = powf(base, (float)exph);
    }
    const int n4 = (int)p.ncols / 4;
    float4 v[SMW_KEEP];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < SMW_KEEP; i++) {
        const int j = lane + 32 * i;
        if (j < n4) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(x) + j);
            float4 e = make_float4(a.x * p.scale, a.y * p.scale, a.z * p.scale, a.w * p.scale);
            if (mask) {
                const float4 m = mask4<T>(mask, j);
                e.x += slope * m.x, e.y += slope * m.y, e.z += slope * m.z, e.w += slope * m.w;
            }
            v[i] = e;
            mx = fmaxf(mx, fmaxf(fmaxf(e.x, e.y), fmaxf(e.z, e.w)));
        }
    }
    mx = warp_max(mx);
    if (sinks) mx = fmaxf(mx, sinks[i02]);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < SMW_KEEP; i++) {
        if (lane + 32 * i < n4) {
            v[i] = make_float4(expf(v[i].x - mx), expf(v[i].y - mx), expf(v[i].z - mx), expf(v[i].w - mx));
            s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        }
    }
    s = warp_sum(s);
    if (sinks) s += expf(sinks[i02] - mx);
    const float inv = 1.0f / s;
#pragma unroll
    for (int i = 0; i < SMW_KEEP; i++)
        if (lane + 32 * i < n4)
            reinterpret_cast<float4*>(dst)[lane + 32 * i] = make_float4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv);
}

}  // namespace

const void* cfi_native_rms_norm(int do_multiply, int do_add) {
    if (do_multiply && do_add) return reinterpret_cast<const void*>(&cfi_rms_norm<1, 1>);
    if (do_multiply) return reinterpret_cast<const void*>(&cfi_rms_norm<1, 0>);
    if (do_add) return reinterpret_cast<const void*>(&cfi_rms_norm<0, 1>);
    return reinterpret_cast<const void*>(&cfi_rms_norm<0, 0>);
}
const void* cfi_native_rms_norm_block(int do_multiply, int do_add) {
    if (do_multiply && do_add) return reinterpret_cast<const void*>(&cfi_rms_norm_block<1, 1>);
    if (do_multiply) return reinterpret_cast<const void*>(&cfi_rms_norm_block<1, 0>);
    if (do_add) return reinterpret_cast<const void*>(&cfi_rms_norm_block<0, 1>);
    return reinterpret_cast<const void*>(&cfi_rms_norm_block<0, 0>);
}
const void* cfi_native_rms_norm_plain() { return reinterpret_cast<const void*>(&cfi_rms_norm_plain); }
const void* cfi_native_rope_neox(int forward, int has_ff) {
    if (forward) return has_ff ? reinterpret_cast<const void*>(&cfi_rope_neox<1, 1>) : reinterpret_cast<const void*>(&cfi_rope_neox<1, 0>);
    return has_ff ? reinterpret_cast<const void*>(&cfi_rope_neox<0, 1>) : reinterpret_cast<const void*>(&cfi_rope_neox<0, 0>);
}
const void* cfi_native_soft_max(int mask_f16) {
    return mask_f16 ? reinterpret_cast<const void*>(&cfi_soft_max<__half>) : reinterpret_cast<const void*>(&cfi_soft_max<float>);
}
const void* cfi_native_soft_max_rows(int mask_f16) {
    return mask_f16 ? reinterpret_cast<const void*>(&cfi_soft_max_rows<__half>)
                    : reinterpret_cast<const void*>(&cfi_soft_max_rows<float>);
}
int cfi_soft_max_rows_max_cols() { return SMW_MAX; }
const void* cfi_native_rope_neox_pairs(int forward, int has_ff) {
    if (forward)
        return has_ff ? reinterpret_cast<const void*>(&cfi_rope_neox_pairs<1, 1>) : reinterpret_cast<const void*>(&cfi_rope_neox_pairs<1, 0>);
    return has_ff ? reinterpret_cast<const void*>(&cfi_rope_neox_pairs<0, 1>) : reinterpret_cast<const void*>(&cfi_rope_neox_pairs<0, 0>);
}
int cfi_rope_rows_per_warp(uint32_t nrows) {
    // four rows per warp once a launch has that many per warp of a full GPU (8 warps x 148 SMs)
    return nrows >= (uint32_t)(ROPE_ROWS * (CFI_ROWOP_THREADS / 32) * 148) ? ROPE_ROWS : 1;
}
int cfi_rope_max_ne0() { return 2 * 32 * ROPE_MAXP; }
