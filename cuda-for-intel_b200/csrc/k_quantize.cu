// k_quantize.cu -- activation quantizers of the substitution path (sm_100a).
//
// quantize_q8_1: fp32 rows -> block_q8_1 {half d, half s, int8 qs[32]}.  Same parameter list as
// ggml-cuda's `quantize_q8_1(const float*, void*, i64 ne00, s01, s02, s03, ne0, u32 ne1, uint3
// ne2)` (cuda-for-intel src/subst/quantize.rs:1-18), so the caller's kernelParams are forwarded
// unchanged.  Byte-exact to the reference (src/subst/refs.rs:117-147): d = amax/127 with an IEEE
// divide, q = roundf(x/d), and the float sum reproduces the 32-lane xor butterfly exactly even
// though each thread owns 4 consecutive values (see butterfly32_from4).
//
// quantize_mmq_q8_1: fp32 columns -> block_q8_1_mmq (144 B per 128 values), the input format of
// the prefill GEMM (refs.rs:742-769): d_inv = 127/amax, q = roundf(x*d_inv), d = 1/d_inv; layout
// D4 stores float d per 32 values, DS4 stores half2 {d, sum} with the sum taken as the sequential
// left fold of the 32 floats, as the reference does.
#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "sm100_ptx.cuh"
#include "q81_block.cuh"

// Native quantize_q8_1: 256 threads x 4 values = 1024 values of one row per CTA in x.
// Grid (ceil(ne0/1024), ne1, ne2*ne3); ne0 % 32 == 0 (ggml pads rows to 512).
extern "C" __global__ void __launch_bounds__(256)
    cfi_quantize_q8_1(const float* __restrict__ x, void* __restrict__ vy, int64_t ne00, int64_t s01, int64_t s02,
                      int64_t s03, int64_t ne0, uint32_t ne1, uint3 ne2) {
    // programmatic dependent launch: let the next kernel (a GEMV, which before its own wait only
    // prefetches its weights into L2) start at once, then wait for the producer of x
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int64_t i0 = ((int64_t)blockIdx.x * 256 + threadIdx.x) * 4;
    // whole 8-thread groups (32 values) leave together (ne0 is a multiple of 32); the shuffles
    // below stay inside a group, over the lanes that remain
    const unsigned mask = __ballot_sync(0xffffffffu, i0 < ne0);
    if (i0 >= ne0) return;
    const uint32_t bz = blockIdx.z;
    const uint32_t i3 = fastdiv(bz, ne2);
    const uint32_t i2 = bz - i3 * ne2.z;
    const int64_t i1 = blockIdx.y;
    const float* row = x + (int64_t)i3 * s03 + (int64_t)i2 * s02 + i1 * s01;
    const Q81Part p = q81_quantize4(q81_load4(row, i0, ne00), mask);
    const int64_t i_cont = (((int64_t)i3 * ne2.z + i2) * ne1 + i1) * ne0 + i0;
    uint8_t* blk = static_cast<uint8_t*>(vy) + (i_cont / QK8_1) * Q8_1_BYTES;
    const int iqs = (int)(i_cont % QK8_1);
    *reinterpret_cast<char4*>(blk + 4 + iqs) = p.q;
    if (iqs == 0) *reinterpret_cast<uint32_t*>(blk) = p.ds;
}

// Native quantize_mmq_q8_1<layout>: parameter list of ggml-cuda's quantize_mmq_q8_1 (x, ids, vy,
// i64 ne00, s01, s02, s03, ne0, int ne1, int ne2).  Grid (ne1, ceil(ne0/512), ne2*ne3), block 128:
// warp w of a CTA owns one 144-byte block (128 values) of column blockIdx.x; lane l holds values
// 4l..4l+3, so the 32-value group g lives on lanes 8g..8g+7.
template <int DS4>
__global__ void __launch_bounds__(128)
    cfi_quantize_mmq_q8_1(const float* __restrict__ x, const int32_t* __restrict__ ids, void* __restrict__ vy,
                          int64_t ne00, int64_t s01, int64_t s02, int64_t s03, int64_t ne0, int ne1, int ne2) {
    sm100::pdl_launch_dependents();
    sm100::pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t i0 = ((int64_t)blockIdx.y * 128 + threadIdx.x) * 4;
    if (i0 >= ne0) return;  // whole warps: ne0 % 128 == 0
    const int64_t i1 = blockIdx.x;
    const int64_t i2 = blockIdx.z % ne2;
    const int64_t i3 = blockIdx.z / ne2;
    const int64_t i01 = ids ? ids[i1] : i1;
    const float* row = x + i3 * s03 + i2 * s02 + i01 * s01;
    float4 v;
    if (i0 + 3 < ne00 && ((reinterpret_cast<uintptr_t>(row + i0) & 15) == 0)) {
        v = *reinterpret_cast<const float4*>(row + i0);
    } else {
        v.x = i0 + 0 < ne00 ? row[i0 + 0] : 0.0f;
        v.y = i0 + 1 < ne00 ? row[i0 + 1] : 0.0f;
        v.z = i0 + 2 < ne00 ? row[i0 + 2] : 0.0f;
        v.w = i0 + 3 < ne00 ? row[i0 + 3] : 0.0f;
    }
    const float amax = amax8_from4(v, 0xffffffffu);
    const float d_inv = __fdiv_rn(127.0f, amax);
    char4 q;
    float d;
    if (amax == 0.0f) {
        q = make_char4(0, 0, 0, 0);
        d = 0.0f;
    } else {
        q.x = (int8_t)(int32_t)roundf(__fmul_rn(v.x, d_inv));
        q.y = (int8_t)(int32_t)roundf(__fmul_rn(v.y, d_inv));
        q.z = (int8_t)(int32_t)roundf(__fmul_rn(v.z, d_inv));
        q.w = (int8_t)(int32_t)roundf(__fmul_rn(v.w, d_inv));
        d = __fdiv_rn(1.0f, d_inv);
    }
    const int64_t ib0 = (int64_t)blockIdx.z * ((int64_t)gridDim.x * gridDim.y * 4);  // blocks per channel
    const int64_t ib = ib0 + (i0 / 128) * ne1 + blockIdx.x;
    const int iqs = (int)(i0 % 128);
    uint8_t* blk = static_cast<uint8_t*>(vy) + ib * MMQ_BLOCK_BYTES;
    *reinterpret_cast<char4*>(blk + 16 + iqs) = q;
    float sum = 0.0f;
    if (DS4) {
        // sequential left fold 0 + v0 + v1 + ... + v31 of the group (all 8 lanes compute it)
        const int src0 = lane & ~7;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, v.x, src0 + j));
            sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, v.y, src0 + j));
            sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, v.z, src0 + j));
            sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, v.w, src0 + j));
        }
    }
    if ((iqs & 31) != 0) return;
    const int g = iqs / 32;
    if (DS4) {
        uint32_t ds = (uint32_t)f2h_bits(d) | ((uint32_t)f2h_bits(sum) << 16);
        reinterpret_cast<uint32_t*>(blk)[g] = ds;
    } else {
        reinterpret_cast<float*>(blk)[g] = d;
    }
}

const void* cfi_native_quantize_q8_1() { return reinterpret_cast<const void*>(&cfi_quantize_q8_1); }
const void* cfi_native_quantize_mmq(int ds4) {
    return ds4 ? reinterpret_cast<const void*>(&cfi_quantize_mmq_q8_1<1>)
               : reinterpret_cast<const void*>(&cfi_quantize_mmq_q8_1<0>);
}
