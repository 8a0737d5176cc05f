// q81_block.cuh -- one block_q8_1 {half d, half s, int8 qs[32]} from 32 fp32 values held by an
// 8-thread group, thread t of the group holding values 4t..4t+3.  Shared by the native
// quantize_q8_1 and by the GEMV that absorbs a deferred quantize_q8_1, so both produce the same
// bytes: d = amax/127 (IEEE divide), q = roundf(x/d) with x/d the IEEE quotient (0 when amax ==
// 0), s = the sum in the reference's 32-lane xor-butterfly order (cuda-for-intel
// src/subst/refs.rs:103-147).
#pragma once
#include "cfi_common.cuh"

// The 32-lane butterfly (offsets 16,8,4,2,1) of the reference, evaluated when thread t of an
// 8-thread group holds values 4t..4t+3: offsets 16/8/4 pair threads (xor 4/2/1), offsets 2/1 pair
// components inside a thread.  Returns lane 0's value of the 32-lane form on every thread.
CFI_DEV float butterfly32_from4(float4 v, unsigned mask) {
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
        v.x += __shfl_xor_sync(mask, v.x, o);
        v.y += __shfl_xor_sync(mask, v.y, o);
        v.z += __shfl_xor_sync(mask, v.z, o);
        v.w += __shfl_xor_sync(mask, v.w, o);
    }
    float t0 = __fadd_rn(v.x, v.z), t1 = __fadd_rn(v.y, v.w);
    return __fadd_rn(t0, t1);
}

CFI_DEV float amax8_from4(float4 v, unsigned mask) {
    float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(mask, a, o));
    return a;
}

// Loads values i0..i0+3 of `row` (zeros at and past ne00), vectorised when aligned.
CFI_DEV float4 q81_load4(const float* row, int64_t i0, int64_t ne00) {
    if (i0 + 3 < ne00 && ((reinterpret_cast<uintptr_t>(row + i0) & 15) == 0)) return *reinterpret_cast<const float4*>(row + i0);
    float4 v;
    v.x = i0 + 0 < ne00 ? row[i0 + 0] : 0.0f;
    v.y = i0 + 1 < ne00 ? row[i0 + 1] : 0.0f;
    v.z = i0 + 2 < ne00 ? row[i0 + 2] : 0.0f;
    v.w = i0 + 3 < ne00 ? row[i0 + 3] : 0.0f;
    return v;
}

// roundf(fl(x / d)) without the IEEE divide in the common case.  With |x| <= 127.01 d (x within
// the block whose amax gave d = fl(amax / 127)), qa = fl(x * rcp.approx(d)) differs from the
// correctly rounded quotient fl(x / d) by at most (1 ulp of rcp.approx (PTX ISA bound) + 0.5 ulp of
// the product + 0.5 ulp of fl(x / d)) x 127.01 < 3.1e-5.  So when qa is further than 1e-3 from
// every half-integer, no rounding boundary of roundf lies between qa and fl(x / d) and both round
// to the same integer; otherwise (and for d whose reciprocal is not a normal float) the quotient
// is taken with the IEEE divide.  The result is always the divide's.
CFI_DEV float q81_rcp_approx(float d) {
    float r;
    asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(d));
    return r;
}
CFI_DEV float q81_round_quot(float x, float d, float r, bool fast) {
    const float qa = __fmul_rn(x, r);
    const float a = fabsf(qa);
    if (fast && fabsf(a - floorf(a) - 0.5f) > 1e-3f) return roundf(qa);
    return roundf(__fdiv_rn(x, d));
}

struct Q81Part {
    char4 q;     // this thread's four quants
    uint32_t ds;  // half d | half s << 16 (the block header word)
    float d;
};

// The group's block from this thread's four values; `mask` covers the group's lanes.
CFI_DEV Q81Part q81_quantize4(float4 v, unsigned mask) {
    const float amax = amax8_from4(v, mask);
    const float sum = butterfly32_from4(v, mask);
    const float d = __fdiv_rn(amax, 127.0f);
    Q81Part p;
    if (amax == 0.0f) {
        p.q = make_char4(0, 0, 0, 0);
    } else {
        const bool fast = d >= 0x1p-120f && d <= 0x1p120f;  // 1/d normal, no overflow
        const float r = q81_rcp_approx(d);
        p.q.x = (int8_t)(int32_t)q81_round_quot(v.x, d, r, fast);
        p.q.y = (int8_t)(int32_t)q81_round_quot(v.y, d, r, fast);
        p.q.z = (int8_t)(int32_t)q81_round_quot(v.z, d, r, fast);
        p.q.w = (int8_t)(int32_t)q81_round_quot(v.w, d, r, fast);
    }
    p.ds = (uint32_t)f2h_bits(d) | ((uint32_t)f2h_bits(sum) << 16);
    p.d = d;
    return p;
}
