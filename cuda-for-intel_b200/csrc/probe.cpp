// probe.cpp -- first-use validation of a native kernel on the device (cuda-for-intel
// src/subst/probe.rs:1-403, re-designed for CUDA).
//
// Before a plan's native kernel serves a caller, it runs once on a small deterministic problem
// (the reference's probe cases and seeds) and its output is compared with a host evaluation of
// the same ggml block math: quantizers byte for byte, float kernels by nmse (below 1e-9 where the
// arithmetic is the reference's, 1e-6 where the B200 kernel legitimately rounds differently:
// the fp16-dequantising tensor-core mmq and CUDA's powf/sincosf in rope).  A failed probe marks
// the plan failed and the caller's stock kernel runs.  The host evaluation below exists only to
// accept or reject a kernel; it never produces results for a caller.
#include <cuda_runtime.h>
#include <math.h>
#include <algorithm>
#include <string.h>

#include <vector>

#include "cfi_kernels.h"
#include "subst_host.hpp"

namespace cfi {

int issue_native(const NativeLaunch& nl, const cfi_plan& plan, void** args, void* stream);

namespace {

// ---- deterministic data (refs.rs:499-538) ----
struct Rng {
    uint64_t s;
    uint64_t next() {
        s ^= s >> 12;
        s ^= s << 25;
        s ^= s >> 27;
        return s * 0x2545F4914F6CDD1Dull;
    }
    uint32_t u32() { return (uint32_t)(next() >> 32); }
    float unit() { return (float)(u32() >> 8) / (float)(1u << 24) * 2.0f - 1.0f; }
};

float h2f(uint16_t h) {
    uint32_t s = h >> 15, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    float mag = e == 0 ? ldexpf((float)m, -24) : (e == 31 ? (m ? NAN : INFINITY) : ldexpf((float)(m | 0x400), (int)e - 25));
    return s ? -mag : mag;
}
uint16_t f2h(float x) {  // round to nearest even
    uint32_t b;
    memcpy(&b, &x, 4);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000);
    int32_t exp = (int32_t)((b >> 23) & 0xff) - 127 + 15;
    uint32_t man = b & 0x7fffff;
    if (((b >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00 | (man ? 0x200 : 0));
    if (exp >= 31) return (uint16_t)(sign | 0x7c00);
    if (exp <= 0) {
        if (exp < -10) return sign;
        uint32_t mant = man | 0x800000, sh = (uint32_t)(14 - exp);
        uint32_t h = mant >> sh, rem = mant & ((1u << sh) - 1), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (h & 1))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)exp << 10) | (man >> 13), rem = man & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return (uint16_t)(sign | h);
}
uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
void wr16(uint8_t* p, uint16_t v) {
    p[0] = (uint8_t)v;
    p[1] = (uint8_t)(v >> 8);
}

size_t block_bytes(uint32_t ty) { return ty == 8 ? 34 : ty == 12 ? 144 : ty == 2 ? 18 : ty == 14 ? 210 : ty == 6 ? 22 : 176; }

std::vector<uint8_t> random_blocks(uint32_t ty, size_t n, Rng& rng) {
    size_t bb = block_bytes(ty);
    std::vector<uint8_t> out(n * bb);
    for (size_t b = 0; b < n; b++) {
        uint8_t* blk = out.data() + b * bb;
        for (size_t i = 0; i < bb; i++) blk[i] = (uint8_t)rng.u32();
        if (ty == 2 || ty == 6 || ty == 8) wr16(blk, f2h(rng.unit() * 0.05f));
        if (ty == 12 || ty == 13) {
            wr16(blk, f2h(rng.unit() * 0.05f));
            wr16(blk + 2, f2h(rng.unit() * 0.05f));
        }
        if (ty == 14) wr16(blk + 208, f2h(rng.unit() * 0.05f));
    }
    return out;
}

int dp4a(uint32_t a, uint32_t b, int c) {
    for (int k = 0; k < 4; k++) c += (int)(int8_t)(a >> (8 * k)) * (int)(int8_t)(b >> (8 * k));
    return c;
}

// block_q8_1 of 32 floats: xor-butterfly sum and max, d = amax/127, q = round(x/d).
void quantize_q8_1(const float* x, size_t n, uint8_t* out) {
    for (size_t ib = 0; ib < n / 32; ib++) {
        float s[32], a[32];
        for (int l = 0; l < 32; l++) s[l] = x[ib * 32 + l], a[l] = fabsf(x[ib * 32 + l]);
        for (int o = 16; o; o >>= 1) {
            float s2[32], a2[32];
            for (int l = 0; l < 32; l++) s2[l] = s[l] + s[l ^ o], a2[l] = fmaxf(a[l], a[l ^ o]);
            memcpy(s, s2, sizeof s);
            memcpy(a, a2, sizeof a);
        }
        float d = a[0] / 127.0f;
        uint8_t* o = out + ib * 36;
        wr16(o, f2h(d));
        wr16(o + 2, f2h(s[0]));
        for (int l = 0; l < 32; l++) o[4 + l] = (uint8_t)(int8_t)(a[0] == 0.0f ? 0 : (int)roundf(x[ib * 32 + l] / d));
    }
}

// One 32-value group of a weight row against its q8_1 block, whole-group lane form.
float lane_dot(uint32_t ty, const uint8_t* xb, const uint8_t* yb, int g, float acc) {
    float d8 = h2f(rd16(yb));
    if (ty == 8) {
        int s = 0;
        for (int i = 0; i < 8; i++) s = dp4a(rd32(xb + 2 + 4 * i), rd32(yb + 4 + 4 * i), s);
        return fmaf(h2f(rd16(xb)) * d8, (float)s, acc);
    }
    const uint8_t* sc = xb + 4;
    int scv, mv;
    if (g < 4) {
        scv = sc[g] & 63;
        mv = sc[g + 4] & 63;
    } else {
        scv = (sc[g + 4] & 0xF) | ((sc[g - 4] >> 6) << 4);
        mv = (sc[g + 4] >> 4) | ((sc[g] >> 6) << 4);
    }
    int si = 0, sy = 0;
    for (int i = 0; i < 8; i++) {
        uint32_t v = (rd32(xb + 16 + 32 * (g / 2) + 4 * i) >> (4 * (g & 1))) & 0x0F0F0F0F;
        si = dp4a(v, rd32(yb + 4 + 4 * i), si);
        sy = dp4a(0x01010101, rd32(yb + 4 + 4 * i), sy);
    }
    float a = d8 * (float)(si * scv), b = d8 * (float)(sy * mv);
    float t1 = h2f(rd16(xb)) * a, t2 = h2f(rd16(xb + 2)) * b;
    return acc + (t1 - t2);
}

// Q6_K group g of a superblock, whole-group lane form (refs.rs:414-430).
float lane_dot_q6k(const uint8_t* xb, const uint8_t* yb, int g, float acc) {
    const float d8 = h2f(rd16(yb));
    const int h = g / 4, sub = g % 4;
    int tot = 0;
    for (int half = 0; half < 2; half++) {
        int si = 0, su = 0;
        for (int i = 4 * half; i < 4 * half + 4; i++) {
            const uint32_t lo = (rd32(xb + 64 * h + 32 * (sub & 1) + 4 * i) >> (4 * (sub >> 1))) & 0x0F0F0F0F;
            const uint32_t hi = ((rd32(xb + 128 + 32 * h + 4 * i) >> (2 * sub)) & 0x03030303) << 4;
            si = dp4a(lo | hi, rd32(yb + 4 + 4 * i), si);
            su = dp4a(0x01010101, rd32(yb + 4 + 4 * i), su);
        }
        tot += (si - (su << 5)) * (int)(int8_t)xb[192 + 8 * h + 2 * sub + half];
    }
    return fmaf(h2f(rd16(xb + 208)) * d8, (float)tot, acc);
}

// Q4_0 half block kqs (words kqs, kqs+1 of the 16 quant bytes; refs.rs:166-259).
float lane_dot_q40(const uint8_t* xb, const uint8_t* yb, int kqs, float acc) {
    int sumi = 0;
    for (int i = 0; i < 2; i++) {
        const uint32_t v = rd32(xb + 2 + 4 * (kqs + i));
        sumi = dp4a(v & 0x0F0F0F0F, rd32(yb + 4 + 4 * (kqs + i)), sumi);
        sumi = dp4a((v >> 4) & 0x0F0F0F0F, rd32(yb + 4 + 4 * (kqs + i + 4)), sumi);
    }
    const float inner = fmaf(h2f(rd16(yb)), (float)sumi, h2f(rd16(yb + 2)) * -4.0f);
    return fmaf(h2f(rd16(xb)), inner, acc);
}

float row_dot(uint32_t ty, const uint8_t* row, uint32_t ncols_x, const uint8_t* ycol) {
    const uint32_t qk = (ty == 12 || ty == 14) ? 256 : 32, nb = ncols_x / qk;
    // threads per block: whole 32-value groups (Q8_0, Q4_K, Q6_K), half blocks (Q4_0)
    const uint32_t tpb = ty == 2 ? 2 : qk / 32, step = 32 / tpb;
    float lanes[32];
    for (uint32_t l = 0; l < 32; l++) {
        float acc = 0.0f;
        for (uint32_t k = l / tpb; k < nb; k += step) {
            const uint8_t* xb = row + k * block_bytes(ty);
            if (ty == 2)
                acc = lane_dot_q40(xb, ycol + k * 36, 2 * (int)(l % 2), acc);
            else if (ty == 14)
                acc = lane_dot_q6k(xb, ycol + (k * tpb + l % tpb) * 36, (int)(l % tpb), acc);
            else
                acc = lane_dot(ty, xb, ycol + (k * tpb + l % tpb) * 36, (int)(l % tpb), acc);
        }
        lanes[l] = acc;
    }
    for (int o = 16; o; o >>= 1) {
        float t[32];
        for (int l = 0; l < 32; l++) t[l] = lanes[l] + lanes[l ^ o];
        memcpy(lanes, t, sizeof t);
    }
    return lanes[0];
}

double nmse(const std::vector<float>& got, const std::vector<float>& want) {
    double num = 0, den = 0;
    for (size_t i = 0; i < want.size(); i++) {
        double d = (double)got[i] - (double)want[i];
        num += d * d;
        den += (double)want[i] * want[i];
    }
    return den == 0 ? num : num / den;
}

// ---- device scratch for a probe ----
struct Dev {
    std::vector<void*> bufs;
    ~Dev() {
        for (void* p : bufs) cudaFree(p);
    }
    // a failing call leaves its error for cudaGetLastError (read by CK)
    void* put(const void* src, size_t n) {
        void* p = nullptr;
        if (cudaMalloc(&p, n ? n : 16) != cudaSuccess) return nullptr;
        bufs.push_back(p);
        if (src && n && cudaMemcpy(p, src, n, cudaMemcpyHostToDevice) != cudaSuccess) return nullptr;
        if (!src && n && cudaMemset(p, 0, n) != cudaSuccess) return nullptr;
        return p;
    }
};


// Kernel parameter storage: one 16-byte-aligned slot per parameter.
struct Args {
    std::vector<uint64_t> store;
    std::vector<void*> ptrs;
    explicit Args(size_t n) : store(n * 16, 0) {}
    void set(size_t i, const void* v, size_t bytes) {
        memcpy(&store[i * 16], v, bytes);
        if (ptrs.size() <= i) ptrs.resize(i + 1);
        ptrs[i] = &store[i * 16];
    }
    void ptr(size_t i, const void* p) { set(i, &p, 8); }
    void u32(size_t i, uint32_t v) { set(i, &v, 4); }
    void u64(size_t i, uint64_t v) { set(i, &v, 8); }
    void f32(size_t i, float v) { set(i, &v, 4); }
    void u3(size_t i, uint32_t a, uint32_t b, uint32_t c) {
        uint32_t t[3] = {a, b, c};
        set(i, t, 12);
    }
    void** data() { return ptrs.data(); }
};

void fastdiv_values(uint32_t d, uint32_t v[3]) {
    uint32_t l = 0;
    while (l < 32 && (1ull << l) < d) l++;
    v[0] = (uint32_t)((((1ull << 32) * ((1ull << l) - d)) / d) + 1);
    v[1] = l;
    v[2] = d;
}

int run(const cfi_plan& plan, const uint32_t grid[3], const uint32_t block[3], Args& a, void* stream, std::string* why) {
    std::vector<uint64_t> vals = arg_values(plan, a.data());
    NativeLaunch nl;
    if (!map_launch(plan, grid, block, vals.data(), (int)vals.size(), a.data(), &nl)) {
        *why = "probe geometry rejected";
        return (int)cudaErrorInvalidConfiguration;
    }
    int rc = issue_native(nl, plan, a.data(), stream);
    if (!rc) rc = (int)cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (rc) *why = std::string("probe launch: ") + cudaGetErrorString((cudaError_t)rc);
    return rc;
}

// A failed allocation or copy is reported with the CUDA error of the call that failed.
#define CK(x)                                                                                   \
    do {                                                                                        \
        if (!(x)) {                                                                             \
            const cudaError_t e_ = cudaGetLastError();                                          \
            *why = std::string("probe allocation/copy failed: ") + cudaGetErrorString(e_);      \
            return (int)(e_ != cudaSuccess ? e_ : cudaErrorMemoryAllocation);                   \
        }                                                                                       \
    } while (0)

// probe.rs:353-368 (one channel, one sample, no ids)
int probe_mmvq(const cfi_plan& plan, void* stream, std::string* why) {
    const uint32_t ty = plan.ty, nc = plan.ncols, nrows = plan.has_fast ? 11 : 5, ncols_x = 512;
    if (ty != 8 && ty != 12 && ty != 14 && ty != 2) {
        *why = "no host check for this type";
        return (int)cudaErrorNotSupported;
    }
    Rng rng{0x5eed + ty};
    const uint32_t qk = (ty == 12 || ty == 14) ? 256 : 32, bpr = ncols_x / qk, ystride = ncols_x / 32;
    std::vector<uint8_t> x = random_blocks(ty, (size_t)nrows * bpr, rng);
    std::vector<float> acts((size_t)ncols_x * nc);
    for (auto& v : acts) v = rng.unit() * 3.0f;
    std::vector<uint8_t> y(acts.size() / 32 * 36);
    quantize_q8_1(acts.data(), acts.size(), y.data());
    std::vector<float> want((size_t)nrows * nc), got(want.size());
    for (uint32_t c = 0; c < nc; c++)
        for (uint32_t r = 0; r < nrows; r++)
            want[(size_t)c * nrows + r] = row_dot(ty, x.data() + (size_t)r * bpr * block_bytes(ty), ncols_x, y.data() + (size_t)c * ystride * 36);
    Dev d;
    void* dx = d.put(x.data(), x.size());
    void* dy = d.put(y.data(), y.size());
    void* dd = d.put(nullptr, want.size() * 4);
    CK(dx && dy && dd);
    uint32_t chr[3], smr[3];
    fastdiv_values(1, chr);
    fastdiv_values(1, smr);
    Args a(17);
    a.ptr(0, dx);
    a.ptr(1, dy);
    a.ptr(2, nullptr);
    a.ptr(3, dd);
    a.u32(4, ncols_x);
    a.u3(5, 0, 0, 0);
    a.u32(6, bpr);
    a.u32(7, ystride);
    a.u32(8, nrows);
    a.u3(9, chr[0], chr[1], chr[2]);
    a.u32(10, nrows * bpr);
    a.u32(11, ystride * nc);
    a.u32(12, nrows * nc);
    a.u3(13, smr[0], smr[1], smr[2]);
    a.u32(14, nrows * bpr);
    a.u32(15, ystride * nc);
    a.u32(16, nrows * nc);
    const uint32_t rpb = nc == 1 ? 1 : 2;
    const uint32_t grid[3] = {(nrows + rpb - 1) / rpb, 1, 1}, block[3] = {32, ggml_mmvq_nwarps(nc), 1};
    int rc = run(plan, grid, block, a, stream, why);
    if (rc) return rc;
    CK(cudaMemcpy(got.data(), dd, got.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    double e = nmse(got, want);
    bool nonzero = false;
    for (float v : want) nonzero = nonzero || v != 0.0f;
    if (!(e < 1e-9) || !nonzero) {
        *why = "mmvq probe nmse " + std::to_string(e);
        return (int)cudaErrorInvalidValue;
    }
    return 0;
}

// probe.rs:392-401: quantize_case(96, 128, 3, 2, 1, 0x71), byte-exact.
int probe_quantize(const cfi_plan& plan, void* stream, std::string* why) {
    const size_t ne00 = 96, ne0 = 128, ne1 = 3, ne2 = 2, ne3 = 1, rows = ne1 * ne2 * ne3;
    Rng rng{0x71};
    std::vector<float> x(ne00 * rows);
    for (auto& v : x) v = rng.unit() * 5.0f;
    for (size_t i = 0; i < 32; i++) x[i] = 0.0f;
    for (size_t i = 32; i < 64; i++) x[i] *= 1e-6f;
    std::vector<uint8_t> want(rows * ne0 / 32 * 36), got(want.size());
    std::vector<float> row(ne0);
    for (size_t r = 0; r < rows; r++) {
        for (size_t i = 0; i < ne0; i++) row[i] = i < ne00 ? x[r * ne00 + i] : 0.0f;
        quantize_q8_1(row.data(), ne0, want.data() + r * ne0 / 32 * 36);
    }
    Dev d;
    void* dx = d.put(x.data(), x.size() * 4);
    void* dy = d.put(nullptr, want.size());
    CK(dx && dy);
    uint32_t fd[3];
    fastdiv_values((uint32_t)ne2, fd);
    Args a(9);
    a.ptr(0, dx);
    a.ptr(1, dy);
    a.u64(2, ne00);
    a.u64(3, ne00);
    a.u64(4, ne00 * ne1);
    a.u64(5, ne00 * ne1 * ne2);
    a.u64(6, ne0);
    a.u32(7, (uint32_t)ne1);
    a.u3(8, fd[0], fd[1], fd[2]);
    const uint32_t grid[3] = {(uint32_t)((ne0 + 255) / 256), (uint32_t)ne1, (uint32_t)(ne2 * ne3)}, block[3] = {256, 1, 1};
    int rc = run(plan, grid, block, a, stream, why);
    if (rc) return rc;
    CK(cudaMemcpy(got.data(), dy, got.size(), cudaMemcpyDeviceToHost) == cudaSuccess);
    size_t bad = 0;
    for (size_t i = 0; i < got.size(); i++) bad += got[i] != want[i];
    if (bad) {
        *why = "quantize probe: " + std::to_string(bad) + " of " + std::to_string(want.size()) + " bytes differ";
        return (int)cudaErrorInvalidValue;
    }
    return 0;
}

// block_q8_1_mmq of `ncols` columns of ne0 values (refs.rs:742-769).
void quantize_mmq(int ds4, const float* x, size_t ne0, size_t ncols, uint8_t* out) {
    for (size_t c = 0; c < ncols; c++)
        for (size_t g = 0; g < ne0 / 32; g++) {
            const float* v = x + c * ne0 + g * 32;
            float amax = 0.0f, sum = 0.0f;
            for (int l = 0; l < 32; l++) amax = fmaxf(amax, fabsf(v[l]));
            for (int l = 0; l < 32; l++) sum += v[l];
            float d_inv = 127.0f / amax, d = amax == 0.0f ? 0.0f : 1.0f / d_inv;
            uint8_t* o = out + ((g / 4) * ncols + c) * 144;
            if (ds4) {
                wr16(o + 4 * (g % 4), f2h(d));
                wr16(o + 4 * (g % 4) + 2, f2h(sum));
            } else {
                memcpy(o + 4 * (g % 4), &d, 4);
            }
            for (int l = 0; l < 32; l++) o[16 + (g % 4) * 32 + l] = (uint8_t)(int8_t)(amax == 0.0f ? 0 : (int)roundf(v[l] * d_inv));
        }
}

int probe_quantize_mmq(const cfi_plan& plan, void* stream, std::string* why) {
    const size_t ne0 = 256, ne1 = 5;
    Rng rng{0x3172};
    std::vector<float> x(ne0 * ne1);
    for (auto& v : x) v = rng.unit() * 2.0f;
    for (size_t i = 0; i < 32; i++) x[i] = 0.0f;
    std::vector<uint8_t> want(ne0 / 128 * ne1 * 144), got(want.size());
    quantize_mmq(plan.ty == 1, x.data(), ne0, ne1, want.data());
    Dev d;
    void* dx = d.put(x.data(), x.size() * 4);
    void* dy = d.put(nullptr, want.size());
    CK(dx && dy);
    Args a(10);
    a.ptr(0, dx);
    a.ptr(1, nullptr);
    a.ptr(2, dy);
    a.u64(3, ne0);
    a.u64(4, ne0);
    a.u64(5, ne0 * ne1);
    a.u64(6, ne0 * ne1);
    a.u64(7, ne0);
    a.u32(8, (uint32_t)ne1);
    a.u32(9, 1);
    const uint32_t grid[3] = {(uint32_t)ne1, (uint32_t)((ne0 + 511) / 512), 1}, block[3] = {128, 1, 1};
    int rc = run(plan, grid, block, a, stream, why);
    if (rc) return rc;
    CK(cudaMemcpy(got.data(), dy, got.size(), cudaMemcpyDeviceToHost) == cudaSuccess);
    size_t bad = 0;
    for (size_t i = 0; i < got.size(); i++) bad += got[i] != want[i];
    if (bad) {
        *why = "quantize_mmq probe: " + std::to_string(bad) + " bytes differ";
        return (int)cudaErrorInvalidValue;
    }
    return 0;
}

// One 32-value group of a weight block as the mmq tile loaders see it (refs.rs:659-740): signed
// quants q, the group scale d (K-quants: half(d * sc)) and, for Q4_K / Q5_K, m = half(-dmin * m).
// Q6_K: the two 16-value int8 scales in sc[] and d = the superblock d.
struct XGroup {
    int8_t q[32];
    float d = 0.0f, m = 0.0f;
    int sc[2] = {0, 0};
};

XGroup decode_group(uint32_t ty, const uint8_t* blk, int g) {
    XGroup r;
    switch (ty) {
    case 8:
        r.d = h2f(rd16(blk));
        for (int i = 0; i < 32; i++) r.q[i] = (int8_t)blk[2 + i];
        break;
    case 2:
        r.d = h2f(rd16(blk));
        for (int i = 0; i < 32; i++) r.q[i] = (int8_t)((i < 16 ? (blk[2 + i] & 15) : (blk[2 + i - 16] >> 4)) - 8);
        break;
    case 6: {
        r.d = h2f(rd16(blk));
        const uint32_t qh = rd32(blk + 2);
        for (int i = 0; i < 32; i++) {
            const int nib = i < 16 ? (blk[6 + i] & 15) : (blk[6 + i - 16] >> 4);
            r.q[i] = (int8_t)((nib | (int)(((qh >> i) & 1) << 4)) - 16);
        }
        break;
    }
    case 12:
    case 13: {
        const uint8_t* s = blk + 4;
        int scv, mv;
        if (g < 4) {
            scv = s[g] & 63;
            mv = s[g + 4] & 63;
        } else {
            scv = (s[g + 4] & 0xF) | ((s[g - 4] >> 6) << 4);
            mv = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
        }
        r.d = h2f(f2h(h2f(rd16(blk)) * (float)scv));
        r.m = h2f(f2h(-h2f(rd16(blk + 2)) * (float)mv));
        for (int i = 0; i < 32; i++) {
            const uint8_t v = blk[(ty == 12 ? 16 : 48) + 32 * (g / 2) + i];
            const int nib = g % 2 == 0 ? (v & 15) : (v >> 4);
            const int hi = ty == 13 ? ((blk[16 + i] >> g) & 1) : 0;
            r.q[i] = (int8_t)(nib | (hi << 4));
        }
        break;
    }
    default: {  // 14: Q6_K
        r.d = h2f(rd16(blk + 208));
        r.sc[0] = (int8_t)blk[192 + 2 * g];
        r.sc[1] = (int8_t)blk[192 + 2 * g + 1];
        for (int i = 0; i < 32; i++) {
            const int v = 32 * g + i, half = v / 128, rr = v % 128, quad = rr / 32, l = rr % 32;
            int lo = blk[64 * half + 32 * (quad & 1) + l];
            lo = (quad >> 1) == 0 ? (lo & 15) : (lo >> 4);
            const int hi = (blk[128 + 32 * half + l] >> (2 * quad)) & 3;
            r.q[i] = (int8_t)((lo | (hi << 4)) - 32);
        }
        break;
    }
    }
    return r;
}

bool mmq_ds4(uint32_t ty) { return ty == 2 || ty == 12 || ty == 13; }
uint32_t mmq_groups(uint32_t ty) { return (ty == 12 || ty == 13 || ty == 14) ? 8 : 1; }

// mmq reference (refs.rs:771-834), one channel and sample.
void mmq_ref(uint32_t ty, const uint8_t* x, const uint8_t* y, uint32_t ncols_x, uint32_t nrows, uint32_t ncols, float* dst) {
    const uint32_t nb = ncols_x / 32, groups = mmq_groups(ty), bb = (uint32_t)block_bytes(ty), srx = nb / groups;
    for (uint32_t c = 0; c < ncols; c++)
        for (uint32_t r = 0; r < nrows; r++) {
            float sum = 0.0f, tmp = 0.0f;
            for (uint32_t kb = 0; kb < nb; kb++) {
                const uint8_t* blk = x + ((size_t)r * srx + kb / groups) * bb;
                const uint8_t* yb = y + ((size_t)(kb / 4) * ncols + c) * 144;
                const uint8_t* yq = yb + 16 + (kb % 4) * 32;
                const XGroup xg = decode_group(ty, blk, (int)(kb % groups));
                int dots[2] = {0, 0};
                for (int i = 0; i < 32; i++) dots[i / 16] += (int)xg.q[i] * (int)(int8_t)yq[i];
                const int dot = dots[0] + dots[1];
                float db, sb = 0.0f;
                if (mmq_ds4(ty)) {
                    db = h2f(rd16(yb + 4 * (kb % 4)));
                    sb = h2f(rd16(yb + 4 * (kb % 4) + 2));
                } else {
                    memcpy(&db, yb + 4 * (kb % 4), 4);
                }
                if (ty == 8 || ty == 2 || ty == 6) {
                    sum = fmaf(xg.d * (float)dot, db, sum);
                } else if (ty == 12 || ty == 13) {
                    sum = fmaf(xg.d * db, (float)dot, sum);
                    sum = fmaf(xg.m, sb, sum);
                } else {
                    tmp = fmaf((float)(dots[0] * xg.sc[0] + dots[1] * xg.sc[1]), db, tmp);
                    if (kb % 4 == 3 || kb == nb - 1) {
                        sum = fmaf(tmp, xg.d, sum);
                        tmp = 0.0f;
                    }
                }
            }
            dst[(size_t)c * nrows + r] = sum;
        }
}

// probe.rs:369-378: mmq_case_ty(ty, 256, 70, 40, 2, 1, 1, 0x3171) (here one channel); the
// tensor-core kernel dequantises to fp16, so the bound is nmse < 1e-6 (1e-3 relative L2).
int probe_mmq(const cfi_plan& plan, void* stream, std::string* why) {
    const uint32_t ty = plan.ty, ncols_x = 256, nrows = 70, ncols = 40;
    if (ty != 8 && ty != 12 && ty != 2 && ty != 6 && ty != 13 && ty != 14) {
        *why = "no host check for this type";
        return (int)cudaErrorNotSupported;
    }
    Rng rng{0x3171};
    const uint32_t groups = mmq_groups(ty), nb = ncols_x / 32 / groups;
    std::vector<uint8_t> x = random_blocks(ty, (size_t)nrows * nb, rng);
    std::vector<float> acts((size_t)ncols_x * ncols);
    for (auto& v : acts) v = rng.unit() * 2.0f;
    std::vector<uint8_t> y(ncols_x / 128 * ncols * 144);
    quantize_mmq(mmq_ds4(ty), acts.data(), ncols_x, ncols, y.data());
    std::vector<float> want((size_t)nrows * ncols), got(want.size());
    mmq_ref(ty, x.data(), y.data(), ncols_x, nrows, ncols, want.data());
    Dev d;
    void* dx = d.put(x.data(), x.size());
    void* dy = d.put(y.data(), y.size());
    void* dd = d.put(nullptr, want.size() * 4);
    CK(dx && dy && dd);
    Args a(23);
    a.ptr(0, dx);
    a.ptr(1, dy);
    a.ptr(2, nullptr);
    a.ptr(3, nullptr);
    a.ptr(4, dd);
    a.ptr(5, nullptr);
    const uint32_t ychan = ncols_x / 128 * ncols * 36;
    const uint32_t w[17] = {ncols_x, nrows, ncols, nb, ncols, nrows, 1, 1, nrows * nb, ychan, nrows * ncols, 1, 1,
                            nrows * nb, ychan, nrows * ncols, ncols};
    for (int i = 0; i < 17; i++) a.u32(6 + i, w[i]);
    const uint32_t grid[3] = {1, 1, 1}, block[3] = {32, 8, 1};
    int rc = run(plan, grid, block, a, stream, why);
    if (rc) return rc;
    CK(cudaMemcpy(got.data(), dd, got.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    double e = nmse(got, want);
    if (!(e < 1e-6)) {
        *why = "mmq probe nmse " + std::to_string(e);
        return (int)cudaErrorInvalidValue;
    }
    return 0;
}

int probe_rms(const cfi_plan& plan, void* stream, std::string* why) {
    const bool plain = plan.kernel == CFI_K_RMS_NORM_PLAIN;
    const uint32_t rows = 4, ncols = plain ? 32 : 896;
    const float eps = plain ? 1e-5f : 1e-6f;
    const bool mul = !plain && (plan.aux & 1), add = !plain && (plan.aux & 2);
    Rng rng{0xA11CE};
    std::vector<float> x((size_t)rows * ncols), w(ncols), b(ncols), want(x.size()), got(x.size());
    for (auto& v : x) v = rng.unit();
    for (auto& v : w) v = rng.unit();
    for (auto& v : b) v = rng.unit();
    for (uint32_t r = 0; r < rows; r++) {
        float ss = 0.0f;
        for (uint32_t c = 0; c < ncols; c++) ss += x[r * ncols + c] * x[r * ncols + c];
        float sc = 1.0f / sqrtf(ss / ncols + eps);
        for (uint32_t c = 0; c < ncols; c++) {
            float v = sc * x[r * ncols + c];
            if (mul) v *= w[c];
            if (add) v += b[c];
            want[r * ncols + c] = v;
        }
    }
    Dev d;
    void* dx = d.put(x.data(), x.size() * 4);
    void* dw = d.put(w.data(), w.size() * 4);
    void* db = d.put(b.data(), b.size() * 4);
    void* dd = d.put(nullptr, x.size() * 4);
    CK(dx && dw && db && dd);
    const uint32_t grid[3] = {rows, 1, 1};
    int rc;
    if (plain) {
        Args a(9);
        a.ptr(0, dx);
        a.ptr(1, dd);
        a.u32(2, ncols);
        a.u32(3, 1);
        a.u32(4, 1);
        a.u64(5, ncols);
        a.u64(6, (uint64_t)rows * ncols);
        a.u64(7, (uint64_t)rows * ncols);
        a.f32(8, eps);
        const uint32_t block[3] = {32, 1, 1};
        rc = run(plan, grid, block, a, stream, why);
    } else {
        uint32_t fc[3], f1[3];
        fastdiv_values(ncols, fc);
        fastdiv_values(1, f1);
        Args a(23);
        a.ptr(0, dx);
        a.ptr(1, dd);
        a.u32(2, ncols);
        a.u64(3, ncols);
        a.u64(4, (uint64_t)rows * ncols);
        a.u64(5, (uint64_t)rows * ncols);
        a.f32(6, eps);
        a.ptr(7, dw);
        a.u64(8, 0);
        a.u64(9, 0);
        a.u64(10, 0);
        a.u3(11, fc[0], fc[1], fc[2]);
        a.u3(12, f1[0], f1[1], f1[2]);
        a.u3(13, f1[0], f1[1], f1[2]);
        a.u3(14, f1[0], f1[1], f1[2]);
        a.ptr(15, db);
        a.u64(16, 0);
        a.u64(17, 0);
        a.u64(18, 0);
        a.u3(19, fc[0], fc[1], fc[2]);
        a.u3(20, f1[0], f1[1], f1[2]);
        a.u3(21, f1[0], f1[1], f1[2]);
        a.u3(22, f1[0], f1[1], f1[2]);
        const uint32_t block[3] = {256, 1, 1};
        rc = run(plan, grid, block, a, stream, why);
    }
    if (rc) return rc;
    CK(cudaMemcpy(got.data(), dd, got.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    double e = nmse(got, want);
    if (!(e < 1e-9)) {
        *why = "rms_norm probe nmse " + std::to_string(e);
        return (int)cudaErrorInvalidValue;
    }
    return 0;
}

int probe_rope(const cfi_plan& plan, void* stream, std::string* why) {
    const int ne0 = 64, ne1 = 2, ntok = 3, n_dims = 64;
    const bool fwd = plan.aux & 1, has_ff = (plan.aux >> 1) & 1;
    const float base = 1e6f, theta_scale = powf(base, -2.0f / n_dims);
    const int32_t pos[ntok] = {0, 3, 631};
    Rng rng{0xC0FFEE};
    std::vector<float> x((size_t)ne0 * ne1 * ntok), ff(n_dims / 2), want(x.size()), got(x.size());
    for (auto& v : x) v = rng.unit();
    for (auto& v : ff) v = 1.0f + 0.5f * (rng.unit() + 1.0f);
    for (int t = 0; t < ntok; t++)
        for (int h = 0; h < ne1; h++) {
            const float* s = &x[(size_t)(t * ne1 + h) * ne0];
            float* o = &want[(size_t)(t * ne1 + h) * ne0];
            for (int i = 0; i < n_dims / 2; i++) {
                float th = (float)pos[t] * powf(theta_scale, (float)i);
                if (has_ff) th /= ff[i];
                float cs = cosf(th), sn = sinf(th);
                if (!fwd) sn = -sn;
                o[i] = s[i] * cs - s[i + n_dims / 2] * sn;
                o[i + n_dims / 2] = s[i] * sn + s[i + n_dims / 2] * cs;
            }
            for (int i = n_dims; i < ne0; i++) o[i] = s[i];
        }
    Dev d;
    void* dx = d.put(x.data(), x.size() * 4);
    void* dp = d.put(pos, sizeof pos);
    void* df = d.put(ff.data(), ff.size() * 4);
    void* dd = d.put(nullptr, x.size() * 4);
    CK(dx && dp && df && dd);
    Args a(14);
    a.ptr(0, dx);
    a.ptr(1, dd);
    a.u32(2, ne0);
    a.u32(3, ne1);
    a.u32(4, ne0);
    a.u32(5, ne0 * ne1);
    a.u32(6, n_dims);
    a.ptr(7, dp);
    a.f32(8, 1.0f);
    a.f32(9, 0.0f);
    a.f32(10, 1.0f);
    const float corr[2] = {0.0f, 0.0f};
    a.set(11, corr, 8);
    a.f32(12, theta_scale);
    a.ptr(13, has_ff ? df : nullptr);
    const uint32_t grid[3] = {(uint32_t)(ne1 * ntok), (uint32_t)((ne0 + 511) / 512), 1}, block[3] = {1, 256, 1};
    int rc = run(plan, grid, block, a, stream, why);
    if (rc) return rc;
    CK(cudaMemcpy(got.data(), dd, got.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    double e = nmse(got, want);
    if (!(e < 1e-6)) {
        *why = "rope probe nmse " + std::to_string(e);
        return (int)cudaErrorInvalidValue;
    }
    return 0;
}

// tests/gpu/soft_max_generic.rs:64-92 case: 12 columns, 2 heads, scale 0.125, last column masked.
int probe_soft_max(const cfi_plan& plan, void* stream, std::string* why) {
    const int ne0 = 12, ne1 = 1, ne2 = 2;
    const float scale = 0.125f;
    const bool f16 = plan.aux & 1;
    std::vector<float> x(ne0 * ne1 * ne2), mask(ne0 * ne1), want(x.size()), got(x.size());
    for (size_t i = 0; i < x.size(); i++) x[i] = 0.03f * (float)(i % 23) - 0.2f;
    for (int i = 0; i < ne0; i++) mask[i] = i < 11 ? 0.0f : -INFINITY;
    for (int r = 0; r < ne1 * ne2; r++) {
        const float* s = &x[r * ne0];
        const float* m = &mask[(r % ne1) * ne0];
        float mx = -INFINITY, sum = 0.0f;
        for (int i = 0; i < ne0; i++) mx = fmaxf(mx, s[i] * scale + m[i]);
        for (int i = 0; i < ne0; i++) sum += (want[r * ne0 + i] = expf(s[i] * scale + m[i] - mx));
        for (int i = 0; i < ne0; i++) want[r * ne0 + i] /= sum;
    }
    std::vector<uint16_t> mask16(mask.size());
    for (size_t i = 0; i < mask.size(); i++) mask16[i] = f2h(mask[i]);
    Dev d;
    void* dx = d.put(x.data(), x.size() * 4);
    void* dm = f16 ? d.put(mask16.data(), mask16.size() * 2) : d.put(mask.data(), mask.size() * 4);
    void* dd = d.put(nullptr, x.size() * 4);
    CK(dx && dm && dd);
    struct {
        int64_t nheads;
        uint32_t n_head_log2, pad;
        int64_t ncols, nrows_x, nrows_y, ne00, ne01, ne02, ne03, nb11, nb12, nb13, ne12, ne13;
        float scale, max_bias, m0, m1;
    } p = {ne2, 1, 0, ne0, ne1 * ne2, ne1, ne0, ne1, ne2, 1,
           (int64_t)ne0 * (f16 ? 2 : 4), (int64_t)ne0 * ne1 * (f16 ? 2 : 4), (int64_t)ne0 * ne1 * (f16 ? 2 : 4), 1, 1,
           scale, 0.0f, 1.0f, 1.0f};
    static_assert(sizeof(p) == 128, "params");
    Args a(5);
    a.ptr(0, dx);
    a.ptr(1, dm);
    a.ptr(2, nullptr);
    a.ptr(3, dd);
    std::vector<uint64_t> big(16);
    memcpy(big.data(), &p, 128);
    a.ptrs.resize(5);
    a.ptrs[4] = big.data();
    const uint32_t grid[3] = {(uint32_t)ne1, (uint32_t)ne2, 1}, block[3] = {32, 1, 1};
    int rc = run(plan, grid, block, a, stream, why);
    if (rc) return rc;
    CK(cudaMemcpy(got.data(), dd, got.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    double e = nmse(got, want);
    if (!(e < 1e-9)) {
        *why = "soft_max probe nmse " + std::to_string(e);
        return (int)cudaErrorInvalidValue;
    }
    return 0;
}

}  // namespace

// probe.rs:379-390: one FlashAttention tile (16 + 3 queries), 4 heads over 2 KV heads, 70 keys
// (a partial chunk), causal mask with a padded third, seed 0xfa77 (probe.rs:421-446); exact f64
// attention on the host.  fp16 Q and P on the tensor cores (nmse about 4e-8): accepted below 1e-6.
int probe_fattn(const cfi_plan& plan, void* stream, std::string* why) {
    const uint32_t d = plan.aux, nq = 19, nh = 4, nhk = 2, nkv = 70, ns = 1, nq_pad = 32;
    if (d != 64 && d != 128) {
        *why = "no host check for this head size";
        return (int)cudaErrorNotSupported;
    }
    Rng rng{0xfa77};
    std::vector<float> q((size_t)d * nq * nh * ns);
    std::vector<uint16_t> k((size_t)d * nkv * nhk * ns), v(k.size()), m((size_t)nkv * nq_pad * ns);
    for (auto& x : q) x = rng.unit();
    for (auto& x : k) x = f2h(rng.unit());
    for (auto& x : v) x = f2h(rng.unit());
    for (uint32_t i = 0; i < nq_pad; i++)
        for (uint32_t j = 0; j < nkv; j++) {
            const uint32_t nvis = nkv - nkv / 3;
            const bool visible = j < nvis && j + nq <= nvis + i;
            m[(size_t)i * nkv + j] = visible ? f2h(rng.unit() * 0.5f) : (uint16_t)0xfc00;
        }
    const float scale = 1.0f / sqrtf((float)d);
    std::vector<float> want((size_t)d * nh * nq * ns), got(want.size());
    for (uint32_t h = 0; h < nh; h++)
        for (uint32_t i = 0; i < nq; i++) {
            std::vector<double> sc(nkv);
            double mx = -INFINITY;
            for (uint32_t j = 0; j < nkv; j++) {
                double acc = 0;
                for (uint32_t t = 0; t < d; t++)
                    acc += (double)(q[((size_t)h * nq + i) * d + t] * scale) * (double)h2f(k[((size_t)(h / 2) * nkv + j) * d + t]);
                acc += (double)h2f(m[(size_t)i * nkv + j]);
                sc[j] = acc;
                mx = std::max(mx, acc);
            }
            double l = 0;
            for (auto& x : sc) l += (x = exp(x - mx));
            for (uint32_t t = 0; t < d; t++) {
                double o = 0;
                for (uint32_t j = 0; j < nkv; j++) o += sc[j] * (double)h2f(v[((size_t)(h / 2) * nkv + j) * d + t]);
                want[((size_t)i * nh + h) * d + t] = (float)(o / l);
            }
        }
    Dev dv;
    void* dq = dv.put(q.data(), q.size() * 4);
    void* dk = dv.put(k.data(), k.size() * 2);
    void* dvv = dv.put(v.data(), v.size() * 2);
    void* dm = dv.put(m.data(), m.size() * 2);
    void* dd = dv.put(nullptr, want.size() * 4);
    CK(dq && dk && dvv && dm && dd);
    Args a(37);
    a.ptr(0, dq);
    a.ptr(1, dk);
    a.ptr(2, dvv);
    a.ptr(3, dm);
    a.ptr(4, nullptr);
    a.ptr(5, nullptr);
    a.ptr(6, dd);
    a.ptr(7, nullptr);
    a.f32(8, scale);
    a.f32(9, 0.0f);
    a.f32(10, 1.0f);
    a.f32(11, 1.0f);
    a.u32(12, 0);
    a.f32(13, 0.0f);
    const uint32_t w[] = {d, nq, nh, ns, d * 4, d * 4 * nq, d * 4 * nq * nh, d, nkv, nhk, ns, d * 2, d * 2 * nkv};
    for (int i = 0; i < 13; i++) a.u32(14 + i, w[i]);
    a.u64(27, (uint64_t)d * 2 * nkv * nhk);
    a.u32(28, d * 2);
    a.u32(29, d * 2 * nkv);
    a.u64(30, (uint64_t)d * 2 * nkv * nhk);
    a.u32(31, nkv);
    a.u32(32, nq_pad);
    a.u32(33, ns);
    a.u32(34, nkv * 2);
    a.u32(35, nkv * 2 * nq_pad);
    a.u64(36, (uint64_t)nkv * 2 * nq_pad);
    const uint32_t grid[3] = {2, nh, ns}, block[3] = {32, 4, 1};
    int rc = run(plan, grid, block, a, stream, why);
    if (rc) return rc;
    CK(cudaMemcpy(got.data(), dd, got.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    const double e = nmse(got, want);
    if (!(e < 1e-6)) {
        *why = "fattn probe nmse " + std::to_string(e);
        return (int)cudaErrorInvalidValue;
    }
    return 0;
}

int probe_validate(const cfi_plan& plan, void* stream, std::string* why) {
    switch (plan.kernel) {
    case CFI_K_FATTN: return probe_fattn(plan, stream, why);
    case CFI_K_FATTN_FIXUP: return 0;
    case CFI_K_MMVQ: return probe_mmvq(plan, stream, why);
    case CFI_K_QUANTIZE_Q8_1: return probe_quantize(plan, stream, why);
    case CFI_K_QUANTIZE_MMQ: return probe_quantize_mmq(plan, stream, why);
    case CFI_K_MMQ: return probe_mmq(plan, stream, why);
    case CFI_K_MMQ_FIXUP: return 0;
    case CFI_K_RMS_NORM:
    case CFI_K_RMS_NORM_PLAIN: return probe_rms(plan, stream, why);
    case CFI_K_ROPE_NEOX: return probe_rope(plan, stream, why);
    case CFI_K_SOFT_MAX: return probe_soft_max(plan, stream, why);
    default: *why = "unknown kernel"; return (int)cudaErrorNotSupported;
    }
}

}  // namespace cfi
