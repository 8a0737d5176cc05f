// k_mmq_sm100.cu -- prefill quantized GEMM (the native mul_mat_q) on the 5th-generation tensor
// cores of sm_100a.
//
// dst[col][row] = sum_k W[row][k] * X[col][k] with W in ggml Q8_0 (or Q4_K) blocks and X in
// block_q8_1_mmq (144 B per 128 values of a column), the inputs of ggml-cuda's
// mul_mat_q<type, mmq_x, need_check> (cuda-for-intel src/subst/mmq.rs:1-14, refs.rs:771-834).
//
// Design (one CTA per 128-row x BN-column output tile, BN <= 256, 320 threads):
//   1. pre-pass: the quantized activations become an fp16 K-major matrix  Xh[plane][col][Kt]
//      (fp16(q * d) per value; for Q4_K the per-32 float sums s are appended as extra K columns);
//   2. warp 9 streams Xh tiles with TMA (128-byte swizzle, the UMMA canonical K-major layout);
//   3. warps 0-7 stream the raw weight bytes with coalesced cp.async into shared memory (a copy
//      plan computed once per thread) and dequantize them, two threads per tile row, to fp16 in
//      the same swizzled layout (Q8_0: fp16(q * d); Q4_K: fp16(q * half(d*sc)) and, in the
//      appended K columns, half(-dmin*m) against s -- the reference's `fma(dmA.y, dsB.y, sum)`
//      term); one reducing named barrier per stage;
//   4. one thread of warp 8 issues tcgen05.mma kind::f16 (M=128, N=BN, K=16) with the fp32
//      accumulator in tensor memory; commits free each pipeline slot;
//   5. warps 0-7 drain TMEM (tcgen05.ld 32x32b) into 32x32 chunks in shared memory, stored by
//      TMA (or, for strides TMA cannot describe, as 16-byte runs of rows).
// Integer exactness does not apply here: fp16 rounding of q*d keeps the result within 1e-3
// relative L2 of the reference (measured ~1e-4), the bound this path is held to.
#include <cuda.h>

#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/cfi_glue.h"
#include "../../include/cfi_peer.h"
#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "sm100_ptx.cuh"
#include "subst_host.hpp"
#include "tc_epilogue.cuh"

static __device__ unsigned int g_cfi_device_error;

namespace {

using namespace sm100;

constexpr int BM = 128;          // rows per tile (TMEM lanes)
constexpr int BK = 64;           // K per pipeline stage (one 128-byte swizzle atom of fp16)
constexpr int NSTAGE = 4;        // A/B smem ring
constexpr int NRAW = 3;          // raw weight staging ring (cp.async prefetch depth NRAW - 1)
constexpr int A_STAGE = BM * BK * 2;      // 16 KB
constexpr int B_STAGE = 256 * BK * 2;     // 32 KB (sized for BN = 256)
constexpr int RAW_WORDS_Q8 = 17;          // 68 bytes = 2 Q8_0 blocks per row per stage
constexpr int RAW_STAGE = BM * 20 * 4;    // 10 KB (room for 20 words per row)
constexpr int NPROD = 256;                // warps 0-7: weight producers, then the epilogue
constexpr int MMA_WARP = 8, TMA_WARP = 9;
constexpr int THREADS = 320;
constexpr size_t SMEM_BYTES = 1024 /*align slack*/ + (size_t)NSTAGE * (A_STAGE + B_STAGE) + (size_t)NRAW * RAW_STAGE + 256;

struct MmqArgs {
    const uint8_t* x;     // weights (ggml blocks)
    float* dst;
    uint32_t K, Kt;       // K of the product; Kt = K plus appended correction columns (Q4_K)
    uint32_t nrows, ncols_dst, bn;
    uint32_t stride_row_x;                     // blocks
    uint32_t stride_col_dst;
    uint32_t nchannels_y, channel_ratio, sample_ratio;
    uint32_t stride_channel_x, stride_sample_x;    // blocks
    uint32_t stride_channel_dst, stride_sample_dst;
    int tma_c;  // dst stored through tmap_c (16-byte aligned column, channel and sample strides)
    unsigned int* err;
};

CFI_DEV uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// 4 signed bytes -> two half2 {b0,b1}, {b2,b3} (exact), scaled by d (one fp16 rounding each).
CFI_DEV void dequant4(uint32_t w, __half2 d2, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t p0 = __byte_perm(u, 0x64646464u, 0x4140);
    const uint32_t p1 = __byte_perm(u, 0x64646464u, 0x4342);
    const __half2 bias = __float2half2_rn(1152.0f);
    __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&p0), bias);
    __half2 b = __hsub2(*reinterpret_cast<const __half2*>(&p1), bias);
    lo = h2_bits(__hmul2(a, d2));
    hi = h2_bits(__hmul2(b, d2));
}

// Unsigned nibbles (0..15) of 4 bytes selected by `shift` -> two half2, scaled by d.
CFI_DEV void dequant4_u4(uint32_t w, uint32_t shift, __half2 d2, uint32_t& lo, uint32_t& hi) {
    const uint32_t n = (w >> shift) & 0x0F0F0F0Fu;
    const uint32_t p0 = __byte_perm(n, 0x64646464u, 0x4140);
    const uint32_t p1 = __byte_perm(n, 0x64646464u, 0x4342);
    const __half2 bias = __float2half2_rn(1024.0f);
    __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&p0), bias);
    __half2 b = __hsub2(*reinterpret_cast<const __half2*>(&p1), bias);
    lo = h2_bits(__hmul2(a, d2));
    hi = h2_bits(__hmul2(b, d2));
}

// Per-type mmq traits (refs.rs:641-649): values per weight block, block bytes, the q8_1_mmq
// activation layout (DS4: half d + half sum per 32 values; else float d) and whether the
// min term needs appended correction columns (Q4_K, Q5_K).
template <uint32_t TY> constexpr uint32_t mmq_qk() { return (TY == T_Q4_K || TY == T_Q5_K || TY == T_Q6_K) ? 256u : 32u; }
template <uint32_t TY> constexpr uint32_t mmq_bb() {
    return TY == T_Q8_0 ? Q8_0_BYTES : TY == T_Q4_0 ? Q4_0_BYTES : TY == T_Q5_0 ? Q5_0_BYTES
         : TY == T_Q4_K ? Q4_K_BYTES : TY == T_Q5_K ? Q5_K_BYTES : Q6_K_BYTES;
}
template <uint32_t TY> constexpr int mmq_ds4() { return (TY == T_Q4_0 || TY == T_Q4_K || TY == T_Q5_K) ? 1 : 0; }
template <uint32_t TY> constexpr int mmq_corr() { return (TY == T_Q4_K || TY == T_Q5_K) ? 1 : 0; }

// 4 unsigned bytes (0..255, exact in fp16) -> two half2, scaled by d.
CFI_DEV void dequant4_ub(uint32_t b, __half2 d2, uint32_t& lo, uint32_t& hi) {
    const uint32_t p0 = __byte_perm(b, 0x64646464u, 0x4140);
    const uint32_t p1 = __byte_perm(b, 0x64646464u, 0x4342);
    const __half2 bias = __float2half2_rn(1024.0f);
    __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&p0), bias);
    __half2 c = __hsub2(*reinterpret_cast<const __half2*>(&p1), bias);
    lo = h2_bits(__hmul2(a, d2));
    hi = h2_bits(__hmul2(c, d2));
}

CFI_DEV void st_chunk(uint8_t* atom, int r, int c, uint32_t a, uint32_t b, uint32_t cc, uint32_t d) {
    uint4 v = make_uint4(a, b, cc, d);
    *reinterpret_cast<uint4*>(atom + r * 128 + ((c ^ (r & 7)) << 4)) = v;
}

CFI_DEV int scale_byte(const uint32_t* s, int k) { return (int)((s[k >> 2] >> (8 * (k & 3))) & 0xffu); }

// bar.red.and over `n` threads of named barrier `id`: true on every thread iff `v` on all.
CFI_DEV bool named_bar_and(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

// Warp roles: 0-7 weight producers (two threads per tile row, one 32-value group each per stage)
// and afterwards the epilogue; 8 tensor memory + MMA issue; 9 activation TMA.
template <uint32_t TY>
__global__ void __launch_bounds__(THREADS, 1)
    cfi_mmq_tc(const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ CUtensorMap tmap_c, const MmqArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = sA + NSTAGE * A_STAGE;
    uint8_t* sRaw = sB + NSTAGE * B_STAGE;
    uint64_t* full = reinterpret_cast<uint64_t*>(sRaw + NRAW * RAW_STAGE);
    uint64_t* empty = full + NSTAGE;
    uint64_t* done = empty + NSTAGE;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* epi_ok = abort_flag + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t bn = a.bn;
    const uint32_t tmem_cols = bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : 256;
    const int nstages = (int)(a.Kt / BK);
    const int kstages = (int)(a.K / BK);

    if (tid == 0) {
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(&full[i], NPROD / 32 + 1);  // one arrival per producer warp + the TMA thread's expect_tx
            mbar_init(&empty[i], 1);         // tcgen05.commit
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == MMA_WARP) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // tile coordinates
    const uint32_t row0 = blockIdx.x * BM, col0 = blockIdx.y * bn, plane = blockIdx.z;
    const uint32_t wt = plane / a.nchannels_y, zt = plane - wt * a.nchannels_y;
    const size_t x_off = (size_t)(wt / a.sample_ratio) * a.stride_sample_x + (size_t)(zt / a.channel_ratio) * a.stride_channel_x;
    float* dst = a.dst + (size_t)wt * a.stride_sample_dst + (size_t)zt * a.stride_channel_dst;

    if (warp < NPROD / 32) {
        // ================= weight producers (256 threads) =================
        constexpr uint32_t BB = TY == T_Q4_K ? Q4_K_BYTES : Q8_0_BYTES;
        // raw words per row per stage: Q8_0 two blocks (17 words); Q4_K header (4) + 32 qs bytes (8);
        // RS is the padded row stride in shared memory (odd: conflict-free row-per-thread reads)
        constexpr int RW = TY == T_Q4_K ? 12 : RAW_WORDS_Q8;
        constexpr int RS = TY == T_Q4_K ? 13 : RAW_WORDS_Q8;
        constexpr int NCP = (BM * RW + NPROD - 1) / NPROD;  // raw words this thread copies per stage
        const int r = tid & (BM - 1), hh = tid >> 7;        // tile row, group of the stage (0/1)
        // copy plan, fixed for the whole K loop: word w = tid + NPROD * m of the stage
        const uint8_t* xbase = a.x + (x_off + (size_t)row0 * a.stride_row_x) * BB;
        uint32_t goff[NCP], soff[NCP], live = 0, inrow = 0, qsword = 0;
#pragma unroll
        for (int m = 0; m < NCP; m++) {
            const int w = tid + NPROD * m;
            const int rr = w / RW, j = w - rr * RW;
            const uint32_t row = row0 + (uint32_t)rr;
            goff[m] = (min(row, a.nrows - 1) - row0) * a.stride_row_x * BB +
                      (uint32_t)(TY == T_Q4_K ? (j < 4 ? 4 * j : 16 + 4 * (j - 4)) : 4 * j);
            soff[m] = (uint32_t)(rr * RS + j) * 4u;
            if (w < BM * RW) live |= 1u << m;
            if (row < a.nrows) inrow |= 1u << m;
            if (TY == T_Q4_K && j >= 4) qsword |= 1u << m;
        }
        auto issue = [&](int s) {
            if (s >= kstages) return;  // Q4_K correction stages read their headers directly
            uint8_t* raw = sRaw + (s % NRAW) * RAW_STAGE;
            const uint32_t st = TY == T_Q4_K ? (uint32_t)(s >> 2) * Q4_K_BYTES : (uint32_t)s * 68u;
            const uint32_t sq = TY == T_Q4_K ? 32u * (uint32_t)(s & 3) : 0u;
#pragma unroll
            for (int m = 0; m < NCP; m++)
                if (live >> m & 1u)
                    cp_async4(raw + soff[m], xbase + goff[m] + st + ((qsword >> m & 1u) ? sq : 0u), (inrow >> m & 1u) ? 4u : 0u);
        };
        for (int s = 0; s < NRAW - 1; s++) {
            if (s < nstages) issue(s);
            cp_async_commit();
        }
        for (int s = 0; s < nstages; s++) {
            cp_async_wait<NRAW - 2>();  // this thread's copies of stage s have landed
            const int slot = s % NSTAGE;
            const uint32_t round = (uint32_t)(s / NSTAGE);
            bool ok = lane != 0 || mbar_wait(&empty[slot], (round & 1) ^ 1, abort_flag);
            // (lane 0 of each warp waits for the MMA to release this A slot)  every producer's
            // stage-s copies are visible, every producer finished stage s-1 (its raw slot may be
            // refilled), and the slot is free -- on all threads or none
            ok = named_bar_and(1, NPROD, ok);
            if (!ok) {
                if (tid == 0) {
                    cfi_set_error(a.err, 0x100 + slot);
                    *abort_flag = 1;
                }
                break;
            }
            if (s + NRAW - 1 < nstages) issue(s + NRAW - 1);
            cp_async_commit();
            const uint32_t* W = reinterpret_cast<const uint32_t*>(sRaw + (s % NRAW) * RAW_STAGE) + r * RS;
            uint8_t* atom = sA + slot * A_STAGE;
            if (TY == T_Q8_0) {
                if (hh == 0) {  // block 0: d at bytes 0..1, quants at bytes 2..33
                    uint32_t w[9];
#pragma unroll
                    for (int j = 0; j < 9; j++) w[j] = W[j];
                    const __half2 d0 = __half2half2(__ushort_as_half((uint16_t)(w[0] & 0xffffu)));
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const uint32_t q0 = __funnelshift_r(w[2 * c], w[2 * c + 1], 16);
                        const uint32_t q1 = __funnelshift_r(w[2 * c + 1], w[2 * c + 2], 16);
                        uint32_t v0, v1, v2, v3;
                        dequant4(q0, d0, v0, v1);
                        dequant4(q1, d0, v2, v3);
                        st_chunk(atom, r, c, v0, v1, v2, v3);
                    }
                } else {  // block 1: d at bytes 34..35, quants at bytes 36..67 (words 9..16)
                    uint32_t w[9];
#pragma unroll
                    for (int j = 0; j < 9; j++) w[j] = W[8 + j];
                    const __half2 d1 = __half2half2(__ushort_as_half((uint16_t)(w[0] >> 16)));
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        uint32_t v0, v1, v2, v3;
                        dequant4(w[1 + 2 * c], d1, v0, v1);
                        dequant4(w[2 + 2 * c], d1, v2, v3);
                        st_chunk(atom, r, 4 + c, v0, v1, v2, v3);
                    }
                }
            } else if (s < kstages) {  // Q4_K: sub-block 2(s%4) + hh of superblock s/4
                uint32_t hdr[4], q[8];
#pragma unroll
                for (int j = 0; j < 4; j++) hdr[j] = W[j];
#pragma unroll
                for (int j = 0; j < 8; j++) q[j] = W[4 + j];
                const float dd = __half2float(__ushort_as_half((uint16_t)(hdr[0] & 0xffffu)));
                const uint32_t* sc = hdr + 1;
                const int g = 2 * (s & 3) + hh;
                int scv;
                if (g < 4)
                    scv = scale_byte(sc, g) & 63;
                else
                    scv = (scale_byte(sc, g + 4) & 0xF) | ((scale_byte(sc, g - 4) >> 6) << 4);
                // the reference's tile loader stores half(d * sc) (refs.rs:709-712)
                const __half2 d2 = __half2half2(__float2half_rn(dd * (float)scv));
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    uint32_t v0, v1, v2, v3;
                    dequant4_u4(q[2 * c], 4 * hh, d2, v0, v1);
                    dequant4_u4(q[2 * c + 1], 4 * hh, d2, v2, v3);
                    st_chunk(atom, r, 4 * hh + c, v0, v1, v2, v3);
                }
            } else {  // Q4_K correction stage: A[r][K + g] = half(-dmin * m_g) (refs.rs:712)
                const int g0 = (s - kstages) * BK;
                const int ngroups = (int)(a.K / 32);
                const uint32_t row = row0 + r;
                const uint8_t* rowp = xbase + (size_t)(min(row, a.nrows - 1) - row0) * a.stride_row_x * BB;
#pragma unroll 1
                for (int sbl = 4 * hh; sbl < 4 * hh + 4; sbl++) {  // 8 superblocks (8 groups each) per stage
                    const int gbase = g0 + 8 * sbl;
                    uint32_t hw0 = 0, hs[3] = {0, 0, 0};
                    if (row < a.nrows && gbase < ngroups) {
                        const uint32_t* H = reinterpret_cast<const uint32_t*>(rowp + (size_t)(gbase / 8) * Q4_K_BYTES);
                        hw0 = __ldg(H);
                        hs[0] = __ldg(H + 1);
                        hs[1] = __ldg(H + 2);
                        hs[2] = __ldg(H + 3);
                    }
                    const float dmin = __half2float(__ushort_as_half((uint16_t)(hw0 >> 16)));
                    uint32_t v[4];
#pragma unroll
                    for (int p = 0; p < 4; p++) {
                        uint32_t hv[2];
#pragma unroll
                        for (int e = 0; e < 2; e++) {
                            const int gg = 2 * p + e;
                            const int mv = gg < 4 ? (scale_byte(hs, gg + 4) & 63)
                                                  : ((scale_byte(hs, gg + 4) >> 4) | ((scale_byte(hs, gg) >> 6) << 4));
                            hv[e] = gbase < ngroups ? (uint32_t)__half_as_ushort(__float2half_rn(-dmin * (float)mv)) : 0u;
                        }
                        v[p] = hv[0] | (hv[1] << 16);
                    }
                    st_chunk(atom, r, sbl, v[0], v[1], v[2], v[3]);
                }
            }
            fence_proxy_async_smem();  // this thread's A-tile writes, visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[slot]);
        }
        cp_async_wait<0>();
        // ================= epilogue: TMEM -> shared -> dst (16-byte stores) =================
        if (tid == 0) {
            bool got = false;
            if (!*abort_flag) {
                got = mbar_wait(done, 0, abort_flag);
                if (!got) {
                    cfi_set_error(a.err, 0x200);
                    *abort_flag = 1;
                }
            }
            *epi_ok = got ? 1 : 0;
        }
        named_bar_sync(1, NPROD);
        tc_fence_after();
        if (*epi_ok && a.tma_c) {
            // every MMA has completed: the A ring holds the 8 KB per-warp staging buffers
            float* tbuf = reinterpret_cast<float*>(sA) + warp * 2048;
            tmem_tile_tma_store(tmem, warp, lane, NPROD / 32, bn, tbuf, &tmap_c, (int)row0, (int)col0, (int)zt, (int)wt,
                                [](float v) { return v; });
        } else if (*epi_ok) {
            // every MMA has completed: the A ring is free for the 4 KB per-warp staging buffers
            float* buf = reinterpret_cast<float*>(sA) + warp * 1024;
            const bool vec = (a.stride_col_dst & 3u) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
            tmem_tile_store(tmem, warp, lane, NPROD / 32, bn, buf, [&](uint32_t c, uint32_t rr, float4 f) {
                const uint32_t col = col0 + c, row = row0 + rr;
                if (col >= a.ncols_dst || row >= a.nrows) return;
                float* p = dst + (size_t)col * a.stride_col_dst + row;
                if (vec && row + 3 < a.nrows) {
                    *reinterpret_cast<float4*>(p) = f;
                } else {
                    p[0] = f.x;
                    if (row + 1 < a.nrows) p[1] = f.y;
                    if (row + 2 < a.nrows) p[2] = f.z;
                    if (row + 3 < a.nrows) p[3] = f.w;
                }
            });
        }
    } else if (warp == MMA_WARP) {
        // ================= MMA issuer =================
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(BM, bn, 0);
            for (int s = 0; s < nstages; s++) {
                const int slot = s % NSTAGE;
                if (!mbar_wait(&full[slot], (uint32_t)(s / NSTAGE) & 1, abort_flag)) {
                    cfi_set_error(a.err, 0x300 + slot);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t abase = smem_u32(sA + slot * A_STAGE), bbase = smem_u32(sB + slot * B_STAGE);
#pragma unroll
                for (int k = 0; k < BK / 16; k++)
                    mma_f16(tmem, sw128_kmajor_desc(abase + 32 * k), sw128_kmajor_desc(bbase + 32 * k), idesc,
                            (s > 0 || k > 0) ? 1u : 0u);
                mma_commit(&empty[slot]);
            }
            mma_commit(done);  // also after a failure: `done` then tracks the MMAs already issued
        }
        __syncwarp();
    } else {
        // ================= activation TMA =================
        if (lane == 0) {
            prefetch_tmap(&tmap_b);
            const uint32_t bytes = bn * BK * 2;
            for (int s = 0; s < nstages; s++) {
                const int slot = s % NSTAGE;
                if (!mbar_wait(&empty[slot], ((uint32_t)(s / NSTAGE) & 1) ^ 1, abort_flag)) {
                    cfi_set_error(a.err, 0x400 + slot);
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full[slot], bytes);
                tma_load_3d(sB + slot * B_STAGE, &tmap_b, s * BK, (int)col0, (int)plane, &full[slot]);
            }
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
}

// ---- quantized GEMM with TMA-staged raw weight tiles (the default prefill path) ----
// Warp 10 streams the raw weight bytes of one 256-value K chunk for the tile's 128 rows per TMA
// load (Q4_K: one superblock, 144 B per row; Q8_0: eight blocks, 272 B per row) into a ring of
// raw slots; warps 0-7 dequantize each 64-value stage of a chunk into the fp16 A ring (two
// threads per row, one 32-value group each, stored in the 128-byte swizzled K-major layout);
// warp 9 streams the fp16 activations (Xh) with TMA; one thread of warp 8 issues tcgen05.mma.
// Q4_K's appended correction stages (half(-dmin m) against the per-group sums) read the
// superblock headers from global memory.  K may be split over blockIdx.z (plane * splits +
// split) in whole chunks; split partials go to a workspace through the C tensor map and an
// ordered reduction kernel sums them.
// G groups of 8 dequantising warps (G = 2: the groups take alternate K stages, so two stages'
// hand-off chains overlap), then the MMA, B-load and raw-load warps
template <int G> constexpr int qmm_threads() { return (8 * G + 3) * 32; }
constexpr int QMM_THREADS = qmm_threads<1>();
constexpr int QMM_MAX_NS = 6, QMM_MAX_RAW = 4;

struct QmmArgs {
    const uint8_t* x;  // weights (for the Q4_K correction stages)
    uint32_t K, Kt, nrows, ncols_dst, bn;
    uint32_t ns, nraw, b_stage;  // A/B ring depth, raw ring depth, bytes of a B stage
    uint32_t pre;                // bytes before the B ring: the A ring, or (A in TMEM) what the
                                 // epilogue's staging needs beyond the B ring it reuses
    uint32_t splits, kchunk;     // stages per split (a multiple of 4)
    uint32_t stride_row_x, stride_channel_x, stride_sample_x;  // blocks
    uint32_t nchannels_y, channel_ratio, sample_ratio;
    int tma_c;  // 0: dst stored with plain 16-byte stores (splits == 1 only)
    float* dst;
    uint32_t stride_col_dst, stride_channel_dst, stride_sample_dst;
    unsigned int* err;
    // Q8_0 rows whose stride is not a multiple of 16 bytes (no tensor map can address them): the
    // raw-load warp copies the chunks with cp.async instead; row_bytes = K / 32 * 34
    uint32_t raw_direct, row_bytes;
};

template <uint32_t TY>
constexpr uint32_t qmm_raw_row() { return TY == T_Q4_K ? 144u : 272u; }

// Where a dequantising thread puts the 8 fp16 values (4 words) of 16-byte chunk `chunk` of its
// row's 64-value stage (`rel`: the chunk's index among the thread's four): the SW128 shared-memory
// atom of the A ring, or registers bound for the TMEM A ring (word 4 rel + i = TMEM column 4 rel + i
// of the thread's 16: the fp16 pairs of K elements in order).
struct ASinkSmem {
    uint8_t* atom;
    int r;
    CFI_DEV void put(int chunk, int, uint32_t a, uint32_t b, uint32_t c, uint32_t d) const { st_chunk(atom, r, chunk, a, b, c, d); }
};
struct ASinkRegs {
    uint32_t* w;
    CFI_DEV void put(int, int rel, uint32_t a, uint32_t b, uint32_t c, uint32_t d) const {
        w[4 * rel] = a;
        w[4 * rel + 1] = b;
        w[4 * rel + 2] = c;
        w[4 * rel + 3] = d;
    }
};

// Q8_0 stage s4 of a chunk, block 2 s4 + hh of row r: the block starts 4 s4 + 2 hh bytes into the
// 16-byte aligned 48-byte window at row + 64 s4 + 32 hh.
template <int S4, class Sink>
CFI_DEV void qmm_dequant_q80(const uint8_t* rowp, int hh, const Sink& sink) {
    const uint4* win = reinterpret_cast<const uint4*>(rowp + 64 * S4 + 32 * hh);
    const uint4 c0 = win[0], c1 = win[1], c2 = win[2];
    const uint32_t w[12] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w, c2.x, c2.y, c2.z, c2.w};
    if (hh == 0) {  // d in the low half of word S4, quants from byte 2 of it
        const __half2 d2 = __half2half2(__ushort_as_half((uint16_t)(w[S4] & 0xffffu)));
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint32_t q0 = __funnelshift_r(w[S4 + 2 * c], w[S4 + 2 * c + 1], 16);
            const uint32_t q1 = __funnelshift_r(w[S4 + 2 * c + 1], w[S4 + 2 * c + 2], 16);
            uint32_t v0, v1, v2, v3;
            dequant4(q0, d2, v0, v1);
            dequant4(q1, d2, v2, v3);
            sink.put(c, c, v0, v1, v2, v3);
        }
    } else {  // d in the high half of word S4, quants word-aligned from word S4 + 1
        const __half2 d2 = __half2half2(__ushort_as_half((uint16_t)(w[S4] >> 16)));
#pragma unroll
        for (int c = 0; c < 4; c++) {
            uint32_t v0, v1, v2, v3;
            dequant4(w[S4 + 1 + 2 * c], d2, v0, v1);
            dequant4(w[S4 + 2 + 2 * c], d2, v2, v3);
            sink.put(4 + c, c, v0, v1, v2, v3);
        }
    }
}

// TA: the dequantised A tiles go to a ring in tensor memory (tcgen05.st from the dequantising
// warps, each into its own 32-lane quadrant) and the MMAs read A from there, so shared memory
// carries only B, the raw weights and the epilogue; else to the SW128 A ring in shared memory.
template <uint32_t TY, bool TA, int G>
__global__ void __launch_bounds__(qmm_threads<G>(), 1)
    cfi_qmm_tc(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_b,
               const __grid_constant__ CUtensorMap tmap_c, const QmmArgs a) {
    constexpr uint32_t RAW_ROW = qmm_raw_row<TY>();
    constexpr uint32_t RAW_BYTES = BM * RAW_ROW;  // 18 KB / 34 KB (multiples of 1024)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t NS = a.ns, NR = a.nraw;
    uint8_t* sA = smem;  // the A ring (TA: no A ring; the epilogue's staging from here on)
    uint8_t* sB = sA + a.pre;
    uint8_t* sRaw = sB + NS * a.b_stage;
    uint64_t* full = reinterpret_cast<uint64_t*>(sRaw + NR * RAW_BYTES);
    uint64_t* empty = full + QMM_MAX_NS;
    uint64_t* raw_full = empty + QMM_MAX_NS;
    uint64_t* raw_empty = raw_full + QMM_MAX_RAW;
    uint64_t* done = raw_empty + QMM_MAX_RAW;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* epi_ok = abort_flag + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int QMM_MMA_WARP = 8 * G, QMM_B_WARP = 8 * G + 1;
    const uint32_t bn = a.bn;
    // TMEM: the accumulator in columns [0, bn); with TA the A ring (NS x 32 columns: 64 fp16 per
    // lane and stage) from column acol, the allocation the next power of two
    const uint32_t acol = (bn + 31) / 32 * 32;
    const uint32_t tneed = TA ? acol + NS * (BK / 2) : bn;
    const uint32_t tmem_cols = tneed <= 32 ? 32 : tneed <= 64 ? 64 : tneed <= 128 ? 128 : tneed <= 256 ? 256 : 512;
    const int kmain = (int)(a.K / BK), ktotal = (int)(a.Kt / BK);
    const uint32_t split = blockIdx.z % a.splits, plane = blockIdx.z / a.splits;
    const int k0 = (int)(split * a.kchunk);
    const int k1 = min(ktotal, k0 + (int)a.kchunk);
    const int nsteps = max(0, k1 - k0);
    const int nchunks = k0 < kmain ? (min(k1, kmain) - k0 + 3) / 4 : 0;
    const uint32_t row0 = blockIdx.x * BM, col0 = blockIdx.y * bn;
    const uint32_t wt = plane / a.nchannels_y, zt = plane - wt * a.nchannels_y;
    const uint32_t sx = wt / a.sample_ratio, cx = zt / a.channel_ratio;

    if (tid == 0) {
        for (uint32_t i = 0; i < NS; i++) {
            mbar_init(&full[i], 8 + 1);  // one arrival per dequantizing warp + the B load's expect_tx
            mbar_init(&empty[i], 1);     // tcgen05.commit
        }
        for (uint32_t i = 0; i < NR; i++) {
            mbar_init(&raw_full[i], a.raw_direct ? 32 : 1);  // the raw load's expect_tx, or each lane's copies
            mbar_init(&raw_empty[i], 8 * G);  // every dequantising warp, after its last stage of the chunk
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == QMM_MMA_WARP) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();  // weights and activations may come from the previous kernel

    if (warp < 8 * G) {
        // ================= dequantization (256 threads per group), then the epilogue =================
        // group grp takes stages grp, grp + G, ...; row r, K half hh of each
        const int r = tid & (BM - 1), hh = (tid >> 7) & 1, grp = warp >> 3;
        for (int i = grp; i < nsteps; i += G) {
            const int s = k0 + i;
            const uint32_t slot = (uint32_t)i % NS;
            const int j = i >> 2;  // chunk of the CTA (k0 is a multiple of 4)
            bool ok = true;
            // the group's first stage of a raw chunk waits for the chunk
            if (s < kmain && (i & 3) < G) ok = mbar_wait(&raw_full[j % NR], (uint32_t)(j / NR) & 1, abort_flag);
            if (ok) ok = mbar_wait(&empty[slot], ((uint32_t)(i / NS) & 1) ^ 1, abort_flag);
            if (!ok) {
                if (lane == 0) {
                    cfi_set_error(a.err, 0x800 + (uint32_t)warp);
                    *abort_flag = 1;
                }
                break;
            }
            if (TA) tc_fence_after();  // the MMAs that read this TMEM stage have completed
            uint8_t* atom = sA + slot * A_STAGE;
            uint32_t tw[16];
            const ASinkSmem ss{atom, r};
            const ASinkRegs sr{tw};
            if (s < kmain) {
                const uint8_t* rowp = sRaw + (j % NR) * RAW_BYTES + r * RAW_ROW;
                if (TY == T_Q8_0) {
                    if (TA) {
                        switch (s & 3) {
                        case 0: qmm_dequant_q80<0>(rowp, hh, sr); break;
                        case 1: qmm_dequant_q80<1>(rowp, hh, sr); break;
                        case 2: qmm_dequant_q80<2>(rowp, hh, sr); break;
                        default: qmm_dequant_q80<3>(rowp, hh, sr); break;
                        }
                    } else {
                        switch (s & 3) {
                        case 0: qmm_dequant_q80<0>(rowp, hh, ss); break;
                        case 1: qmm_dequant_q80<1>(rowp, hh, ss); break;
                        case 2: qmm_dequant_q80<2>(rowp, hh, ss); break;
                        default: qmm_dequant_q80<3>(rowp, hh, ss); break;
                        }
                    }
                } else {  // Q4_K: sub-block g = 2 (s % 4) + hh of the chunk's superblock
                    const uint4 h = *reinterpret_cast<const uint4*>(rowp);
                    const uint4 q0 = *reinterpret_cast<const uint4*>(rowp + 16 + 32 * (s & 3));
                    const uint4 q1 = *reinterpret_cast<const uint4*>(rowp + 32 + 32 * (s & 3));
                    const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                    const uint32_t sc[3] = {h.y, h.z, h.w};
                    const float dd = __half2float(__ushort_as_half((uint16_t)(h.x & 0xffffu)));
                    const int g = 2 * (s & 3) + hh;
                    const int scv = g < 4 ? (scale_byte(sc, g) & 63)
                                          : ((scale_byte(sc, g + 4) & 0xF) | ((scale_byte(sc, g - 4) >> 6) << 4));
                    // the reference's tile loader stores half(d * sc) (refs.rs:709-712)
                    const __half2 d2 = __half2half2(__float2half_rn(dd * (float)scv));
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        uint32_t v0, v1, v2, v3;
                        dequant4_u4(q[2 * c], 4 * hh, d2, v0, v1);
                        dequant4_u4(q[2 * c + 1], 4 * hh, d2, v2, v3);
                        if (TA)
                            sr.put(4 * hh + c, c, v0, v1, v2, v3);
                        else
                            ss.put(4 * hh + c, c, v0, v1, v2, v3);
                    }
                }
            } else if constexpr (TY == T_Q4_K) {  // Q4_K correction stage: A[r][K + g] = half(-dmin * m_g) (refs.rs:712)
                const int g0 = (s - kmain) * BK;
                const int ngroups = (int)(a.K / 32);
                const uint32_t row = row0 + r;
                const uint8_t* rowg = a.x + ((size_t)sx * a.stride_sample_x + (size_t)cx * a.stride_channel_x +
                                             (size_t)min(row, a.nrows - 1) * a.stride_row_x) * Q4_K_BYTES;
                // the four superblock headers of this thread, all loads issued before any use
                uint4 hdr[4];
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const int gbase = g0 + 8 * (4 * hh + t);
                    hdr[t] = (row < a.nrows && gbase < ngroups)
                                 ? __ldg(reinterpret_cast<const uint4*>(rowg + (size_t)(gbase / 8) * Q4_K_BYTES))
                                 : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const int sbl = 4 * hh + t;
                    const int gbase = g0 + 8 * sbl;
                    const uint32_t hw0 = hdr[t].x, hs[3] = {hdr[t].y, hdr[t].z, hdr[t].w};
                    const float dmin = __half2float(__ushort_as_half((uint16_t)(hw0 >> 16)));
                    uint32_t v[4];
#pragma unroll
                    for (int p = 0; p < 4; p++) {
                        uint32_t hv[2];
#pragma unroll
                        for (int e = 0; e < 2; e++) {
                            const int gg = 2 * p + e;
                            const int mv = gg < 4 ? (scale_byte(hs, gg + 4) & 63)
                                                  : ((scale_byte(hs, gg + 4) >> 4) | ((scale_byte(hs, gg) >> 6) << 4));
                            hv[e] = gbase < ngroups ? (uint32_t)__half_as_ushort(__float2half_rn(-dmin * (float)mv)) : 0u;
                        }
                        v[p] = hv[0] | (hv[1] << 16);
                    }
                    if (TA)
                        sr.put(sbl, t, v[0], v[1], v[2], v[3]);
                    else
                        ss.put(sbl, t, v[0], v[1], v[2], v[3]);
                }
            }

            if (TA) {
                // lanes 32 (warp % 4) .. + 31 = rows; columns acol + 32 slot + 16 hh .. + 15
                tmem_st16(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + acol + slot * (BK / 2) + 16 * hh, tw);
                tmem_st_wait();
                tc_fence_before();
            } else {
                fence_proxy_async_smem();  // this thread's A-tile writes, visible to the tensor core
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&full[slot]);
                // the group's last stage of the chunk releases it
                const int last = min(4 * j + 3, min(nsteps - 1, kmain - 1 - k0));
                if (s < kmain && i + G > last) mbar_arrive(&raw_empty[j % NR]);
            }
        }
        if (warp >= 8) goto exit_roles;  // the second group has no epilogue part
        // ================= epilogue: TMEM -> shared -> TMA stores =================
        if (tid == 0) {
            bool got = false;
            if (!*abort_flag) {
                got = mbar_wait(done, 0, abort_flag);
                if (!got) {
                    cfi_set_error(a.err, 0x900);
                    *abort_flag = 1;
                }
            }
            *epi_ok = got ? 1 : 0;
        }
        named_bar_sync(1, 256);
        tc_fence_after();
        if (*epi_ok && a.tma_c) {
            // every MMA has completed: the A/B rings hold the 8 KB per-warp staging buffers
            float* tbuf = reinterpret_cast<float*>(sA) + warp * 2048;
            if (a.splits > 1)  // raw partial sums into the split-K workspace (plane, split)
                tmem_tile_tma_store(tmem, warp, lane, 8, bn, tbuf, &tmap_c, (int)row0, (int)col0, (int)plane, (int)split,
                                    [](float v) { return v; });
            else
                tmem_tile_tma_store(tmem, warp, lane, 8, bn, tbuf, &tmap_c, (int)row0, (int)col0, (int)zt, (int)wt,
                                    [](float v) { return v; });
        } else if (*epi_ok) {
            float* dst = a.dst + (size_t)wt * a.stride_sample_dst + (size_t)zt * a.stride_channel_dst;
            float* buf = reinterpret_cast<float*>(sA) + warp * 1024;
            const bool vec = (a.stride_col_dst & 3u) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
            tmem_tile_store(tmem, warp, lane, 8, bn, buf, [&](uint32_t c, uint32_t rr, float4 f) {
                const uint32_t col = col0 + c, row = row0 + rr;
                if (col >= a.ncols_dst || row >= a.nrows) return;
                float* p = dst + (size_t)col * a.stride_col_dst + row;
                if (vec && row + 3 < a.nrows) {
                    *reinterpret_cast<float4*>(p) = f;
                } else {
                    p[0] = f.x;
                    if (row + 1 < a.nrows) p[1] = f.y;
                    if (row + 2 < a.nrows) p[2] = f.z;
                    if (row + 3 < a.nrows) p[3] = f.w;
                }
            });
        }
    } else if (warp == QMM_MMA_WARP) {
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(BM, bn, 0);
            for (int i = 0; i < nsteps; i++) {
                const uint32_t slot = (uint32_t)i % NS;
                if (!mbar_wait(&full[slot], (uint32_t)(i / NS) & 1, abort_flag)) {
                    cfi_set_error(a.err, 0xa00 + slot);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t abase = smem_u32(sA + slot * A_STAGE), bbase = smem_u32(sB + slot * a.b_stage);
#pragma unroll
                for (int k = 0; k < BK / 16; k++) {
                    if (TA)  // A: 8 TMEM columns (16 fp16 per lane) per K step
                        mma_f16_ts(tmem, tmem + acol + slot * (BK / 2) + 8 * k, sw128_kmajor_desc(bbase + 32 * k), idesc,
                                   (i > 0 || k > 0) ? 1u : 0u);
                    else
                        mma_f16(tmem, sw128_kmajor_desc(abase + 32 * k), sw128_kmajor_desc(bbase + 32 * k), idesc,
                                (i > 0 || k > 0) ? 1u : 0u);
                }
                mma_commit(&empty[slot]);
            }
            mma_commit(done);  // also after a failure: `done` then tracks the MMAs already issued
        }
        __syncwarp();
    } else if (warp == QMM_B_WARP) {
        if (lane == 0) {
            prefetch_tmap(&tmap_b);
            const uint32_t bytes = bn * BK * 2;
            for (int i = 0; i < nsteps; i++) {
                const uint32_t slot = (uint32_t)i % NS;
                if (!mbar_wait(&empty[slot], ((uint32_t)(i / NS) & 1) ^ 1, abort_flag)) {
                    cfi_set_error(a.err, 0xb00 + slot);
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full[slot], bytes);
                tma_load_3d(sB + slot * a.b_stage, &tmap_b, (k0 + i) * BK, (int)col0, (int)plane, &full[slot]);
            }
        }
        __syncwarp();
    } else if (warp == 8 * G + 2) {
        // ================= raw weight chunks =================
        if (TY == T_Q8_0 && a.raw_direct) {
            // each lane copies rows lane, lane + 32, ... of a chunk with cp.async: 16-byte pieces
            // where the row's chunk starts 16-byte aligned, else 8-byte pieces (rows are 8-byte
            // aligned); a chunk past K (K not a multiple of 256) stops at the row's end, a
            // multiple of 8 bytes (K % 128 == 0); rows past the matrix copy its last row
            const uint8_t* base = a.x + ((size_t)sx * a.stride_sample_x + (size_t)cx * a.stride_channel_x) * Q8_0_BYTES;
            const size_t rstride = (size_t)a.stride_row_x * Q8_0_BYTES;
            for (int j = 0; j < nchunks; j++) {
                const uint32_t rs = (uint32_t)j % NR;
                if (!__all_sync(0xffffffffu, mbar_wait(&raw_empty[rs], ((uint32_t)(j / NR) & 1) ^ 1, abort_flag))) {
                    if (lane == 0) {
                        cfi_set_error(a.err, 0xc00 + rs);
                        *abort_flag = 1;
                    }
                    break;
                }
                const uint32_t cbyte = (uint32_t)(k0 / 4 + j) * RAW_ROW;
                const uint32_t cb = min(RAW_ROW, a.row_bytes - cbyte);
                for (uint32_t r = lane; r < BM; r += 32) {
                    const uint8_t* src = base + (size_t)min(row0 + r, a.nrows - 1) * rstride + cbyte;
                    const uint32_t d = smem_u32(sRaw + rs * RAW_BYTES + r * RAW_ROW);
                    uint32_t o = 0;
                    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0)
                        for (; o + 16 <= cb; o += 16) cp_async16_cg(d + o, src + o);
                    for (; o < cb; o += 8) cp_async8_ca(d + o, src + o);
                }
                cp_async_mbar_arrive_noinc(&raw_full[rs]);
            }
            asm volatile("cp.async.wait_all;" ::: "memory");  // nothing in flight when the CTA ends
        } else if (lane == 0) {
            prefetch_tmap(&tmap_w);
            constexpr int XU = TY == T_Q4_K ? 144 : 136;  // chunk width in tensor-map elements (u8 / u16)
            for (int j = 0; j < nchunks; j++) {
                const uint32_t rs = (uint32_t)j % NR;
                if (!mbar_wait(&raw_empty[rs], ((uint32_t)(j / NR) & 1) ^ 1, abort_flag)) {
                    cfi_set_error(a.err, 0xc00 + rs);
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&raw_full[rs], RAW_BYTES);
                tma_load_4d(sRaw + rs * RAW_BYTES, &tmap_w, (k0 / 4 + j) * XU, (int)row0, (int)cx, (int)sx, &raw_full[rs]);
            }
        }
        __syncwarp();
    }
exit_roles:
    tc_fence_before();
    __syncthreads();
    if (warp == QMM_MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
}

// block_q8_1_mmq -> fp16 K-major rows: Xh[plane][col][k] = fp16(q * d) for k < K; for DS4
// (Q4_K) Xh[plane][col][K + g] = s_g (the half float sum of group g), zero up to Kt.
// One warp per (column, 128-value block); lane l handles values 4l..4l+3.
template <int DS4, int SUMS>
CFI_DEV void x_to_f16(uint32_t bx, uint32_t plane, const uint8_t* __restrict__ y, __half* __restrict__ xh, uint32_t K,
                      uint32_t Kt, uint32_t ncols, uint32_t ncols_y, uint32_t nchannels_y, uint32_t stride_channel_y,
                      uint32_t stride_sample_y) {
    const uint32_t warp_g = (bx * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const uint32_t nkb = K / 128;
    if (warp_g >= ncols * nkb) return;
    const uint32_t col = warp_g / nkb, kb = warp_g - col * nkb;
    const uint32_t wt = plane / nchannels_y, zt = plane - wt * nchannels_y;
    const uint8_t* yb = y + ((size_t)wt * stride_sample_y + (size_t)zt * stride_channel_y) * 4 +
                        ((size_t)kb * ncols_y + col) * MMQ_BLOCK_BYTES;
    const uint32_t qv = *reinterpret_cast<const uint32_t*>(yb + 16 + 4 * lane);
    float d;
    uint32_t sbits = 0;
    if (DS4) {
        const uint32_t ds = *reinterpret_cast<const uint32_t*>(yb + 4 * (lane >> 3));
        d = h2f_bits((uint16_t)(ds & 0xffffu));
        sbits = ds >> 16;
    } else {
        d = *reinterpret_cast<const float*>(yb + 4 * (lane >> 3));
    }
    const float f0 = (float)(int8_t)(qv & 0xff) * d, f1 = (float)(int8_t)((qv >> 8) & 0xff) * d;
    const float f2 = (float)(int8_t)((qv >> 16) & 0xff) * d, f3 = (float)(int8_t)(qv >> 24) * d;
    __half2 lo = __floats2half2_rn(f0, f1), hi = __floats2half2_rn(f2, f3);
    __half* row = xh + ((size_t)plane * ncols + col) * Kt;
    uint2 out = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
    *reinterpret_cast<uint2*>(row + kb * 128 + 4 * lane) = out;
    if (SUMS) {
        if ((lane & 7) == 0) row[K + kb * 4 + (lane >> 3)] = __ushort_as_half((uint16_t)sbits);
        // zero the padding of the appended columns once (block kb == 0 of each column)
        if (kb == 0)
            for (uint32_t k = K + K / 32 + lane; k < Kt; k += 32) row[k] = __float2half(0.0f);
    }
}

template <int DS4, int SUMS>
__global__ void __launch_bounds__(256)
    cfi_mmq_x_to_f16(const uint8_t* __restrict__ y, __half* __restrict__ xh, uint32_t K, uint32_t Kt, uint32_t ncols,
                     uint32_t ncols_y, uint32_t nchannels_y, uint32_t stride_channel_y, uint32_t stride_sample_y) {
    pdl_launch_dependents();
    pdl_wait();
    x_to_f16<DS4, SUMS>(blockIdx.x, blockIdx.y, y, xh, K, Kt, ncols, ncols_y, nchannels_y, stride_channel_y, stride_sample_y);
}

// Weights -> fp16 K-major rows: Wh[xplane][row][k].  Q8_0: fp16(q * d).  Q4_K: fp16(q *
// half(d * sc)) and, in the appended columns K + g, half(-dmin * m_g) (the terms the fused kernel
// builds in shared memory; refs.rs:709-712), zero up to Kt.  One thread per weight block
// (Q8_0: 32 values, Q4_K: 256 values), consecutive threads on consecutive blocks of a row.
// Q4_0 / Q5_0 / Q6_K blocks are only 2-byte aligned: halfword loads.
CFI_DEV uint32_t ldg_w2(const uint8_t* p) {  // 4 bytes at a 2-byte-aligned address
    const unsigned short* h = reinterpret_cast<const unsigned short*>(p);
    return (uint32_t)__ldg(h) | ((uint32_t)__ldg(h + 1) << 16);
}

template <uint32_t TY>
CFI_DEV void w_to_f16(uint32_t bx, uint32_t xp, const uint8_t* __restrict__ x, __half* __restrict__ wh, uint32_t K,
                      uint32_t Kt, uint32_t nrows, uint32_t srx, uint32_t nch_x, uint32_t scx, uint32_t ssx) {
    constexpr uint32_t QKB = mmq_qk<TY>();
    const uint32_t nb = K / QKB;
    const uint64_t t = (uint64_t)bx * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)nrows * nb) return;
    const uint32_t row = (uint32_t)(t / nb), b = (uint32_t)(t - (uint64_t)row * nb);
    const uint32_t sx = xp / nch_x, cx = xp - sx * nch_x;
    __half* out = wh + ((size_t)xp * nrows + row) * Kt;
    const uint8_t* blk = x + ((size_t)sx * ssx + (size_t)cx * scx + (size_t)row * srx + b) * mmq_bb<TY>();
    if (TY == T_Q4_0 || TY == T_Q5_0) {
        // Q4_0: q = nibble - 8; Q5_0: q = (nibble | qh bit << 4) - 16; values 0..15 from the low
        // nibbles of qs, 16..31 from the high; fp16(q * d)
        const __half2 d2 = __half2half2(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(blk))));
        const uint32_t qh = TY == T_Q5_0 ? ldg_w2(blk + 2) : 0u;
        const uint8_t* qs = blk + (TY == T_Q5_0 ? 6 : 2);
        uint32_t v[16];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t w = ldg_w2(qs + 4 * j);
#pragma unroll
            for (int hi = 0; hi < 2; hi++) {
                uint32_t n = (w >> (4 * hi)) & 0x0F0F0F0Fu;
                if (TY == T_Q5_0) {
                    const uint32_t bits = qh >> (16 * hi + 4 * j);
                    n |= ((bits & 1u) << 4) | ((bits & 2u) << 11) | ((bits & 4u) << 18) | ((bits & 8u) << 25);
                }
                const uint32_t q = __vsub4(n, TY == T_Q5_0 ? 0x10101010u : 0x08080808u);
                uint32_t lo, hh;
                dequant4(q, d2, lo, hh);
                v[8 * hi + 2 * j] = lo;
                v[8 * hi + 2 * j + 1] = hh;
            }
        }
        uint4* o = reinterpret_cast<uint4*>(out + (size_t)b * 32);
#pragma unroll
        for (int i = 0; i < 4; i++) o[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else if (TY == T_Q6_K) {
        // q = (ql nibble | 2 qh bits << 4) - 32, fp16(d * (sc * q)) with an int8 scale per 16 values
        const float d = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(blk + 208))));
        uint4* o = reinterpret_cast<uint4*>(out + (size_t)b * 256);
#pragma unroll 1
        for (int g = 0; g < 8; g++) {
            const int h = g >> 2, quad = g & 3;
            const uint32_t scw = __ldg(reinterpret_cast<const unsigned short*>(blk + 192 + 2 * g));
            const int sc0 = (int)(int8_t)(scw & 0xffu), sc1 = (int)(int8_t)(scw >> 8);
            uint32_t v[16];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t lw = (ldg_w2(blk + 64 * h + 32 * (quad & 1) + 4 * j) >> (4 * (quad >> 1))) & 0x0F0F0F0Fu;
                const uint32_t hw = ((ldg_w2(blk + 128 + 32 * h + 4 * j) >> (2 * quad)) & 0x03030303u) << 4;
                const uint32_t q = lw | hw;
                const int sc = j < 4 ? sc0 : sc1;
                float f[4];
#pragma unroll
                for (int e = 0; e < 4; e++) f[e] = d * (float)(sc * ((int)((q >> (8 * e)) & 0xffu) - 32));
                const __half2 a = __floats2half2_rn(f[0], f[1]), c = __floats2half2_rn(f[2], f[3]);
                v[2 * j] = h2_bits(a);
                v[2 * j + 1] = h2_bits(c);
            }
#pragma unroll
            for (int i = 0; i < 4; i++) o[g * 4 + i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
    } else if (TY == T_Q5_K) {
        // Q4_K's layout plus one high bit per value (qh bit g of byte i): q in 0..31
        const uint4* b4 = reinterpret_cast<const uint4*>(blk);
        const uint4 h = __ldg(b4);
        const uint32_t hs[3] = {h.y, h.z, h.w};
        const float dd = __half2float(__ushort_as_half((uint16_t)(h.x & 0xffffu)));
        const float dmin = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
        const uint4 qh0 = __ldg(b4 + 1), qh1 = __ldg(b4 + 2);
        const uint32_t qh[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
        uint4* o = reinterpret_cast<uint4*>(out + (size_t)b * 256);
        uint32_t corr[4];
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 q0 = __ldg(b4 + 3 + 2 * c), q1 = __ldg(b4 + 4 + 2 * c);
            const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            uint32_t hv[2];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int g = 2 * c + e;
                int scv, mv;
                if (g < 4) {
                    scv = scale_byte(hs, g) & 63;
                    mv = scale_byte(hs, g + 4) & 63;
                } else {
                    scv = (scale_byte(hs, g + 4) & 0xF) | ((scale_byte(hs, g - 4) >> 6) << 4);
                    mv = (scale_byte(hs, g + 4) >> 4) | ((scale_byte(hs, g) >> 6) << 4);
                }
                const __half2 d2 = __half2half2(__float2half_rn(dd * (float)scv));
                hv[e] = (uint32_t)__half_as_ushort(__float2half_rn(-dmin * (float)mv));
#pragma unroll
                for (int i = 0; i < 8; i += 2) {
                    uint32_t a0, a1, b0, b1;
                    const uint32_t u0 = ((q[i] >> (4 * e)) & 0x0F0F0F0Fu) | (((qh[i] >> g) & 0x01010101u) << 4);
                    const uint32_t u1 = ((q[i + 1] >> (4 * e)) & 0x0F0F0F0Fu) | (((qh[i + 1] >> g) & 0x01010101u) << 4);
                    dequant4_ub(u0, d2, a0, a1);
                    dequant4_ub(u1, d2, b0, b1);
                    o[g * 4 + i / 2] = make_uint4(a0, a1, b0, b1);
                }
            }
            corr[c] = hv[0] | (hv[1] << 16);
        }
        *reinterpret_cast<uint4*>(out + K + (size_t)b * 8) = make_uint4(corr[0], corr[1], corr[2], corr[3]);
        if (b == 0)  // the padding of the appended columns, once per row
            for (uint32_t k = K + K / 32; k < Kt; k++) out[k] = __float2half(0.0f);
    } else if (TY == T_Q8_0) {
        const uint8_t* blk = x + ((size_t)sx * ssx + (size_t)cx * scx + (size_t)row * srx + b) * Q8_0_BYTES;
        const uint32_t* wa = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(blk) & ~(uintptr_t)3);
        const uint32_t sh = (uint32_t)(reinterpret_cast<uintptr_t>(blk) & 3) * 8;  // 0 or 16
        // the 9 aligned words that hold the 34-byte block (the bytes outside it share a word
        // with block bytes, so no page is touched that the block does not touch)
        uint32_t w[9];
#pragma unroll
        for (int i = 0; i < 9; i++) w[i] = __ldg(wa + i);
        const uint16_t dbits = (uint16_t)(__funnelshift_r(w[0], w[1], sh) & 0xffffu);
        const __half2 d2 = __half2half2(__ushort_as_half(dbits));
        uint32_t v[16];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t q = __funnelshift_r(w[i], w[i + 1], sh + 16);  // quants start 2 bytes in
            uint32_t lo, hi;
            dequant4(sh + 16 >= 32 ? w[i + 1] : q, d2, lo, hi);
            v[2 * i] = lo;
            v[2 * i + 1] = hi;
        }
        uint4* o = reinterpret_cast<uint4*>(out + (size_t)b * 32);
#pragma unroll
        for (int i = 0; i < 4; i++) o[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
        const uint4* blk = reinterpret_cast<const uint4*>(x + ((size_t)sx * ssx + (size_t)cx * scx + (size_t)row * srx + b) * Q4_K_BYTES);
        const uint4 h = __ldg(blk);
        const uint32_t hs[3] = {h.y, h.z, h.w};
        const float dd = __half2float(__ushort_as_half((uint16_t)(h.x & 0xffffu)));
        const float dmin = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
        uint4* o = reinterpret_cast<uint4*>(out + (size_t)b * 256);
        uint32_t corr[4];
#pragma unroll
        for (int c = 0; c < 4; c++) {  // 32 bytes of nibbles: sub-blocks 2c (low) and 2c+1 (high)
            const uint4 q0 = __ldg(blk + 1 + 2 * c), q1 = __ldg(blk + 2 + 2 * c);
            const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            uint32_t hv[2];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int g = 2 * c + e;
                int scv, mv;
                if (g < 4) {
                    scv = scale_byte(hs, g) & 63;
                    mv = scale_byte(hs, g + 4) & 63;
                } else {
                    scv = (scale_byte(hs, g + 4) & 0xF) | ((scale_byte(hs, g - 4) >> 6) << 4);
                    mv = (scale_byte(hs, g + 4) >> 4) | ((scale_byte(hs, g) >> 6) << 4);
                }
                const __half2 d2 = __half2half2(__float2half_rn(dd * (float)scv));
                hv[e] = (uint32_t)__half_as_ushort(__float2half_rn(-dmin * (float)mv));
#pragma unroll
                for (int i = 0; i < 8; i += 2) {
                    uint32_t a0, a1, b0, b1;
                    dequant4_u4(q[i], 4 * e, d2, a0, a1);
                    dequant4_u4(q[i + 1], 4 * e, d2, b0, b1);
                    o[g * 4 + i / 2] = make_uint4(a0, a1, b0, b1);
                }
            }
            corr[c] = hv[0] | (hv[1] << 16);
        }
        *reinterpret_cast<uint4*>(out + K + (size_t)b * 8) = make_uint4(corr[0], corr[1], corr[2], corr[3]);
        if (b == 0)  // the padding of the appended columns, once per row
            for (uint32_t k = K + K / 32; k < Kt; k++) out[k] = __float2half(0.0f);
    }
}

// Both pre-passes in one launch: grid.y < planes converts activation plane y, the rest weight
// plane y - planes.  Lets the GEMM launch at once (programmatic dependent launch); it waits for
// this grid before its first tensor load.
template <uint32_t TY>
__global__ void __launch_bounds__(256)
    cfi_mmq_prepass(const uint8_t* __restrict__ y, __half* __restrict__ xh, const uint8_t* __restrict__ x,
                    __half* __restrict__ wh, uint32_t K, uint32_t Kt, uint32_t ncols, uint32_t ncols_y,
                    uint32_t nchannels_y, uint32_t stride_channel_y, uint32_t stride_sample_y, uint32_t planes,
                    uint32_t nrows, uint32_t srx, uint32_t nch_x, uint32_t scx, uint32_t ssx) {
    pdl_launch_dependents();
    pdl_wait();
    if (blockIdx.y < planes)
        x_to_f16<mmq_ds4<TY>(), mmq_corr<TY>()>(blockIdx.x, blockIdx.y, y, xh, K, Kt, ncols, ncols_y, nchannels_y, stride_channel_y,
                                       stride_sample_y);
    else
        w_to_f16<TY>(blockIdx.x, blockIdx.y - planes, x, wh, K, Kt, nrows, srx, nch_x, scx, ssx);
}

// ---- host side ----
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled encode_fn() {
    static PFN_encodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

// Activation scratch (fp16 copy of X, and the fp16 weights of the pre-pass path): the calling
// stream's own buffer (stream_state.cpp), grown outside stream capture only.
int scratch_for(size_t bytes, cudaStream_t stream, void** out) {
    int err = 0;
    *out = cfi_stream_buffer(CFI_BUF_MMQ_SCRATCH, bytes, stream, &err);
    return *out ? 0 : (err ? err : (int)cudaErrorMemoryAllocation);
}

unsigned int* device_error_ptr() {
    static CfiSymbolPtr<unsigned int> p;
    return p.get(g_cfi_device_error);
}

// Tile width: the fewest tiles of at most 256 columns, balanced (631 columns -> 3 x 224).
// (a multiple of 32 when there are several: the epilogue writes whole 32-column chunks).
uint32_t tile_n(uint32_t ncols_dst) {
    const uint32_t tiles = (ncols_dst + 255) / 256;
    const uint32_t per = (ncols_dst + tiles - 1) / tiles;
    return tiles > 1 ? (per + 31) / 32 * 32 : (per + 15) / 16 * 16;
}

// Q8_0 whose raw chunks no tensor map can address (a row stride of 4 mod 8 blocks, or K not a
// multiple of 256) but whose rows, channels and samples start 8-byte aligned and whose K is a
// multiple of 128 (the last chunk a multiple of 8 bytes): the raw-load warp copies with cp.async.
// K = 896 (28-block rows of the Qwen2.5-0.5B projections) is the case.  Only with
// CFI_MMQ_RAW_DIRECT=1: on config 3's 4864 x 896 x 631 it measured 19.5 us against 14.5 us for the
// fp16 weight pre-pass and the plain tensor-core GEMM (the fused kernel's dequantising chain, not
// the pre-pass, limits a CTA that runs 14 K stages).
inline bool qmm_raw_direct(uint32_t K, uint32_t srx, uint32_t scx, uint32_t ssx, uint32_t nch_x, uint32_t ns_x) {
    const char* e = getenv("CFI_MMQ_RAW_DIRECT");
    if (!(e && strcmp(e, "1") == 0)) return false;
    if (K % 256 == 0 && srx % 8 == 0 && (nch_x == 1 || scx % 8 == 0) && (ns_x == 1 || ssx % 8 == 0)) return false;
    return K % 128 == 0 && srx % 4 == 0 && (nch_x == 1 || scx % 4 == 0) && (ns_x == 1 || ssx % 4 == 0);
}

// The fused quantized GEMM applies when the raw weight chunks can be staged: TMA when every row,
// channel and sample starts 16-byte aligned -- Q4_K (144-byte superblocks) always, Q8_0 (34-byte
// blocks) when K and the block strides are multiples of 256 values / 8 blocks -- else, on request,
// Q8_0 by cp.async (qmm_raw_direct).  CFI_MMQ_FUSED=0 off.
template <uint32_t TY>
bool qmm_applicable(const uint8_t* x, uint32_t K, uint32_t srx, uint32_t scx, uint32_t ssx, uint32_t nch_x,
                    uint32_t ns_x) {
    if (TY != T_Q4_K && TY != T_Q8_0) return false;
    const char* e = getenv("CFI_MMQ_FUSED");
    if (e && strcmp(e, "0") == 0) return false;
    if (reinterpret_cast<uintptr_t>(x) & 15) return false;
    if (TY == T_Q4_K) return K % 256 == 0;
    if (K % 256 == 0 && srx % 8 == 0 && (nch_x == 1 || scx % 8 == 0) && (ns_x == 1 || ssx % 8 == 0)) return true;
    return qmm_raw_direct(K, srx, scx, ssx, nch_x, ns_x);
}

constexpr uint32_t QMM_SMEM_LIMIT = 232448;  // 227 KB of dynamic shared memory per CTA

// Activations -> Xh (pre-pass), then cfi_qmm_tc (+ the split-K reduction).  Returns a CUDA error.
template <uint32_t TY>
int launch_qmm(const uint8_t* x, const uint8_t* y, float* dst, void* xh, uint32_t K, uint32_t Kt, uint32_t nrows,
               uint32_t ncols_dst, uint32_t srx, uint32_t ncols_y, uint32_t scd, uint32_t chr, uint32_t nch, uint32_t scx,
               uint32_t scy, uint32_t scdst, uint32_t smr, uint32_t ns, uint32_t ssx, uint32_t ssy, uint32_t ssd,
               cudaStream_t stream, bool may_allocate = true) {
    PFN_encodeTiled enc = encode_fn();
    if (!enc) return (int)cudaErrorNotSupported;
    const char* ep = getenv("CFI_PDL");
    const bool pdl = !(ep && strcmp(ep, "0") == 0);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    const uint32_t planes = nch * ns, nch_x = nch / chr, ns_x = ns / smr;
    // 1. activations -> fp16 K-major
    {
        const uint32_t warps = ncols_dst * (K / 128);
        cudaLaunchConfig_t c = {};
        c.gridDim = dim3((warps * 32 + 255) / 256, planes, 1);
        c.blockDim = dim3(256, 1, 1);
        c.stream = stream;
        c.attrs = at;
        c.numAttrs = pdl ? 1 : 0;
        cudaError_t e = TY == T_Q4_K
                            ? cudaLaunchKernelEx(&c, cfi_mmq_x_to_f16<1, 1>, y, static_cast<__half*>(xh), K, Kt, ncols_dst,
                                                 ncols_y, nch, scy, ssy)
                            : cudaLaunchKernelEx(&c, cfi_mmq_x_to_f16<0, 0>, y, static_cast<__half*>(xh), K, Kt, ncols_dst,
                                                 ncols_y, nch, scy, ssy);
        if (e != cudaSuccess) return (int)e;
    }
    // 2. tensor maps: raw weights (4-D: chunk bytes, rows, channels, samples), Xh, dst
    constexpr uint32_t RAW_ROW = qmm_raw_row<TY>();
    constexpr uint32_t BB = TY == T_Q4_K ? Q4_K_BYTES : Q8_0_BYTES;
    CUtensorMap tw, tb, tc;
    const bool raw_direct = TY == T_Q8_0 && qmm_raw_direct(K, srx, scx, ssx, nch_x, ns_x);
    if (raw_direct) {
        memset(&tw, 0, sizeof tw);  // not read: the raw chunks are copied with cp.async
    } else {
        const uint32_t es = TY == T_Q4_K ? 1 : 2;
        const cuuint64_t rowb = (cuuint64_t)srx * BB;
        const cuuint64_t chb = nch_x > 1 ? (cuuint64_t)scx * BB : rowb * nrows;
        const cuuint64_t smb = ns_x > 1 ? (cuuint64_t)ssx * BB : chb * nch_x;
        cuuint64_t dw[4] = {(cuuint64_t)(K / 256) * RAW_ROW / es, nrows, nch_x, ns_x};
        cuuint64_t sw[3] = {rowb, chb, smb};
        cuuint32_t bw[4] = {RAW_ROW / es, (cuuint32_t)BM, 1, 1}, ew[4] = {1, 1, 1, 1};
        if (enc(&tw, TY == T_Q4_K ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 4,
                const_cast<uint8_t*>(x), dw, sw, bw, ew, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    }
    constexpr uint32_t RAW_BYTES = BM * qmm_raw_row<TY>();
    // Column tile and ring depths.  Default: tile_n's tile, one CTA per SM with 3-4 A/B stages and
    // up to 4 raw slots.  When that needs more than one wave, the widest tile of at most 160
    // columns whose grid fits two CTAs per SM is used instead, with 2-deep rings (about 110 KB of
    // shared memory, so two CTAs share an SM and hide each other's latencies): Q4_K 8960 x 1536 x
    // 631, 210 CTAs in 1.4 waves -> 280 in one, measured 45.7 -> 32.5 us.  CFI_QMM_BN (a multiple of
    // 16, 16..256), CFI_QMM_STAGES and CFI_QMM_RAW (2..4) override.
    auto env_in = [](const char* n, uint32_t dflt, uint32_t lo, uint32_t hi) {
        const char* e = getenv(n);
        const int v = e ? atoi(e) : 0;
        return (v >= (int)lo && v <= (int)hi && (v % 16 == 0 || hi <= 16)) ? (uint32_t)v : dflt;
    };
    const uint32_t rtiles = (nrows + BM - 1) / BM;
    // CFI_QMM_TMEM_A=0: the dequantised A tiles through shared memory instead of tensor memory
    // (in TMEM the A ring costs no shared memory)
    const char* eta = getenv("CFI_QMM_TMEM_A");
    const bool ta = !(eta && strcmp(eta, "0") == 0);
    uint32_t bn = tile_n(ncols_dst), ns_dflt = bn <= 128 ? 4 : 3, raw_dflt = QMM_MAX_RAW;
    if ((uint64_t)rtiles * ((ncols_dst + bn - 1) / bn) * planes > (uint64_t)sms) {
        for (uint32_t ct = (ncols_dst + 159) / 160; ct <= (ncols_dst + 63) / 64; ct++) {
            const uint32_t b2 = ((ncols_dst + ct - 1) / ct + 15) / 16 * 16;
            const size_t sm2 = 1024 + 2 * (size_t)(A_STAGE + b2 * BK * 2) + 256 + 2 * (size_t)RAW_BYTES;
            if ((uint64_t)rtiles * ct * planes <= 2 * (uint64_t)sms && sm2 <= QMM_SMEM_LIMIT / 2 - 3 * 1024) {
                bn = b2;
                ns_dflt = 2;
                raw_dflt = 2;
                break;
            }
        }
    }
    bn = env_in("CFI_QMM_BN", bn, 16, 256);
    {
        cuuint64_t gdim[3] = {Kt, ncols_dst, planes};
        cuuint64_t gstride[2] = {(cuuint64_t)Kt * 2, (cuuint64_t)Kt * 2 * ncols_dst};
        cuuint32_t box[3] = {BK, bn, 1}, estr[3] = {1, 1, 1};
        if (enc(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, xh, gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    memset(&tc, 0, sizeof tc);
    bool tma_c = (scd % 4) == 0 && (nch == 1 || scdst % 4 == 0) && (ns == 1 || ssd % 4 == 0) &&
                 (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    // 3. split K (whole 256-value chunks) when the output tiles fill under half the SMs
    const uint32_t ktotal = Kt / BK;
    uint32_t splits = 1, kchunk = (ktotal + 3) / 4 * 4;
    const uint64_t tiles = (uint64_t)((nrows + BM - 1) / BM) * ((ncols_dst + bn - 1) / bn) * planes;
    float* ws = nullptr;
    const uint32_t ld_ws = (nrows + 3) / 4 * 4;
    const char* es = getenv("CFI_GEMM_SPLITK");
    // Split K in whole 256-value chunks, down to one chunk per split: up to two CTAs per SM on
    // 2-deep rings when those fit in half the shared memory, else up to one (batch-64 Q4_K products
    // 1536 x 1536: 14.0 -> 9.6 us, 256 x 1536: 13.5 -> 9.2, 8960 x 1536: 18.8 -> 16.4, 1536 x 8960:
    // 21.8 -> 20.3; at 631 columns, one CTA per SM, 1536 x 1536: 18.1 -> 16.4, 256 x 1536: 16.2 -> 11.9).
    // CFI_QMM_SPLIT_CTAS=1 restores the coarser split (at least 8 stages per split, one CTA per SM).
    const bool fine = env_in("CFI_QMM_SPLIT_CTAS", 2, 1, 2) == 2;
    const uint32_t per_sm =
        fine && 1024 + 2 * (size_t)(A_STAGE + bn * BK * 2) + 256 + 2 * (size_t)RAW_BYTES <= QMM_SMEM_LIMIT / 2 - 3 * 1024 ? 2 : 1;
    // (split K needs a device workspace: never on the allocation-free entry point)
    if (may_allocate && tma_c && !(es && strcmp(es, "0") == 0) && tiles * 2 <= (uint64_t)sms && ktotal >= 16) {
        uint32_t sp, kc;
        if (fine) {
            const uint32_t nck = (ktotal + 3) / 4;
            sp = std::min<uint32_t>((uint32_t)(per_sm * sms / tiles), nck);
            kc = 4 * ((nck + sp - 1) / sp);
        } else {
            sp = std::min<uint32_t>((uint32_t)(sms / tiles), ktotal / 8);
            kc = sp >= 2 ? ((ktotal + sp - 1) / sp + 3) / 4 * 4 : ktotal;
        }
        if (sp >= 2) {
            sp = (ktotal + kc - 1) / kc;
            if (sp >= 2) {
                ws = cfi_splitk_workspace((size_t)sp * planes * ncols_dst * ld_ws * 4, stream);
                if (ws) {
                    splits = sp;
                    kchunk = kc;
                    if (per_sm == 2 && tiles * sp > (uint64_t)sms) {
                        ns_dflt = 2;
                        raw_dflt = 2;
                    }
                }
            }
        }
    }
    if (splits > 1) {
        cuuint64_t dw[4] = {nrows, ncols_dst, planes, splits};
        cuuint64_t sw[3] = {(cuuint64_t)ld_ws * 4, (cuuint64_t)ld_ws * 4 * ncols_dst, (cuuint64_t)ld_ws * 4 * ncols_dst * planes};
        cuuint32_t bw[4] = {32, 32, 1, 1}, ew[4] = {1, 1, 1, 1};
        if (enc(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ws, dw, sw, bw, ew, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            splits = 1;
            kchunk = (ktotal + 3) / 4 * 4;
        }
    }
    if (splits == 1 && tma_c) {
        const cuuint64_t s1 = (cuuint64_t)scd * 4;
        const cuuint64_t s2 = nch > 1 ? (cuuint64_t)scdst * 4 : s1 * ncols_dst;
        const cuuint64_t s3 = ns > 1 ? (cuuint64_t)ssd * 4 : s2 * nch;
        cuuint64_t dc[4] = {nrows, ncols_dst, nch, ns};
        cuuint64_t scs[3] = {s1, (s2 + 15) & ~(cuuint64_t)15, (s3 + 15) & ~(cuuint64_t)15};
        cuuint32_t boxc[4] = {32, 32, 1, 1}, esc[4] = {1, 1, 1, 1};
        tma_c = enc(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dst, dc, scs, boxc, esc, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    // 4. ring depths within the shared-memory limit (with A in TMEM the epilogue stages its chunks
    // in the B ring, plus what that ring lacks)
    const uint32_t b_stage = bn * BK * 2;
    const uint32_t stage_need = tma_c ? 8 * 2048 * 4 : 8 * 1024 * 4;  // epilogue staging, 8 warps
    uint32_t ns_ring = env_in("CFI_QMM_STAGES", ns_dflt, 2, ta ? QMM_MAX_NS : 4);
    auto pre_bytes = [&](uint32_t ns_) -> size_t {
        return ta ? (size_t)(stage_need > ns_ * b_stage ? (stage_need - ns_ * b_stage + 1023) / 1024 * 1024 : 0)
                  : (size_t)ns_ * A_STAGE;
    };
    // a CFI_QMM_BN wider than the automatic tile may leave no room for two raw slots at the
    // default depth: give up A/B stages first
    while (ns_ring > 2 && 1024 + pre_bytes(ns_ring) + (size_t)ns_ring * b_stage + 256 + 2 * (size_t)RAW_BYTES > QMM_SMEM_LIMIT)
        ns_ring--;
    const size_t fixed = 1024 + pre_bytes(ns_ring) + (size_t)ns_ring * b_stage + 256;
    const uint32_t nraw = std::min<uint32_t>(env_in("CFI_QMM_RAW", raw_dflt, 2, QMM_MAX_RAW),
                                             (uint32_t)std::min<size_t>(QMM_MAX_RAW, (QMM_SMEM_LIMIT - fixed) / RAW_BYTES));
    if (nraw < 2) return (int)cudaErrorInvalidValue;
    const size_t smem = fixed + (size_t)nraw * RAW_BYTES;
    QmmArgs a;
    a.x = x;
    a.K = K;
    a.Kt = Kt;
    a.nrows = nrows;
    a.ncols_dst = ncols_dst;
    a.bn = bn;
    a.ns = ns_ring;
    a.nraw = nraw;
    a.b_stage = b_stage;
    a.pre = (uint32_t)pre_bytes(ns_ring);
    a.splits = splits;
    a.kchunk = kchunk;
    a.stride_row_x = srx;
    a.stride_channel_x = scx;
    a.stride_sample_x = ssx;
    a.nchannels_y = nch;
    a.channel_ratio = chr;
    a.sample_ratio = smr;
    a.tma_c = tma_c ? 1 : 0;
    a.dst = dst;
    a.stride_col_dst = scd;
    a.stride_channel_dst = scdst;
    a.stride_sample_dst = ssd;
    a.err = device_error_ptr();
    a.raw_direct = raw_direct ? 1u : 0u;
    a.row_bytes = K / 32 * Q8_0_BYTES;
    static CfiPerDeviceOnce attr;
    cfi_once_per_device(attr, [] {
        cudaFuncSetAttribute(cfi_qmm_tc<TY, true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QMM_SMEM_LIMIT);
        cudaFuncSetAttribute(cfi_qmm_tc<TY, false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QMM_SMEM_LIMIT);
        cudaFuncSetAttribute(cfi_qmm_tc<TY, true, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QMM_SMEM_LIMIT);
        cudaFuncSetAttribute(cfi_qmm_tc<TY, false, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QMM_SMEM_LIMIT);
    });
    // two dequantising groups where a CTA has the SM to itself (more than half the shared
    // memory); CFI_QMM_GROUPS=1 keeps one
    const char* eg = getenv("CFI_QMM_GROUPS");
    const int groups = (eg && atoi(eg) == 1) ? 1 : (eg && atoi(eg) == 2) ? 2 : (smem > QMM_SMEM_LIMIT / 2 ? 2 : 1);
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((nrows + BM - 1) / BM, (ncols_dst + bn - 1) / bn, planes * splits);
    c.blockDim = dim3(groups == 2 ? qmm_threads<2>() : qmm_threads<1>(), 1, 1);
    c.dynamicSmemBytes = smem;
    c.stream = stream;
    c.attrs = at;
    c.numAttrs = pdl ? 1 : 0;
    cudaError_t e = groups == 2 ? (ta ? cudaLaunchKernelEx(&c, cfi_qmm_tc<TY, true, 2>, tw, tb, tc, a)
                                      : cudaLaunchKernelEx(&c, cfi_qmm_tc<TY, false, 2>, tw, tb, tc, a))
                                : (ta ? cudaLaunchKernelEx(&c, cfi_qmm_tc<TY, true, 1>, tw, tb, tc, a)
                                      : cudaLaunchKernelEx(&c, cfi_qmm_tc<TY, false, 1>, tw, tb, tc, a));
    if (e != cudaSuccess) return (int)e;
    if (splits > 1)
        return cfi_splitk_reduce_f32(ws, ld_ws, nrows, ncols_dst, planes, splits, dst, (long long)scd, (long long)scdst,
                                     (long long)ssd, nch, stream, pdl);
    return 0;
}

template <uint32_t TY>
int launch_tc(const uint64_t* v, cudaStream_t stream, void* fixed_xh = nullptr, size_t fixed_cap = 0) {
    // v: the 23 mul_mat_q words (6 pointers, 17 u32), subst_hook.rs arg order (probe.rs:293-321)
    const uint8_t* x = reinterpret_cast<const uint8_t*>(v[0]);
    const uint8_t* y = reinterpret_cast<const uint8_t*>(v[1]);
    float* dst = reinterpret_cast<float*>(v[4]);
    const uint32_t K = (uint32_t)v[6], nrows = (uint32_t)v[7], ncols_dst = (uint32_t)v[8];
    const uint32_t srx = (uint32_t)v[9], ncols_y = (uint32_t)v[10], scd = (uint32_t)v[11];
    const uint32_t chr = (uint32_t)v[12], nch = (uint32_t)v[13], scx = (uint32_t)v[14], scy = (uint32_t)v[15];
    const uint32_t scdst = (uint32_t)v[16], smr = (uint32_t)v[17], ns = (uint32_t)v[18], ssx = (uint32_t)v[19];
    const uint32_t ssy = (uint32_t)v[20], ssd = (uint32_t)v[21];
    if (K % 128 || !nrows || !ncols_dst || !nch || !ns || !chr || !smr) return (int)cudaErrorInvalidValue;
    if (K % mmq_qk<TY>()) return (int)cudaErrorInvalidValue;
    if (TY == T_Q8_0 && ((reinterpret_cast<uintptr_t>(x) & 3) || (srx & 1) || (scx & 1) || (ssx & 1)))
        return (int)cudaErrorInvalidValue;
    // Q4_K / Q5_K superblocks are read as 16-byte words; the other types need 2-byte alignment
    if ((TY == T_Q4_K || TY == T_Q5_K) && (reinterpret_cast<uintptr_t>(x) & 15)) return (int)cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(x) & 1) return (int)cudaErrorInvalidValue;
    // the fixed-scratch kernel's producers address a tile's 128 rows with 32-bit offsets
    if ((uint64_t)BM * srx * mmq_bb<TY>() >= (1ull << 31)) return (int)cudaErrorInvalidValue;
    const uint32_t Kc = mmq_corr<TY>() ? (K / 32 + BK - 1) / BK * BK : 0;
    const uint32_t Kt = K + Kc;
    const uint32_t planes = nch * ns;
    void* xh = nullptr;
    const size_t xh_bytes = (size_t)planes * ncols_dst * Kt * 2;
    // weight planes: (samples / sample_ratio) x (channels / channel_ratio)
    const uint32_t nch_x = nch / chr, planes_x = (ns / smr) * nch_x;
    if (nch % chr || ns % smr) return (int)cudaErrorInvalidValue;
    const size_t xh_pad = (xh_bytes + 255) & ~(size_t)255;
    const size_t wh_bytes = (size_t)planes_x * nrows * Kt * 2;
    int rc = 0;
    // at most 64 columns (a decode batch): the skinny kernel streams the weights once on the
    // warp-level int8 MMAs, in one launch (not for the allocation-free entry point: its K split
    // takes the stream's buffers)
    if (!fixed_xh && cfi_mmq_skinny_applies(TY, x, y, K, ncols_dst, srx, planes)) {
        const char* ep = getenv("CFI_PDL");
        return cfi_mmq_skinny_launch(TY, x, y, dst, K, nrows, ncols_dst, ncols_y, srx, scd, device_error_ptr(), stream,
                                     !(ep && strcmp(ep, "0") == 0));
    }
    const bool fused = qmm_applicable<TY>(x, K, srx, scx, ssx, nch_x, ns / smr);
    if (fixed_xh) {
        if (xh_bytes > fixed_cap) return (int)cudaErrorInvalidValue;
        xh = fixed_xh;
    } else {
        rc = scratch_for(fused ? xh_pad : xh_pad + wh_bytes, stream, &xh);
    }
    if (rc) return rc;
    if (fused)
        return launch_qmm<TY>(x, y, dst, xh, K, Kt, nrows, ncols_dst, srx, ncols_y, scd, chr, nch, scx, scy, scdst, smr, ns,
                              ssx, ssy, ssd, stream, fixed_xh == nullptr);
    if (!fixed_xh) {
        // 1. activations and weights -> fp16 K-major (one launch), then the shared TMA-fed
        // tcgen05 GEMM (C = Wh Xh^T per plane)
        __half* wh = reinterpret_cast<__half*>(static_cast<uint8_t*>(xh) + xh_pad);
        const uint64_t nblk = (uint64_t)nrows * (K / mmq_qk<TY>());
        const uint32_t gx_w = (uint32_t)((nblk + 255) / 256);
        const uint32_t gx_x = (ncols_dst * (K / 128) * 32 + 255) / 256;
        dim3 pgrid(std::max(gx_w, gx_x), planes + planes_x);
        cfi_mmq_prepass<TY><<<pgrid, 256, 0, stream>>>(y, static_cast<__half*>(xh), x, wh, K, Kt, ncols_dst, ncols_y, nch,
                                                       scy, ssy, planes, nrows, srx, nch_x, scx, ssx);
        rc = (int)cudaGetLastError();
        if (rc) return rc;
        TcGemm d;
        d.a = wh;
        d.b = xh;
        d.c = dst;
        d.fmt = 0;
        d.m = nrows;
        d.n = ncols_dst;
        d.k = Kt;
        d.lda = Kt;
        d.ldb = Kt;
        d.a_plane = (uint64_t)nrows * Kt;
        d.b_plane = (uint64_t)ncols_dst * Kt;
        d.a_planes = planes_x;
        d.nch = nch;
        d.nsamples = ns;
        d.chr = chr;
        d.smr = smr;
        d.c_type = 0;  // f32
        d.ldc = scd;
        d.c_zstride = scdst;
        d.c_wstride = ssd;
        d.alpha = 1.0f;
        d.beta = 0.0f;
        d.alpha_ptr = nullptr;
        d.beta_ptr = nullptr;
        d.scalar_f16 = 0;
        rc = cfi_tc_gemm(d, stream);
        return rc < 0 ? (int)cudaErrorInvalidValue : rc;
    }
    // fixed scratch (no room for the fp16 weights): activations -> fp16, then the fused kernel
    // dequantizes weight tiles in shared memory (Q8_0 and Q4_K only)
    if constexpr (TY != T_Q8_0 && TY != T_Q4_K) {
        return (int)cudaErrorNotSupported;
    } else {
    {
        const uint32_t warps = ncols_dst * (K / 128);
        dim3 grid((warps * 32 + 255) / 256, planes);
        if (TY == T_Q4_K)
            cfi_mmq_x_to_f16<1, 1><<<grid, 256, 0, stream>>>(y, static_cast<__half*>(xh), K, Kt, ncols_dst, ncols_y, nch, scy, ssy);
        else
            cfi_mmq_x_to_f16<0, 0><<<grid, 256, 0, stream>>>(y, static_cast<__half*>(xh), K, Kt, ncols_dst, ncols_y, nch, scy, ssy);
        rc = (int)cudaGetLastError();
        if (rc) return rc;
    }
    // 2. tensor map over Xh: dims (Kt, ncols, planes), box (64, BN, 1), 128-byte swizzle
    const uint32_t bn = tile_n(ncols_dst);
    PFN_encodeTiled enc = encode_fn();
    if (!enc) return (int)cudaErrorNotSupported;
    CUtensorMap tmap;
    cuuint64_t gdim[3] = {Kt, ncols_dst, planes};
    cuuint64_t gstride[2] = {(cuuint64_t)Kt * 2, (cuuint64_t)Kt * 2 * ncols_dst};
    cuuint32_t box[3] = {BK, bn, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult cr = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, xh, gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return (int)cudaErrorInvalidValue;
    // dst through TMA stores when its strides allow (16-byte multiples, aligned base)
    CUtensorMap tmap_c;
    memset(&tmap_c, 0, sizeof tmap_c);
    bool tma_c = (scd % 4) == 0 && (nch == 1 || scdst % 4 == 0) && (ns == 1 || ssd % 4 == 0) &&
                 (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    if (tma_c) {
        const cuuint64_t s1 = (cuuint64_t)scd * 4;
        const cuuint64_t s2 = nch > 1 ? (cuuint64_t)scdst * 4 : s1 * ncols_dst;
        const cuuint64_t s3 = ns > 1 ? (cuuint64_t)ssd * 4 : s2 * nch;
        cuuint64_t dc[4] = {nrows, ncols_dst, nch, ns};
        cuuint64_t scs[3] = {s1, (s2 + 15) & ~(cuuint64_t)15, (s3 + 15) & ~(cuuint64_t)15};
        cuuint32_t boxc[4] = {32, 32, 1, 1}, esc[4] = {1, 1, 1, 1};
        tma_c = enc(&tmap_c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dst, dc, scs, boxc, esc, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    MmqArgs a;
    a.tma_c = tma_c ? 1 : 0;
    a.x = x;
    a.dst = dst;
    a.K = K;
    a.Kt = Kt;
    a.nrows = nrows;
    a.ncols_dst = ncols_dst;
    a.bn = bn;
    a.stride_row_x = srx;
    a.stride_col_dst = scd;
    a.nchannels_y = nch;
    a.channel_ratio = chr;
    a.sample_ratio = smr;
    a.stride_channel_x = scx;
    a.stride_sample_x = ssx;
    a.stride_channel_dst = scdst;
    a.stride_sample_dst = ssd;
    a.err = device_error_ptr();
    static CfiPerDeviceOnce attr;
    cfi_once_per_device(attr, [] {
        cudaFuncSetAttribute(cfi_mmq_tc<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    });
    dim3 grid((nrows + BM - 1) / BM, (ncols_dst + bn - 1) / bn, planes);
    cfi_mmq_tc<TY><<<grid, THREADS, SMEM_BYTES, stream>>>(tmap, tmap_c, a);
    return (int)cudaGetLastError();
    }
}

}  // namespace

namespace cfi {
int mmq_tile_n(uint32_t ncols_dst) { return (int)tile_n(ncols_dst); }
int mmq_threads() { return THREADS; }
bool mmq_type_ok(uint32_t ty) {
    return ty == T_Q8_0 || ty == T_Q4_K || ty == T_Q4_0 || ty == T_Q5_0 || ty == T_Q5_K || ty == T_Q6_K;
}

int mmq_launch(const cfi_plan& plan, void** args, void* stream) {
    std::vector<uint64_t> v = arg_values(plan, args);
    if (v.size() != 23) return (int)cudaErrorInvalidValue;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (plan.ty) {
    case T_Q8_0: return launch_tc<T_Q8_0>(v.data(), s);
    case T_Q4_K: return launch_tc<T_Q4_K>(v.data(), s);
    case T_Q4_0: return launch_tc<T_Q4_0>(v.data(), s);
    case T_Q5_0: return launch_tc<T_Q5_0>(v.data(), s);
    case T_Q5_K: return launch_tc<T_Q5_K>(v.data(), s);
    case T_Q6_K: return launch_tc<T_Q6_K>(v.data(), s);
    default: return (int)cudaErrorNotSupported;
    }
}
}  // namespace cfi

// ---------------------------------------------------------------------------------------------
// cfi_mmq_static_scratch: the same GEMM for callers that may not allocate device memory.  Its fp16
// activation copy lives in this fixed array (CFI_MMQ_STATIC_SCRATCH_BYTES on every GPU where the
// library is loaded, held until the process exits) instead of a buffer from cudaMalloc.  Host
// code must not hand the array's name to a kernel (on the host it is only a stand-in for the
// device symbol): its device address is looked up once per device with cudaGetSymbolAddress.
// ---------------------------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_mmq_static_scratch[CFI_MMQ_STATIC_SCRATCH_BYTES];

namespace {
constexpr int MAX_DEVICES = 64;
std::mutex g_static_mu;
void* g_static_addr[MAX_DEVICES];

// Device address of the static scratch on the current device (set up on first use).
int static_scratch_addr(void** out, std::string* why) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *why = std::string("no current CUDA device: ") + cudaGetErrorString(e);
        return (int)e;
    }
    if (dev < 0 || dev >= MAX_DEVICES) {
        *why = "device index out of range";
        return (int)cudaErrorInvalidDevice;
    }
    std::lock_guard<std::mutex> g(g_static_mu);
    if (!g_static_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_mmq_static_scratch);
        if (e != cudaSuccess || !p) {
            *why = std::string("cudaGetSymbolAddress of the static scratch failed: ") + cudaGetErrorString(e);
            return (int)(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
        }
        g_static_addr[dev] = p;
    }
    *out = g_static_addr[dev];
    return 0;
}
}  // namespace

extern "C" int cfi_mmq_static_scratch(uint32_t ggml_type, void** kernel_params, void* stream, char* why, size_t why_len) {
    std::string w;
    auto fail = [&](int code) {
        if (why && why_len) snprintf(why, why_len, "%s", w.c_str());
        return code;
    };
    if (!kernel_params) {
        w = "kernel_params is NULL";
        return fail((int)cudaErrorInvalidValue);
    }
    if (ggml_type != T_Q8_0 && ggml_type != T_Q4_K) {
        w = "only Q8_0 (8) and Q4_K (12) weights are supported";
        return fail((int)cudaErrorNotSupported);
    }
    uint64_t v[23];
    for (int i = 0; i < 23; i++) {
        if (!kernel_params[i]) {
            w = "kernel_params entry " + std::to_string(i) + " is NULL";
            return fail((int)cudaErrorInvalidValue);
        }
        v[i] = 0;
        memcpy(&v[i], kernel_params[i], i < 6 ? 8 : 4);
    }
    if (v[2] != 0 || v[3] != 0) {
        w = "expert routing (ids_dst / expert_bounds) is not supported";
        return fail((int)cudaErrorNotSupported);
    }
    const uint64_t K = (uint32_t)v[6], ncols_dst = (uint32_t)v[8], planes = (uint64_t)(uint32_t)v[13] * (uint32_t)v[18];
    if (K == 0 || K % 128 || ncols_dst == 0 || planes == 0) {
        w = "ncols_x must be a non-zero multiple of 128 and ncols_dst, nchannels_y, nsamples_y non-zero";
        return fail((int)cudaErrorInvalidValue);
    }
    if (planes > UINT32_MAX) {  // the launch counts channel x sample planes in 32 bits
        w = "nchannels_y x nsamples_y exceeds 2^32 - 1";
        return fail((int)cudaErrorInvalidValue);
    }
    // fp16 activation columns of Kt values: K, plus for Q4_K the correction columns (one per 32
    // values, padded to the 64-value pipeline stage), i.e. Kt = K + ceil(K / 2048) * 64
    const uint64_t Kt = K + (ggml_type == T_Q4_K ? (K / 32 + BK - 1) / BK * BK : 0);
    const unsigned __int128 need = (unsigned __int128)planes * ncols_dst * Kt * 2;  // cannot wrap
    if (need > CFI_MMQ_STATIC_SCRATCH_BYTES) {
        const uint64_t shown = need > UINT64_MAX ? UINT64_MAX : (uint64_t)need;
        w = "this GEMM needs " + std::to_string(shown) + " bytes of scratch (planes x ncols_dst x Kt x 2, Kt = ncols_x" +
            (ggml_type == T_Q4_K ? std::string(" + ceil(ncols_x / 2048) x 64 for Q4_K") : std::string()) +
            "); the static scratch holds " + std::to_string((unsigned long long)CFI_MMQ_STATIC_SCRATCH_BYTES);
        return fail((int)cudaErrorInvalidValue);
    }
    void* scratch = nullptr;
    int rc = static_scratch_addr(&scratch, &w);
    if (rc) return fail(rc);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rc = ggml_type == T_Q8_0 ? launch_tc<T_Q8_0>(v, s, scratch, CFI_MMQ_STATIC_SCRATCH_BYTES)
                             : launch_tc<T_Q4_K>(v, s, scratch, CFI_MMQ_STATIC_SCRATCH_BYTES);
    if (rc) w = std::string("launch failed: ") + cudaGetErrorString((cudaError_t)rc);
    return rc ? fail(rc) : 0;
}

unsigned int cfi_gemm_error_take();  // k_gemm_sm100.cu
namespace cfi {
unsigned int fattn_error_take();     // k_fattn_sm100.cu
}

extern "C" int cfi_mmq_skinny_group(uint32_t type, int n, const void* const* x, const void* y, float* const* dst,
                                    const uint32_t* nrows, const uint32_t* stride_row_x, const uint32_t* stride_col_dst,
                                    uint32_t K, uint32_t ncols, uint32_t ncols_y, void* stream) {
    if ((type != T_Q4_K && type != T_Q8_0) || !x || !dst || !nrows || !stride_row_x || !stride_col_dst || ncols == 0 ||
        ncols > 64)
        return (int)cudaErrorInvalidValue;
    const char* ep = getenv("CFI_PDL");
    return cfi_mmq_skinny_group_launch(type, n, x, y, dst, nrows, stride_row_x, stride_col_dst, K, ncols, ncols_y,
                                       device_error_ptr(), static_cast<cudaStream_t>(stream), !(ep && strcmp(ep, "0") == 0));
}

extern "C" int cfi_mmq_skinny_group_peers(uint32_t type, int n, const void* const* x, const void* y, float* const* dst,
                                          const uint32_t* nrows, const uint32_t* stride_row_x,
                                          const uint32_t* stride_col_dst, uint32_t K, uint32_t ncols, uint32_t ncols_y,
                                          const CfiPeerSet* peers, void* stream) {
    if ((type != T_Q4_K && type != T_Q8_0) || !x || !dst || !nrows || !stride_row_x || !stride_col_dst || ncols == 0 ||
        ncols > 64)
        return (int)cudaErrorInvalidValue;
    CfiPeerDev pd;
    const int rc = cfi_peer_dev(peers, &pd);
    if (rc) return rc;
    const char* ep = getenv("CFI_PDL");
    return cfi_mmq_skinny_group_launch(type, n, x, y, dst, nrows, stride_row_x, stride_col_dst, K, ncols, ncols_y,
                                       device_error_ptr(), static_cast<cudaStream_t>(stream), !(ep && strcmp(ep, "0") == 0),
                                       &pd);
}

// The library's device error word (the bounded waits of the kernels in other files record there).
unsigned int* cfi_device_error_word() { return device_error_ptr(); }

extern "C" unsigned int cfi_device_error(void) {
    unsigned int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_cfi_device_error, sizeof v) != cudaSuccess) {
        cudaGetLastError();
        v = 0;
    } else {
        cudaMemcpyToSymbol(g_cfi_device_error, &z, sizeof z);
    }
    const unsigned int g = cfi_gemm_error_take();
    const unsigned int m = cfi_mmvq_error_take();
    const unsigned int f = cfi::fattn_error_take();
    return v ? v : (g ? g : (m ? m : f));
}
