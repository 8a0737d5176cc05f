// k_gemm_sm100.cu -- cuBLAS-compatible GEMM of libcfi_b200.so (the dense path ggml reaches through
// cublasGemmEx, served by cuda-for-intel's cuBLAS shim, crates/cublas_shim/src/lib.rs:627-1076).
//
// C = alpha * op(A) * op(B) + beta * C, column-major.  The layout ggml uses -- op(A) = A^T (A stored
// k x m, lda >= k) and op(B) = B (B stored k x n, ldb >= k), f16 or bf16 -- has both operands
// K-major and runs on the tensor cores:
//   * one thread of warp 5 streams 128 x 64 tiles of A and BN x 64 tiles of B with TMA
//     (128-byte swizzle: the UMMA canonical K-major layout; rows/columns/K past the matrix read as
//     zero), strided batches as the third tensor dimension;
//   * one thread of warp 4 issues tcgen05.mma kind::f16 (M 128, N BN <= 256, K 16) into an fp32
//     accumulator in tensor memory;
//   * warps 0-3 apply alpha/beta and store C: f32 with beta 0 through TMA tensor stores of
//     32 x 32 chunks, otherwise in its dtype (f32, f16 or bf16) in runs of 4 rows (accumulator
//     chunks transposed through shared memory).
// Every other legal call (other transposes, f32 inputs, device pointer arrays) runs a tiled SIMT
// kernel with fp32 accumulation.  Validation follows cuBLAS (plan.rs:160-215).
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <type_traits>
#include <vector>

#include "../../include/cfi_cublas.h"
#include "cfi_common.cuh"
#include "sm100_ptx.cuh"
#include "tc_epilogue.cuh"
#include "cfi_kernels.h"

namespace {

using namespace sm100;

constexpr int BM = 128, BK = 64, NSTAGE = 4, THREADS = 192;
constexpr int A_STAGE = BM * BK * 2, B_STAGE = 256 * BK * 2;
constexpr size_t SMEM_BYTES = 1024 + (size_t)NSTAGE * (A_STAGE + B_STAGE) + 256;

static __device__ unsigned int g_gemm_error;

struct GemmArgs {
    void* c;
    long long c_zstride, c_wstride;  // elements between output channel / sample planes
    int c_type, ldc;
    uint32_t m, n, k, bn;
    uint32_t nch, chr, smr, nch_x;   // output plane p: channel p % nch, sample p / nch; A plane below
    float alpha, beta;
    const void* alpha_ptr;  // device pointer mode
    const void* beta_ptr;
    int scalar_f16;
    int tma_c;  // C is f32, beta 0 and host scalars: the epilogue stores through tmc
    uint32_t splits, kchunk;  // split K: blockIdx.z = plane * splits + split, k steps [split kchunk, ..)
    unsigned int* err;
};

CFI_DEV float load_scalar(const void* p, int f16) {
    return f16 ? __half2float(*static_cast<const __half*>(p)) : *static_cast<const float*>(p);
}

CFI_DEV float ld_elem(const void* p, size_t i, int t) {
    if (t == CFI_R_32F) return static_cast<const float*>(p)[i];
    if (t == CFI_R_16F) return __half2float(static_cast<const __half*>(p)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
CFI_DEV void st_elem(void* p, size_t i, int t, float v) {
    if (t == CFI_R_32F)
        static_cast<float*>(p)[i] = v;
    else if (t == CFI_R_16F)
        static_cast<__half*>(p)[i] = __float2half_rn(v);
    else
        static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

template <int FMT>
__global__ void __launch_bounds__(THREADS, 1)
    cfi_gemm_tc(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                const __grid_constant__ CUtensorMap tmc, const GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = sA + NSTAGE * A_STAGE;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + NSTAGE * B_STAGE);
    uint64_t* empty = full + NSTAGE;
    uint64_t* done = empty + NSTAGE;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* epi_ok = abort_flag + 1;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t bn = a.bn;
    const uint32_t tmem_cols = bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : 256;
    const int ktotal = (int)((a.k + BK - 1) / BK);
    const uint32_t split = blockIdx.z % a.splits;
    const uint32_t m0 = blockIdx.x * BM, n0 = blockIdx.y * bn, z = blockIdx.z / a.splits;
    // this CTA's k steps [k0, k0 + ksteps) (all of K unless split)
    const int k0 = (int)(split * a.kchunk);
    const int ksteps = max(0, min(ktotal, k0 + (int)a.kchunk) - k0);
    // output plane z = (sample wt, channel zt); its A plane follows the channel / sample ratios
    const uint32_t wt = z / a.nch, zt = z - wt * a.nch;
    const uint32_t za = (wt / a.smr) * a.nch_x + zt / a.chr;

    if (tid == 0) {
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 4) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();  // launched early (programmatic dependent launch): the operands may come from the previous kernel

    if (warp == 5) {
        if (lane == 0) {
            prefetch_tmap(&tma);
            prefetch_tmap(&tmb);
            const uint32_t bytes = (BM + bn) * BK * 2;
            for (int s = 0; s < ksteps; s++) {
                const int slot = s % NSTAGE;
                if (!mbar_wait(&empty[slot], ((uint32_t)(s / NSTAGE) & 1) ^ 1, abort_flag)) {
                    cfi_set_error(a.err, 0x500 + slot);
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full[slot], bytes);
                tma_load_3d(sA + slot * A_STAGE, &tma, (k0 + s) * BK, (int)m0, (int)za, &full[slot]);
                tma_load_3d(sB + slot * B_STAGE, &tmb, (k0 + s) * BK, (int)n0, (int)z, &full[slot]);
            }
        }
        __syncwarp();
    } else if (warp == 4) {
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(BM, bn, FMT);
            for (int s = 0; s < ksteps; s++) {
                const int slot = s % NSTAGE;
                if (!mbar_wait(&full[slot], (uint32_t)(s / NSTAGE) & 1, abort_flag)) {
                    cfi_set_error(a.err, 0x600 + slot);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t ab = smem_u32(sA + slot * A_STAGE), bb = smem_u32(sB + slot * B_STAGE);
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++)
                    mma_f16(tmem, sw128_kmajor_desc(ab + 32 * kk), sw128_kmajor_desc(bb + 32 * kk), idesc,
                            (s > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&empty[slot]);
            }
            mma_commit(done);
        }
        __syncwarp();
    } else {
        // ================= epilogue (warps 0-3: TMEM lanes = rows of the tile) =================
        if (tid == 0) {
            bool got = false;
            if (!*abort_flag) {
                got = mbar_wait(done, 0, abort_flag);
                if (!got) {
                    cfi_set_error(a.err, 0x700);
                    *abort_flag = 1;
                }
            }
            *epi_ok = got ? 1 : 0;
        }
        named_bar_sync(1, 128);
        tc_fence_after();
        if (*epi_ok) {
            const float alpha = a.alpha_ptr ? load_scalar(a.alpha_ptr, a.scalar_f16) : a.alpha;
            const float beta = a.beta_ptr ? load_scalar(a.beta_ptr, a.scalar_f16) : a.beta;
            if (a.tma_c) {
                // every MMA has completed: the A ring holds the 8 KB per-warp staging buffers
                float* tbuf = reinterpret_cast<float*>(sA) + warp * 2048;
                if (a.splits > 1)  // raw partial sums into the split-K workspace (plane, split)
                    tmem_tile_tma_store(tmem, warp, lane, 4, bn, tbuf, &tmc, (int)m0, (int)n0, (int)z, (int)split,
                                        [](float v) { return v; });
                else
                    tmem_tile_tma_store(tmem, warp, lane, 4, bn, tbuf, &tmc, (int)m0, (int)n0, (int)zt, (int)wt,
                                        [&](float v) { return alpha * v; });
            } else {
            const int ct = a.c_type, es = ct == CFI_R_32F ? 4 : 2;
            uint8_t* cz = static_cast<uint8_t*>(a.c) + (size_t)((long long)zt * a.c_zstride + (long long)wt * a.c_wstride) * es;
            // 4 consecutive rows as one 16-byte (f32) or 8-byte (f16/bf16) access
            const bool vec = (a.ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(cz) & (uintptr_t)(4 * es - 1)) == 0;
            // every MMA has completed: the A ring is free for the 4 KB per-warp staging buffers
            float* buf = reinterpret_cast<float*>(sA) + warp * 1024;
            tmem_tile_store(tmem, warp, lane, 4, bn, buf, [&](uint32_t c, uint32_t rr, float4 f) {
                const uint32_t col = n0 + c, row = m0 + rr;
                if (col >= a.n || row >= a.m) return;
                const size_t ci = (size_t)col * a.ldc + row;
                float r[4] = {alpha * f.x, alpha * f.y, alpha * f.z, alpha * f.w};
                if (vec && row + 3 < a.m) {
                    if (ct == CFI_R_32F) {
                        float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(cz) + ci);
                        if (beta != 0.0f) {
                            const float4 o = *p;
                            r[0] += beta * o.x;
                            r[1] += beta * o.y;
                            r[2] += beta * o.z;
                            r[3] += beta * o.w;
                        }
                        *p = make_float4(r[0], r[1], r[2], r[3]);
                    } else {
                        uint2* p = reinterpret_cast<uint2*>(cz + ci * 2);
                        if (beta != 0.0f) {
                            const uint2 o = *p;
                            const uint16_t h[4] = {(uint16_t)(o.x & 0xffffu), (uint16_t)(o.x >> 16), (uint16_t)(o.y & 0xffffu),
                                                   (uint16_t)(o.y >> 16)};
#pragma unroll
                            for (int e = 0; e < 4; e++)
                                r[e] += beta * (ct == CFI_R_16F ? __half2float(__ushort_as_half(h[e]))
                                                                : __bfloat162float(__ushort_as_bfloat16(h[e])));
                        }
                        uint16_t h[4];
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            h[e] = ct == CFI_R_16F ? __half_as_ushort(__float2half_rn(r[e]))
                                                   : __bfloat16_as_ushort(__float2bfloat16_rn(r[e]));
                        *p = make_uint2((uint32_t)h[0] | ((uint32_t)h[1] << 16), (uint32_t)h[2] | ((uint32_t)h[3] << 16));
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        if (row + e >= a.m) break;
                        float v = r[e];
                        if (beta != 0.0f) v += beta * ld_elem(cz, ci + e, ct);
                        st_elem(cz, ci + e, ct, v);
                    }
                }
            });
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
}

// ---- 2-SM variant: a cluster of 2 CTAs computes a 256-row tile with tcgen05.mma.cta_group::2 ----
// CTA r of the pair holds rows 128 r .. 128 r + 127 of the tile (A) and columns r BN/2 .. of B; the
// leader (r = 0) issues the MMA (M 256, N BN) over both CTAs' shared memory, each CTA's TMEM gets
// its own 128 rows.  Both CTAs' TMA loads complete on the leader's `full` barrier; the leader's
// commits arrive on both CTAs' `empty` and `done` barriers.  Half-width B stages let 6 stages fit.
constexpr int NSTAGE2 = 6;
constexpr int A2_STAGE = BM * BK * 2;   // 16 KB
constexpr int B2_STAGE = 128 * BK * 2;  // 16 KB: half of BN <= 256
constexpr size_t SMEM2_BYTES = 1024 + (size_t)NSTAGE2 * (A2_STAGE + B2_STAGE) + 256;

template <int FMT>
__global__ void __launch_bounds__(THREADS, 1)
    cfi_gemm_tc2(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                 const __grid_constant__ CUtensorMap tmc, const GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = sA + NSTAGE2 * A2_STAGE;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + NSTAGE2 * B2_STAGE);
    uint64_t* empty = full + NSTAGE2;
    uint64_t* done = empty + NSTAGE2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* epi_ok = abort_flag + 1;

    const uint32_t rank = cluster_ctarank();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t bn = a.bn, half = bn / 2;
    const uint32_t tmem_cols = bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : 256;
    const int ksteps = (int)((a.k + BK - 1) / BK);
    const uint32_t m0 = (blockIdx.x >> 1) * (2 * BM) + rank * BM, n0 = blockIdx.y * bn, z = blockIdx.z;
    const uint32_t wt = z / a.nch, zt = z - wt * a.nch;
    const uint32_t za = (wt / a.smr) * a.nch_x + zt / a.chr;

    if (tid == 0) {
        for (int i = 0; i < NSTAGE2; i++) {
            mbar_init(&full[i], 1);   // the leader's expect_tx (bytes of both CTAs)
            mbar_init(&empty[i], 1);  // the leader's tcgen05.commit
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 4) {
        tmem_alloc2(tmem_slot, tmem_cols);
        tmem_relinquish2();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers are initialised before any cross-CTA arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();  // launched early (programmatic dependent launch): the operands may come from the previous kernel

    if (warp == 5) {
        if (lane == 0) {
            prefetch_tmap(&tma);
            prefetch_tmap(&tmb);
            const uint32_t full0 = mapa_shared(smem_u32(&full[0]), 0);
            const uint32_t bytes = 2u * (uint32_t)(A2_STAGE + half * BK * 2);
            for (int s = 0; s < ksteps; s++) {
                const int slot = s % NSTAGE2;
                if (!mbar_wait(&empty[slot], ((uint32_t)(s / NSTAGE2) & 1) ^ 1, abort_flag)) {
                    cfi_set_error(a.err, 0x800 + slot);
                    *abort_flag = 1;
                    break;
                }
                if (rank == 0) mbar_arrive_expect_tx(&full[slot], bytes);
                const uint32_t fb = full0 + (uint32_t)slot * 8u;
                tma_load_3d_2sm(sA + slot * A2_STAGE, &tma, s * BK, (int)m0, (int)za, fb);
                tma_load_3d_2sm(sB + slot * B2_STAGE, &tmb, s * BK, (int)(n0 + rank * half), (int)z, fb);
            }
        }
        __syncwarp();
    } else if (warp == 4) {
        if (rank == 0 && lane == 0) {
            const uint32_t idesc = idesc_f16(2 * BM, bn, FMT);
            for (int s = 0; s < ksteps; s++) {
                const int slot = s % NSTAGE2;
                if (!mbar_wait(&full[slot], (uint32_t)(s / NSTAGE2) & 1, abort_flag)) {
                    cfi_set_error(a.err, 0x900 + slot);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t ab = smem_u32(sA + slot * A2_STAGE), bb = smem_u32(sB + slot * B2_STAGE);
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++)
                    mma2_f16(tmem, sw128_kmajor_desc(ab + 32 * kk), sw128_kmajor_desc(bb + 32 * kk), idesc,
                             (s > 0 || kk > 0) ? 1u : 0u);
                mma2_commit_mc(&empty[slot], 0x3);
            }
            mma2_commit_mc(done, 0x3);  // also after a failure: the MMAs already issued
        }
        __syncwarp();
    } else {
        // ================= epilogue (warps 0-3: this CTA's 128 TMEM lanes) =================
        if (tid == 0) {
            const bool got = mbar_wait(done, 0, abort_flag);
            if (!got) {
                cfi_set_error(a.err, 0xA00);
                *abort_flag = 1;
            }
            *epi_ok = got ? 1 : 0;
        }
        named_bar_sync(1, 128);
        tc_fence_after();
        if (*epi_ok) {
            const float alpha = a.alpha_ptr ? load_scalar(a.alpha_ptr, a.scalar_f16) : a.alpha;
            const float beta = a.beta_ptr ? load_scalar(a.beta_ptr, a.scalar_f16) : a.beta;
            if (a.tma_c) {
                float* tbuf = reinterpret_cast<float*>(sA) + warp * 2048;
                tmem_tile_tma_store(tmem, warp, lane, 4, bn, tbuf, &tmc, (int)m0, (int)n0, (int)zt, (int)wt,
                                    [&](float v) { return alpha * v; });
            } else {
                const int ct = a.c_type, es = ct == CFI_R_32F ? 4 : 2;
                uint8_t* cz = static_cast<uint8_t*>(a.c) + (size_t)((long long)zt * a.c_zstride + (long long)wt * a.c_wstride) * es;
                float* buf = reinterpret_cast<float*>(sA) + warp * 1024;
                tmem_tile_store(tmem, warp, lane, 4, bn, buf, [&](uint32_t c, uint32_t rr, float4 f) {
                    const uint32_t col = n0 + c, row = m0 + rr;
                    if (col >= a.n || row >= a.m) return;
                    const size_t ci = (size_t)col * a.ldc + row;
                    const float r[4] = {alpha * f.x, alpha * f.y, alpha * f.z, alpha * f.w};
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        if (row + e >= a.m) break;
                        float v = r[e];
                        if (beta != 0.0f) v += beta * ld_elem(cz, ci + e, ct);
                        st_elem(cz, ci + e, ct, v);
                    }
                });
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // neither CTA leaves while the pair still reads its TMEM or shared memory
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc2(tmem, tmem_cols);
    }
}

// Split-K reduction: C[plane][col][row] = alpha * sum_s ws[s][plane][col][row] (+ beta C), the
// partials added in split order (deterministic).  Thread: 4 consecutive rows of one column.
struct ReduceArgs {
    const float* ws;
    uint32_t ld_ws, m, n, planes, splits;
    void* c;
    int c_type;
    long long ldc, c_zstride, c_wstride;
    uint32_t nch;
    float alpha, beta;
    const void* alpha_ptr;
    const void* beta_ptr;
    int scalar_f16;
};

__global__ void __launch_bounds__(256) cfi_gemm_splitk_reduce(const ReduceArgs r) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t mq = (r.m + 3) / 4;
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)mq * r.n * r.planes) return;
    const uint32_t rq = (uint32_t)(t % mq);
    const uint64_t cp = t / mq;
    const uint32_t col = (uint32_t)(cp % r.n), plane = (uint32_t)(cp / r.n);
    const uint32_t row = 4 * rq;
    const size_t split_stride = (size_t)r.planes * r.n * r.ld_ws;
    const float* p = r.ws + ((size_t)plane * r.n + col) * r.ld_ws + row;
    float4 acc = *reinterpret_cast<const float4*>(p);
    for (uint32_t sp = 1; sp < r.splits; sp++) {
        const float4 v = *reinterpret_cast<const float4*>(p + sp * split_stride);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    const float alpha = r.alpha_ptr ? load_scalar(r.alpha_ptr, r.scalar_f16) : r.alpha;
    const float beta = r.beta_ptr ? load_scalar(r.beta_ptr, r.scalar_f16) : r.beta;
    const uint32_t wt = plane / r.nch, zt = plane - wt * r.nch;
    const int es = r.c_type == CFI_R_32F ? 4 : 2;
    uint8_t* cz = static_cast<uint8_t*>(r.c) + (size_t)((long long)zt * r.c_zstride + (long long)wt * r.c_wstride) * es;
    const float v[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int e = 0; e < 4; e++) {
        if (row + e >= r.m) break;
        const size_t ci = (size_t)col * r.ldc + row + e;
        float o = alpha * v[e];
        if (beta != 0.0f) o += beta * ld_elem(cz, ci, r.c_type);
        st_elem(cz, ci, r.c_type, o);
    }
}

// Skinny GEMM (op(A) = A^T, op(B) = B, f16/bf16, n <= 8 columns): the decode-time attention
// products (KQ, KQV per KV head).  One warp per output row: 16-byte loads of A's row and of
// each B column over k, fp32 FMAs, a butterfly per column.  Launched with PDL like the other
// kernels.  Strided batches in blockIdx.y.
struct SkinnyArgs {
    const void* a;
    const void* b;
    void* c;
    long long sa, sb, sc;
    int lda, ldb, ldc, ct;
    uint32_t m, n, k;
    float alpha, beta;
    const void* alpha_ptr;
    const void* beta_ptr;
    int scalar_f16;
};

template <int FMT>
__global__ void __launch_bounds__(256) cfi_gemm_skinny(const SkinnyArgs p) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t row = blockIdx.x * 8 + (threadIdx.x >> 5), z = blockIdx.y;
    if (row >= p.m) return;
    typedef typename std::conditional<FMT == 0, __half2, __nv_bfloat162>::type T2;
    const uint16_t* A = static_cast<const uint16_t*>(p.a) + (size_t)z * p.sa + (size_t)row * p.lda;
    const uint16_t* B = static_cast<const uint16_t*>(p.b) + (size_t)z * p.sb;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    auto f2 = [](uint32_t w) -> float2 {
        T2 h = *reinterpret_cast<const T2*>(&w);
        if constexpr (FMT == 0)
            return __half22float2(h);
        else
            return __bfloat1622float2(h);
    };
    for (uint32_t k0 = lane * 8; k0 < p.k; k0 += 256) {
        if (k0 + 8 <= p.k) {
            const uint4 av = *reinterpret_cast<const uint4*>(A + k0);
            const float2 a0 = f2(av.x), a1 = f2(av.y), a2 = f2(av.z), a3 = f2(av.w);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j < (int)p.n) {
                    const uint4 bv = *reinterpret_cast<const uint4*>(B + (size_t)j * p.ldb + k0);
                    const float2 b0 = f2(bv.x), b1 = f2(bv.y), b2 = f2(bv.z), b3 = f2(bv.w);
                    float s = acc[j];
                    s = fmaf(a0.x, b0.x, s);
                    s = fmaf(a0.y, b0.y, s);
                    s = fmaf(a1.x, b1.x, s);
                    s = fmaf(a1.y, b1.y, s);
                    s = fmaf(a2.x, b2.x, s);
                    s = fmaf(a2.y, b2.y, s);
                    s = fmaf(a3.x, b3.x, s);
                    s = fmaf(a3.y, b3.y, s);
                    acc[j] = s;
                }
            }
        } else {
            for (uint32_t kk = k0; kk < p.k; kk++) {
                const float av = FMT == 0 ? __half2float(__ushort_as_half(A[kk])) : __bfloat162float(__ushort_as_bfloat16(A[kk]));
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (j < (int)p.n) {
                        const uint16_t bb = B[(size_t)j * p.ldb + kk];
                        acc[j] = fmaf(av, FMT == 0 ? __half2float(__ushort_as_half(bb)) : __bfloat162float(__ushort_as_bfloat16(bb)), acc[j]);
                    }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    if (lane < p.n) {
        float v = acc[0];
#pragma unroll
        for (int j = 1; j < 8; j++)
            if ((int)lane == j) v = acc[j];
        const float alpha = p.alpha_ptr ? load_scalar(p.alpha_ptr, p.scalar_f16) : p.alpha;
        const float beta = p.beta_ptr ? load_scalar(p.beta_ptr, p.scalar_f16) : p.beta;
        void* cz = static_cast<uint8_t*>(p.c) + (size_t)z * p.sc * (p.ct == CFI_R_32F ? 4 : 2);
        const size_t ci = (size_t)lane * p.ldc + row;
        float r = alpha * v;
        if (beta != 0.0f) r += beta * ld_elem(cz, ci, p.ct);
        st_elem(cz, ci, p.ct, r);
    }
}

// Tiled SIMT GEMM: 16 x 16 output tile per block, any op/dtype combination, fp32 accumulation.
// `ptrs` non-zero: A, B, C are device arrays of per-batch pointers (cublasGemmBatchedEx).
struct SimtArgs {
    const void* a;
    const void* b;
    void* c;
    long long sa, sb, sc;
    int lda, ldb, ldc, ta, tb, at, bt, ct;
    uint32_t m, n, k;
    float alpha, beta;
    const void* alpha_ptr;
    const void* beta_ptr;
    int scalar_f16, ptrs;
};

__global__ void __launch_bounds__(256) cfi_gemm_simt(const SimtArgs p) {
    __shared__ float As[16][17], Bs[16][17];
    const uint32_t tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const uint32_t i = blockIdx.x * 16 + tx, j = blockIdx.y * 16 + ty, z = blockIdx.z;
    const void* A;
    const void* B;
    void* Cp;
    if (p.ptrs) {
        A = static_cast<const void* const*>(p.a)[z];
        B = static_cast<const void* const*>(p.b)[z];
        Cp = static_cast<void* const*>(p.c)[z];
    } else {
        const size_t ea = p.at == CFI_R_32F ? 4 : 2, ec = p.ct == CFI_R_32F ? 4 : 2;
        A = static_cast<const uint8_t*>(p.a) + (size_t)z * p.sa * ea;
        B = static_cast<const uint8_t*>(p.b) + (size_t)z * p.sb * ea;
        Cp = static_cast<uint8_t*>(p.c) + (size_t)z * p.sc * ec;
    }
    float acc = 0.0f;
    for (uint32_t l0 = 0; l0 < p.k; l0 += 16) {
        // As[tx][ty] = op(A)(blockrow + tx, l0 + ty); Bs[ty][tx] = op(B)(l0 + ty, blockcol + tx)
        {
            const uint32_t r = blockIdx.x * 16 + tx, l = l0 + ty;
            float v = 0.0f;
            if (r < p.m && l < p.k) v = ld_elem(A, p.ta ? (size_t)l + (size_t)r * p.lda : (size_t)r + (size_t)l * p.lda, p.at);
            As[tx][ty] = v;
        }
        {
            const uint32_t l = l0 + ty, cidx = blockIdx.y * 16 + tx;
            float v = 0.0f;
            if (cidx < p.n && l < p.k) v = ld_elem(B, p.tb ? (size_t)cidx + (size_t)l * p.ldb : (size_t)l + (size_t)cidx * p.ldb, p.bt);
            Bs[ty][tx] = v;
        }
        __syncthreads();
#pragma unroll
        for (int l = 0; l < 16; l++) acc = fmaf(As[tx][l], Bs[l][ty], acc);
        __syncthreads();
    }
    if (i < p.m && j < p.n) {
        const float alpha = p.alpha_ptr ? load_scalar(p.alpha_ptr, p.scalar_f16) : p.alpha;
        const float beta = p.beta_ptr ? load_scalar(p.beta_ptr, p.scalar_f16) : p.beta;
        const size_t ci = (size_t)j * p.ldc + i;
        float r = alpha * acc;
        if (beta != 0.0f) r += beta * ld_elem(Cp, ci, p.ct);
        st_elem(Cp, ci, p.ct, r);
    }
}

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

unsigned int* err_ptr() {
    static CfiSymbolPtr<unsigned int> p;
    return p.get(g_gemm_error);
}

int scalar_kind(int compute_type) {  // 0 f16, 1 f32, -1 unsupported (plan.rs:84-95)
    switch (compute_type) {
    case 64: case 65: case CFI_R_16F: return 0;
    case 68: case 69: case 74: case 75: case 77: case CFI_R_32F: return 1;
    default: return -1;
    }
}

bool dtype_ok(int t) { return t == CFI_R_32F || t == CFI_R_16F || t == CFI_R_16BF; }

}  // namespace

// Split-K workspace (fp32 partial tiles): the calling stream's own buffer (stream_state.cpp),
// grown outside stream capture only; nullptr (no split) when it would have to grow under capture.
static float* splitk_workspace(size_t bytes, cudaStream_t stream) {
    int err = 0;
    return static_cast<float*>(cfi_stream_buffer(CFI_BUF_SPLITK, bytes, stream, &err));
}

// Shared tensor-core launcher (the cuBLAS-compatible GEMM and the prefill mul_mat_q use it).
// Returns 0 on launch, -1 when the descriptor cannot be expressed with tensor maps (the caller
// then takes another path), or a CUDA error code.
int cfi_tc_gemm(const TcGemm& d, cudaStream_t stream) {
    PFN_encodeTiled enc = encode_fn();
    if (!enc) return -1;
    if ((d.lda % 8) || (d.ldb % 8) || (d.a_plane % 8) || (d.b_plane % 8) || d.k == 0 ||
        (reinterpret_cast<uintptr_t>(d.a) & 15) || (reinterpret_cast<uintptr_t>(d.b) & 15) || d.nch == 0 || d.nsamples == 0 ||
        d.chr == 0 || d.smr == 0 || d.nch % d.chr)
        return -1;
    const uint32_t planes = d.nch * d.nsamples;
    // balanced tiles; a multiple of 32 columns when there are several (the epilogue writes
    // whole 32-column chunks)
    const uint32_t tiles_n = (d.n + 255) / 256;
    const uint32_t per = (d.n + tiles_n - 1) / tiles_n;
    // CTA pairs (2-SM MMA, half-width B tiles) for more than one 128-row tile; CFI_GEMM_2SM=0 off
    // pairs pay off once the single-SM grid needs two or more waves (measured: single-wave, short-K
    // shapes are faster on single SMs)
    const char* e2 = getenv("CFI_GEMM_2SM");
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    }
    const uint64_t ctas1 = (uint64_t)((d.m + BM - 1) / BM) * tiles_n * planes;
    const bool pair = d.m > (uint32_t)BM && (e2 ? strcmp(e2, "0") != 0 : ctas1 >= 2ull * (uint64_t)sms);
    const uint32_t bn = (tiles_n > 1 || pair) ? (per + 31) / 32 * 32 : (per + 15) / 16 * 16;
    const CUtensorMapDataType dt = d.fmt == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap ta, tb, tcm;
    cuuint64_t da[3] = {d.k, d.m, d.a_planes};
    cuuint64_t sA[2] = {d.lda * 2, d.a_plane * 2};
    cuuint64_t db[3] = {d.k, d.n, planes};
    cuuint64_t sB[2] = {d.ldb * 2, d.b_plane * 2};
    cuuint32_t boxa[3] = {BK, BM, 1}, boxb[3] = {BK, pair ? bn / 2 : bn, 1}, es[3] = {1, 1, 1};
    if (enc(&ta, dt, 3, const_cast<void*>(d.a), da, sA, boxa, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        enc(&tb, dt, 3, const_cast<void*>(d.b), db, sB, boxb, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return -1;
    // C through TMA stores: f32, beta 0 known on the host, 16-byte multiple strides, aligned base
    memset(&tcm, 0, sizeof tcm);
    bool tma_c = d.c_type == CFI_R_32F && !d.alpha_ptr && !d.beta_ptr && d.beta == 0.0f && (d.ldc % 4) == 0 &&
                 (reinterpret_cast<uintptr_t>(d.c) & 15) == 0 && (d.nch == 1 || d.c_zstride % 4 == 0) &&
                 (d.nsamples == 1 || d.c_wstride % 4 == 0);
    if (tma_c) {
        const cuuint64_t s1 = d.ldc * 4;
        const cuuint64_t s2 = d.nch > 1 ? (cuuint64_t)d.c_zstride * 4 : s1 * d.n;
        const cuuint64_t s3 = d.nsamples > 1 ? (cuuint64_t)d.c_wstride * 4 : s2 * d.nch;
        cuuint64_t dc[4] = {d.m, d.n, d.nch, d.nsamples};
        cuuint64_t scs[3] = {s1, (s2 + 15) & ~(cuuint64_t)15, (s3 + 15) & ~(cuuint64_t)15};
        cuuint32_t boxc[4] = {32, 32, 1, 1}, esc[4] = {1, 1, 1, 1};
        tma_c = enc(&tcm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, d.c, dc, scs, boxc, esc, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    // split K when the output tiles fill under half the SMs and K is deep (CFI_GEMM_SPLITK=0 off)
    uint32_t splits = 1, kchunk = (d.k + BK - 1) / BK;
    float* ws = nullptr;
    uint32_t ld_ws = 0;
    CUtensorMap wsm;
    {
        const char* es = getenv("CFI_GEMM_SPLITK");
        const uint64_t tiles = (uint64_t)((d.m + BM - 1) / BM) * tiles_n * planes;
        const uint32_t ksteps = kchunk;
        if (!pair && !(es && strcmp(es, "0") == 0) && tiles * 2 <= (uint64_t)sms && ksteps >= 16) {
            uint32_t sp = std::min<uint32_t>((uint32_t)(sms / tiles), ksteps / 8);
            if (sp >= 2) {
                const uint32_t kc = (ksteps + sp - 1) / sp;
                sp = (ksteps + kc - 1) / kc;
                ld_ws = (d.m + 3) / 4 * 4;
                const size_t bytes = (size_t)sp * planes * d.n * ld_ws * 4;
                ws = splitk_workspace(bytes, stream);
                if (ws) {
                    cuuint64_t dw[4] = {d.m, d.n, planes, sp};
                    cuuint64_t sw[3] = {(cuuint64_t)ld_ws * 4, (cuuint64_t)ld_ws * 4 * d.n, (cuuint64_t)ld_ws * 4 * d.n * planes};
                    cuuint32_t bw[4] = {32, 32, 1, 1}, ew[4] = {1, 1, 1, 1};
                    if (enc(&wsm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ws, dw, sw, bw, ew, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
                        splits = sp;
                        kchunk = kc;
                    }
                }
            }
        }
    }
    GemmArgs g;
    g.splits = splits;
    g.kchunk = kchunk;
    g.c = d.c;
    g.c_zstride = d.c_zstride;
    g.c_wstride = d.c_wstride;
    g.c_type = d.c_type;
    g.ldc = (int)d.ldc;
    g.m = d.m;
    g.n = d.n;
    g.k = d.k;
    g.bn = bn;
    g.nch = d.nch;
    g.chr = d.chr;
    g.smr = d.smr;
    g.nch_x = d.nch / d.chr;
    g.alpha = d.alpha;
    g.beta = d.beta;
    g.alpha_ptr = d.alpha_ptr;
    g.beta_ptr = d.beta_ptr;
    g.scalar_f16 = d.scalar_f16;
    g.tma_c = tma_c ? 1 : 0;
    g.err = err_ptr();
    // programmatic dependent launch (CFI_PDL=0 turns it off): the prologue overlaps the tail of
    // the previous kernel; the kernel waits for it before its first tensor load
    const char* ep = getenv("CFI_PDL");
    const bool pdl = !(ep && strcmp(ep, "0") == 0);
    static CfiPerDeviceOnce attr;
    cfi_once_per_device(attr, [] {
        cudaFuncSetAttribute(cfi_gemm_tc<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
        cudaFuncSetAttribute(cfi_gemm_tc<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
        cudaFuncSetAttribute(cfi_gemm_tc2<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM2_BYTES);
        cudaFuncSetAttribute(cfi_gemm_tc2<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM2_BYTES);
    });
    if (pair) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * ((d.m + 2 * BM - 1) / (2 * BM)), (d.n + bn - 1) / bn, planes);
        cfg.blockDim = dim3(THREADS, 1, 1);
        cfg.dynamicSmemBytes = SMEM2_BYTES;
        cfg.stream = stream;
        cudaLaunchAttribute at[2];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        if (pdl) {
            at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            at[1].val.programmaticStreamSerializationAllowed = 1;
            cfg.numAttrs = 2;
        }
        cudaError_t e = d.fmt == 0 ? cudaLaunchKernelEx(&cfg, cfi_gemm_tc2<0>, ta, tb, tcm, g)
                                   : cudaLaunchKernelEx(&cfg, cfi_gemm_tc2<1>, ta, tb, tcm, g);
        return (int)e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((d.m + BM - 1) / BM, (d.n + bn - 1) / bn, planes * splits);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    if (splits > 1) {
        g.tma_c = 1;  // partials go to the workspace through its tensor map
        cudaError_t e = d.fmt == 0 ? cudaLaunchKernelEx(&cfg, cfi_gemm_tc<0>, ta, tb, wsm, g)
                                   : cudaLaunchKernelEx(&cfg, cfi_gemm_tc<1>, ta, tb, wsm, g);
        if (e != cudaSuccess) return (int)e;
        ReduceArgs r;
        r.ws = ws;
        r.ld_ws = ld_ws;
        r.m = d.m;
        r.n = d.n;
        r.planes = planes;
        r.splits = splits;
        r.c = d.c;
        r.c_type = d.c_type;
        r.ldc = (long long)d.ldc;
        r.c_zstride = d.c_zstride;
        r.c_wstride = d.c_wstride;
        r.nch = d.nch;
        r.alpha = d.alpha;
        r.beta = d.beta;
        r.alpha_ptr = d.alpha_ptr;
        r.beta_ptr = d.beta_ptr;
        r.scalar_f16 = d.scalar_f16;
        cudaLaunchConfig_t rc = {};
        const uint64_t nthr = (uint64_t)((d.m + 3) / 4) * d.n * planes;
        rc.gridDim = dim3((uint32_t)((nthr + 255) / 256), 1, 1);
        rc.blockDim = dim3(256, 1, 1);
        rc.stream = stream;
        rc.attrs = at;
        rc.numAttrs = pdl ? 1 : 0;
        return (int)cudaLaunchKernelEx(&rc, cfi_gemm_splitk_reduce, r);
    }
    return (int)(d.fmt == 0 ? cudaLaunchKernelEx(&cfg, cfi_gemm_tc<0>, ta, tb, tcm, g)
                            : cudaLaunchKernelEx(&cfg, cfi_gemm_tc<1>, ta, tb, tcm, g));
}

float* cfi_splitk_workspace(size_t bytes, cudaStream_t stream) { return splitk_workspace(bytes, stream); }

int cfi_splitk_reduce_f32(const float* ws, uint32_t ld_ws, uint32_t m, uint32_t n, uint32_t planes, uint32_t splits,
                          float* c, long long ldc, long long c_zstride, long long c_wstride, uint32_t nch,
                          cudaStream_t stream, bool pdl) {
    ReduceArgs r;
    r.ws = ws;
    r.ld_ws = ld_ws;
    r.m = m;
    r.n = n;
    r.planes = planes;
    r.splits = splits;
    r.c = c;
    r.c_type = CFI_R_32F;
    r.ldc = ldc;
    r.c_zstride = c_zstride;
    r.c_wstride = c_wstride;
    r.nch = nch;
    r.alpha = 1.0f;
    r.beta = 0.0f;
    r.alpha_ptr = nullptr;
    r.beta_ptr = nullptr;
    r.scalar_f16 = 0;
    cudaLaunchConfig_t rc = {};
    const uint64_t nthr = (uint64_t)((m + 3) / 4) * n * planes;
    rc.gridDim = dim3((uint32_t)((nthr + 255) / 256), 1, 1);
    rc.blockDim = dim3(256, 1, 1);
    rc.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    rc.attrs = at;
    rc.numAttrs = pdl ? 1 : 0;
    return (int)cudaLaunchKernelEx(&rc, cfi_gemm_splitk_reduce, r);
}

// Reads and clears the error word of the GEMM kernel's bounded waits (folded into cfi_device_error).
unsigned int cfi_gemm_error_take() {
    unsigned int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof v) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaMemcpyToSymbol(g_gemm_error, &z, sizeof z);
    return v;
}

struct cfi_blas {
    cudaStream_t stream = nullptr;
    int pointer_mode = CFI_POINTER_MODE_HOST;
    int last_path = 0;
};

extern "C" {

int cfi_blas_validate(int transa, int transb, int m, int n, int k, int lda, int ldb, int ldc, int a_type, int b_type,
                      int c_type, int compute_type) {
    if (transa < 0 || transa > 2 || transb < 0 || transb > 2) return CFI_BLAS_INVALID_VALUE;
    if (m < 0 || n < 0 || k < 0) return CFI_BLAS_INVALID_VALUE;
    const int rows_a = transa ? k : m, rows_b = transb ? n : k;
    if (lda < (rows_a > 1 ? rows_a : 1) || ldb < (rows_b > 1 ? rows_b : 1) || ldc < (m > 1 ? m : 1))
        return CFI_BLAS_INVALID_VALUE;
    if (!dtype_ok(a_type) || !dtype_ok(b_type) || !dtype_ok(c_type)) return CFI_BLAS_NOT_SUPPORTED;
    const int sk = scalar_kind(compute_type);
    if (sk < 0) return CFI_BLAS_NOT_SUPPORTED;
    if (a_type != b_type) return CFI_BLAS_NOT_SUPPORTED;
    const bool ok = (a_type == CFI_R_32F && c_type == CFI_R_32F) ||
                    (a_type == CFI_R_16F && (c_type == CFI_R_16F || c_type == CFI_R_32F)) ||
                    (a_type == CFI_R_16BF && (c_type == CFI_R_16BF || c_type == CFI_R_32F));
    if (!ok) return CFI_BLAS_NOT_SUPPORTED;
    if (sk == 0 && (a_type != CFI_R_16F || c_type != CFI_R_16F)) return CFI_BLAS_NOT_SUPPORTED;
    return CFI_BLAS_SUCCESS;
}

int cfi_blas_create(cfi_blas** handle) {
    if (!handle) return CFI_BLAS_INVALID_VALUE;
    *handle = new (std::nothrow) cfi_blas();
    return *handle ? CFI_BLAS_SUCCESS : CFI_BLAS_ALLOC_FAILED;
}
int cfi_blas_destroy(cfi_blas* h) {
    if (!h) return CFI_BLAS_NOT_INITIALIZED;
    delete h;
    return CFI_BLAS_SUCCESS;
}
int cfi_blas_set_stream(cfi_blas* h, void* stream) {
    if (!h) return CFI_BLAS_NOT_INITIALIZED;
    h->stream = static_cast<cudaStream_t>(stream);
    return CFI_BLAS_SUCCESS;
}
int cfi_blas_get_stream(cfi_blas* h, void** stream) {
    if (!h) return CFI_BLAS_NOT_INITIALIZED;
    if (!stream) return CFI_BLAS_INVALID_VALUE;
    *stream = h->stream;
    return CFI_BLAS_SUCCESS;
}
int cfi_blas_set_pointer_mode(cfi_blas* h, int mode) {
    if (!h) return CFI_BLAS_NOT_INITIALIZED;
    if (mode != CFI_POINTER_MODE_HOST && mode != CFI_POINTER_MODE_DEVICE) return CFI_BLAS_INVALID_VALUE;
    h->pointer_mode = mode;
    return CFI_BLAS_SUCCESS;
}
int cfi_blas_last_path(cfi_blas* h) { return h ? h->last_path : 0; }

}  // extern "C"

namespace {

int gemm_common(cfi_blas* h, int transa, int transb, int m, int n, int k, const void* alpha, const void* A, int a_type,
                int lda, long long sa, const void* B, int b_type, int ldb, long long sb, const void* beta, void* C,
                int c_type, int ldc, long long sc, int batch, int compute_type, bool ptr_arrays) {
    if (!h) return CFI_BLAS_NOT_INITIALIZED;
    int st = cfi_blas_validate(transa, transb, m, n, k, lda, ldb, ldc, a_type, b_type, c_type, compute_type);
    if (st) return st;
    if (batch < 0) return CFI_BLAS_INVALID_VALUE;
    if (!alpha || !beta) return CFI_BLAS_INVALID_VALUE;
    h->last_path = 0;
    if (m == 0 || n == 0 || batch == 0) return CFI_BLAS_SUCCESS;
    const int sf16 = scalar_kind(compute_type) == 0;
    const bool dev_ptrs = h->pointer_mode == CFI_POINTER_MODE_DEVICE;
    float al = 0.0f, be = 0.0f;
    if (!dev_ptrs) {
        al = sf16 ? __half2float(*static_cast<const __half*>(alpha)) : *static_cast<const float*>(alpha);
        be = sf16 ? __half2float(*static_cast<const __half*>(beta)) : *static_cast<const float*>(beta);
    }
    const char* tc_env = getenv("CFI_GEMM_TC");
    const bool tc_allowed = !(tc_env && strcmp(tc_env, "0") == 0);
    const bool fmt16 = a_type == CFI_R_16F || a_type == CFI_R_16BF;
    const bool tc = tc_allowed && !ptr_arrays && fmt16 && transa == CFI_OP_T && transb == CFI_OP_N && k > 0 &&
                    compute_type != CFI_COMPUTE_32F_FAST_TF32 && lda % 8 == 0 && ldb % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(A) & 15) == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0 &&
                    (batch == 1 || ((sa % 8) == 0 && (sb % 8) == 0 && sa > 0 && sb > 0));
    // n <= 8 columns (decode attention): the skinny kernel (CFI_GEMM_SKINNY=0 off)
    const char* sk_env = getenv("CFI_GEMM_SKINNY");
    const bool skinny = !(sk_env && strcmp(sk_env, "0") == 0) && !ptr_arrays && fmt16 && b_type == a_type &&
                        transa == CFI_OP_T && transb == CFI_OP_N && n <= 8 && k > 0 && lda % 8 == 0 && ldb % 8 == 0 &&
                        (reinterpret_cast<uintptr_t>(A) & 15) == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0 &&
                        batch <= 65535 && (batch == 1 || ((sa % 8) == 0 && (sb % 8) == 0));
    if (skinny) {
        SkinnyArgs q;
        q.a = A;
        q.b = B;
        q.c = C;
        q.sa = sa;
        q.sb = sb;
        q.sc = sc;
        q.lda = lda;
        q.ldb = ldb;
        q.ldc = ldc;
        q.ct = c_type;
        q.m = (uint32_t)m;
        q.n = (uint32_t)n;
        q.k = (uint32_t)k;
        q.alpha = al;
        q.beta = be;
        q.alpha_ptr = dev_ptrs ? alpha : nullptr;
        q.beta_ptr = dev_ptrs ? beta : nullptr;
        q.scalar_f16 = sf16;
        const char* ep = getenv("CFI_PDL");
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)((m + 7) / 8), (unsigned)batch, 1);
        cfg.blockDim = dim3(256, 1, 1);
        cfg.stream = h->stream;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = (ep && strcmp(ep, "0") == 0) ? 0 : 1;
        cudaError_t e = a_type == CFI_R_16F ? cudaLaunchKernelEx(&cfg, cfi_gemm_skinny<0>, q)
                                            : cudaLaunchKernelEx(&cfg, cfi_gemm_skinny<1>, q);
        if (e != cudaSuccess) return CFI_BLAS_EXECUTION_FAILED;
        h->last_path = 3;
        return CFI_BLAS_SUCCESS;
    }
    if (tc) {
        TcGemm d;
        d.a = A;
        d.b = B;
        d.c = C;
        d.fmt = a_type == CFI_R_16F ? 0 : 1;
        d.m = (uint32_t)m;
        d.n = (uint32_t)n;
        d.k = (uint32_t)k;
        d.lda = (uint64_t)lda;
        d.ldb = (uint64_t)ldb;
        d.a_plane = batch > 1 ? (uint64_t)sa : (uint64_t)lda * m;
        d.b_plane = batch > 1 ? (uint64_t)sb : (uint64_t)ldb * n;
        d.a_planes = (uint32_t)batch;
        d.nch = (uint32_t)batch;
        d.nsamples = 1;
        d.chr = 1;
        d.smr = 1;
        d.c_type = c_type;
        d.ldc = (uint64_t)ldc;
        d.c_zstride = batch > 1 ? sc : (long long)ldc * n;
        d.c_wstride = 0;
        d.alpha = al;
        d.beta = be;
        d.alpha_ptr = dev_ptrs ? alpha : nullptr;
        d.beta_ptr = dev_ptrs ? beta : nullptr;
        d.scalar_f16 = sf16;
        const int rc = cfi_tc_gemm(d, h->stream);
        if (rc == 0) {
            h->last_path = 1;
            return CFI_BLAS_SUCCESS;
        }
        if (rc > 0) return CFI_BLAS_EXECUTION_FAILED;
    }
    SimtArgs p;
    p.a = A;
    p.b = B;
    p.c = C;
    p.sa = sa;
    p.sb = sb;
    p.sc = sc;
    p.lda = lda;
    p.ldb = ldb;
    p.ldc = ldc;
    p.ta = transa != 0;
    p.tb = transb != 0;
    p.at = a_type;
    p.bt = b_type;
    p.ct = c_type;
    p.m = (uint32_t)m;
    p.n = (uint32_t)n;
    p.k = (uint32_t)k;
    p.alpha = al;
    p.beta = be;
    p.alpha_ptr = dev_ptrs ? alpha : nullptr;
    p.beta_ptr = dev_ptrs ? beta : nullptr;
    p.scalar_f16 = sf16;
    p.ptrs = ptr_arrays ? 1 : 0;
    for (int z0 = 0; z0 < batch; z0 += 65535) {
        const int bz = batch - z0 < 65535 ? batch - z0 : 65535;
        SimtArgs q = p;
        if (ptr_arrays) {
            q.a = static_cast<const void* const*>(p.a) + z0;
            q.b = static_cast<const void* const*>(p.b) + z0;
            q.c = const_cast<void**>(static_cast<void* const*>(p.c) + z0);
        } else {
            const size_t ea = a_type == CFI_R_32F ? 4 : 2, ec = c_type == CFI_R_32F ? 4 : 2;
            q.a = static_cast<const uint8_t*>(p.a) + (size_t)z0 * sa * ea;
            q.b = static_cast<const uint8_t*>(p.b) + (size_t)z0 * sb * ea;
            q.c = static_cast<uint8_t*>(p.c) + (size_t)z0 * sc * ec;
        }
        dim3 grid((m + 15) / 16, (n + 15) / 16, bz);
        if (grid.y > 65535) return CFI_BLAS_NOT_SUPPORTED;
        cfi_gemm_simt<<<grid, 256, 0, h->stream>>>(q);
        if (cudaGetLastError() != cudaSuccess) return CFI_BLAS_EXECUTION_FAILED;
    }
    h->last_path = 2;
    return CFI_BLAS_SUCCESS;
}

}  // namespace

extern "C" {

int cfi_blas_gemm_ex(cfi_blas* h, int transa, int transb, int m, int n, int k, const void* alpha, const void* A,
                     int a_type, int lda, const void* B, int b_type, int ldb, const void* beta, void* C, int c_type,
                     int ldc, int compute_type, int algo) {
    (void)algo;
    return gemm_common(h, transa, transb, m, n, k, alpha, A, a_type, lda, 0, B, b_type, ldb, 0, beta, C, c_type, ldc, 0, 1,
                       compute_type, false);
}

int cfi_blas_gemm_strided_batched_ex(cfi_blas* h, int transa, int transb, int m, int n, int k, const void* alpha,
                                     const void* A, int a_type, int lda, long long stride_a, const void* B, int b_type,
                                     int ldb, long long stride_b, const void* beta, void* C, int c_type, int ldc,
                                     long long stride_c, int batch_count, int compute_type, int algo) {
    (void)algo;
    return gemm_common(h, transa, transb, m, n, k, alpha, A, a_type, lda, stride_a, B, b_type, ldb, stride_b, beta, C,
                       c_type, ldc, stride_c, batch_count, compute_type, false);
}

int cfi_blas_gemm_batched_ex(cfi_blas* h, int transa, int transb, int m, int n, int k, const void* alpha,
                             const void* const A[], int a_type, int lda, const void* const B[], int b_type, int ldb,
                             const void* beta, void* const C[], int c_type, int ldc, int batch_count, int compute_type,
                             int algo) {
    (void)algo;
    if (batch_count > 0 && (!A || !B || !C)) return CFI_BLAS_INVALID_VALUE;
    return gemm_common(h, transa, transb, m, n, k, alpha, A, a_type, lda, 0, B, b_type, ldb, 0, beta,
                       const_cast<void*>(static_cast<const void*>(C)), c_type, ldc, 0, batch_count, compute_type, true);
}

int cfi_blas_sgemm(cfi_blas* h, int transa, int transb, int m, int n, int k, const float* alpha, const float* A, int lda,
                   const float* B, int ldb, const float* beta, float* C, int ldc) {
    return gemm_common(h, transa, transb, m, n, k, alpha, A, CFI_R_32F, lda, 0, B, CFI_R_32F, ldb, 0, beta, C, CFI_R_32F,
                       ldc, 0, 1, CFI_COMPUTE_32F, false);
}

}  // extern "C"
