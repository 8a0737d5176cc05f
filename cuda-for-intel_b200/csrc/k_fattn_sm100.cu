// k_fattn_sm100.cu -- the native flash_attn_ext_f16 (prefill FlashAttention) on the 5th-generation
// tensor cores of sm_100a.
//
// Parameters: ggml-cuda's flash_attn_ext_f16<D, D, ncols1, ncols2, nwarps, ntiles, false, false>
// (Q, K, V, mask, sinks, KV_max, dst, dst_meta, f32 scale, max_bias, m0, m1, u32 n_head_log2, f32
// logit_softcap, i32 ne00..ne03, nb01..nb03, ne10..ne13, nb11, nb12, i64 nb13, nb21, nb22, i64 nb23,
// ne31..ne33, nb31, nb32, i64 nb33; cuda-for-intel src/subst/fattn.rs:45-66, mod.rs:239-242).
// Q f32 [seq][head][query][D] (byte strides nb01..nb03), K/V f16 [seq][kv head][key][D], mask f16
// [seq % ne33][query][key] (row stride nb31), dst f32 [seq][query][head][D].  Supported as in the
// reference (mod.rs:27-54): D = 64 or 128, no sinks, max_bias 0, no softcap, GQA; plus 16-byte
// aligned K/V rows (TMA).
//
// One CTA of 608 threads per (128-query tile, head, sequence):
//   * warps 0-15 run the softmax, four warps per TMEM lane quadrant: thread (row, quarter) owns one
//     query row (TMEM lane) and 32 of the 128 key columns of a chunk.  They convert Q (x scale x
//     log2 e) to fp16 in the 128-byte swizzled K-major layout, then per chunk read their score
//     columns from TMEM, add the mask (16-byte loads issued before the wait), exchange the
//     quarter-row maxima through shared memory (one named barrier per quadrant), run the online
//     softmax in log2 units (row max, ex2, sum in fp32) with lazy rescaling -- the output
//     accumulator in TMEM and the sum are rescaled only when the row max grows by more than 2^8 --
//     and write their quarter of P (fp16) as the A operand of the PV product, alternating between
//     two P buffers for D 64; at the end O / l goes to dst;
//   * before the loop the tile's key range is cut to the chunks where some valid query sees some
//     key (mask not -inf), so a causal prompt skips the chunks above the diagonal;
//   * warps 17 and 18 stream K and V chunks with TMA (two stages each, 128 keys x 64 dims per box,
//     keys past the end read as zero); a K stage is free once its S product is done, so K loads run
//     ahead of the PV products;
//   * one thread of warp 16 issues S = Q K^T (M 128, N 128, K = D) into one of two TMEM score
//     buffers and O += P V (M 128, N = D, K 128; V is the MN-major B operand) into the TMEM output.
// TMEM: scores at columns 0 and 128, output at 256.  Every wait is bounded (error word + abort).
// Arithmetic: fp16 Q and P (as ggml's tensor-core kernel rounds them), fp32 scores, softmax and
// accumulation; results agree with the exact softmax attention to about 2e-4 relative L2 (nmse
// about 4e-8 on the reference's probe cases), the error of the two fp16 roundings.
#include <cuda.h>

#include <string.h>

#include <algorithm>
#include <mutex>

#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "sm100_ptx.cuh"
#include "subst_host.hpp"

static __device__ unsigned int g_fattn_error;

namespace {

using namespace sm100;

constexpr int FA_BM = 128;       // queries per CTA (TMEM lanes)
constexpr int FA_BN = 128;       // keys per chunk
constexpr int FA_SOFTMAX_WARPS = 16, FA_MMA_WARP = 16, FA_TMA_WARP = 17, FA_TMA_V_WARP = 18;
constexpr int FA_NQ = 4;                 // softmax threads per query row (key quarters)
constexpr int FA_KQ = FA_BN / FA_NQ;     // keys per softmax thread and chunk
constexpr int FA_FLAG_WORDS = 8;  // chunk-visibility bits: key ranges up to 256 chunks are cut
constexpr int FA_THREADS = 608;  // warps 0-15 softmax (four per TMEM sub-partition), 16 MMA, 17-18 TMA
constexpr uint32_t FA_TMEM_COLS = 512;
constexpr float FA_LOG2E = 1.4426950408889634f;
constexpr float FA_RESCALE_LOG2 = 8.0f;  // rescale O and l only when the row max grows by more than 2^8

CFI_DEV float ex2_approx(float x) {  // 2^x (PTX ex2.approx; -inf -> +0)
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct FaArgs {
    const uint8_t* q;
    float* dst;
    const uint8_t* mask;
    float scale;
    int ne01, ne02, ne03, ne11, ne12;
    long long nb01, nb02, nb03;   // Q byte strides
    long long nb31, nb33;         // mask byte strides (row, sequence)
    int ne31, ne33;               // mask rows, mask sequences
    int nchunks;
    unsigned int* err;
};

// P buffers: two for D 64 (chunk j's P is written while the PV product of chunk j-1 runs); one for
// D 128, where a second 32 KB buffer does not fit next to the 128 KB of K/V stages
template <int D> constexpr int fa_pbufs() { return D == 64 ? 2 : 1; }

template <int D>
constexpr size_t fa_smem_bytes() {
    return 1024 + (size_t)FA_BM * D * 2 + 4 * (size_t)FA_BN * D * 2 + fa_pbufs<D>() * (size_t)FA_BM * FA_BN * 2 + 256;
}

CFI_DEV void st_chunk16(uint8_t* atom, int r, int c, uint32_t a, uint32_t b, uint32_t cc, uint32_t d) {
    *reinterpret_cast<uint4*>(atom + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(a, b, cc, d);
}
CFI_DEV uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

template <int D>
__global__ void __launch_bounds__(FA_THREADS, 1)
    cfi_fattn_tc(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, const FaArgs a) {
    constexpr int DB = D / 64;                          // 64-dim blocks (one swizzle atom column each)
    constexpr int DQ = D / FA_NQ;                       // output columns per softmax thread
    constexpr uint32_t QBYTES = FA_BM * D * 2;
    constexpr uint32_t KVBYTES = FA_BN * D * 2;         // one K or V stage
    constexpr uint32_t BLK_Q = FA_BM * 128, BLK_KV = FA_BN * 128;  // bytes of one 64-dim block
    extern __shared__ uint8_t smem_raw[];
    __shared__ float xmax[2][FA_NQ][FA_BM];  // partial row maxima (chunk parity, key quarter, row)
    __shared__ float xsum[FA_NQ][FA_BM];     // final partial row sums (key quarter, row)
    __shared__ uint32_t chunk_vis[FA_FLAG_WORDS];  // chunks with a visible key for some valid query
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + QBYTES;
    uint8_t* sV = sK + 2 * KVBYTES;
    constexpr int NPB = fa_pbufs<D>();
    uint8_t* sP = sV + 2 * KVBYTES;  // NPB P buffers; chunk j uses buffer j % NPB
    constexpr uint32_t PBYTES = FA_BM * FA_BN * 2;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sP + NPB * PBYTES);
    uint64_t* k_full = bars;        // [2] TMA bytes of K of a chunk
    uint64_t* k_empty = bars + 2;   // [2] the S product of the chunk has read K
    uint64_t* s_full = bars + 4;    // [2] scores of a chunk in TMEM
    uint64_t* s_empty = bars + 6;   // [2] softmax warps have read them (8 arrivals)
    uint64_t* p_full = bars + 8;    // [NPB] P of a chunk in its buffer, output rescaled if needed (8 arrivals)
    uint64_t* pv_done = bars + 10;  // [NPB] O += P V of a chunk completed (its P buffer is free again)
    uint64_t* q_ready = bars + 12;  // fp16 Q in shared memory (8 arrivals)
    uint64_t* v_full = bars + 13;   // [2] TMA bytes of V of a chunk
    uint64_t* v_empty = bars + 15;  // [2] the PV product of the chunk has read V
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q0 = blockIdx.x * FA_BM, head = blockIdx.y, seq = blockIdx.z;
    const int kvh = head / (a.ne02 / a.ne12);

    if (tid == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_empty[i], FA_SOFTMAX_WARPS);
            mbar_init(&p_full[i], FA_SOFTMAX_WARPS);  // (the second pair is unused when NPB == 1)
            mbar_init(&pv_done[i], 1);
        }
        mbar_init(q_ready, FA_SOFTMAX_WARPS);
        *abort_flag = 0;
        for (int w = 0; w < FA_FLAG_WORDS; w++) chunk_vis[w] = 0u;
        fence_mbar_init();
    }
    if (warp == FA_MMA_WARP) {
        tmem_alloc(tmem_slot, FA_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();  // Q, K, V and the mask may come from the previous kernel

    // softmax thread: row r (TMEM lane) and key quarter h (columns 32 h .. 32 h + 31 of a chunk)
    const int r = 32 * (warp & 3) + lane, h = (warp >> 2) & 3, q = q0 + r;
    const bool qvalid = q < a.ne01;
    const uint16_t* mrow = nullptr;
    if (warp < FA_SOFTMAX_WARPS && a.mask && q < a.ne31)
        mrow = reinterpret_cast<const uint16_t*>(a.mask + (size_t)(seq % a.ne33) * a.nb33 + (size_t)q * a.nb31);
    // ---- the tile's key range: the chunks where some valid query sees some key (mask not -inf);
    // fully masked chunks before and after are skipped, as the reference skips them
    // (fattn.rs:258-262).  Every thread tests its row's half of every chunk with independent loads
    // into register bits, then ORs them into shared flags ----
    const int nall = a.nchunks;
    const bool cut = a.mask != nullptr && nall <= 32 * FA_FLAG_WORDS;
    if (warp < FA_SOFTMAX_WARPS && cut && qvalid) {
        uint32_t bits[FA_FLAG_WORDS];
#pragma unroll
        for (int w = 0; w < FA_FLAG_WORDS; w++) bits[w] = 0u;
        const bool vec = mrow && ((reinterpret_cast<uintptr_t>(a.mask) | (uintptr_t)a.nb31 | (uintptr_t)a.nb33) & 15) == 0;
        // vector path: the loads of chunk j+1 are issued before chunk j is tested
        const uint4 ninf4 = make_uint4(0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u);
        auto load_chunk = [&](int j, uint4 (&w)[FA_KQ / 8]) {
            const int k0 = j * FA_BN + FA_KQ * h;
#pragma unroll
            for (int t = 0; t < FA_KQ / 8; t++)
                w[t] = (j < nall && k0 + 8 * t < a.ne11) ? __ldg(reinterpret_cast<const uint4*>(mrow + k0 + 8 * t)) : ninf4;
        };
        uint4 wn[FA_KQ / 8];
        if (vec) load_chunk(0, wn);
        for (int j = 0; j < nall; j++) {
            const int k0 = j * FA_BN + FA_KQ * h;
            bool any = false;
            if (!mrow) {
                any = k0 < a.ne11;  // no mask row for this query: every key counts
            } else if (vec) {
                uint4 w[FA_KQ / 8];
#pragma unroll
                for (int t = 0; t < FA_KQ / 8; t++) w[t] = wn[t];
                load_chunk(j + 1, wn);
#pragma unroll
                for (int t = 0; t < FA_KQ / 8; t++) {
                    const uint32_t x[4] = {w[t].x, w[t].y, w[t].z, w[t].w};
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        const uint32_t hv = (x[e >> 1] >> (16 * (e & 1))) & 0xffffu;
                        any = any || (k0 + 8 * t + e < a.ne11 && hv != 0xfc00u);
                    }
                }
            } else {
#pragma unroll 8
                for (int c = 0; c < FA_KQ; c++) any = any || (k0 + c < a.ne11 && mrow[k0 + c] != 0xfc00u);
            }
            if (any) bits[j >> 5] |= 1u << (j & 31);
        }
#pragma unroll
        for (int w = 0; w < FA_FLAG_WORDS; w++)
            if (bits[w]) atomicOr(&chunk_vis[w], bits[w]);
    }
    __syncthreads();
    int jb = 0, je = nall;  // chunks [jb, je)
    if (cut) {
        jb = nall;
        je = 0;
        for (int j = 0; j < nall; j++)
            if (chunk_vis[j >> 5] >> (j & 31) & 1u) {
                jb = min(jb, j);
                je = j + 1;
            }
        if (je <= jb) jb = je = 0;
    }
    const int nch = je - jb;

    if (warp == FA_TMA_WARP || warp == FA_TMA_V_WARP) {
        // ================= K (warp 9) and V (warp 10) chunks by TMA, each ring on its own =================
        if (lane == 0) {
            const bool isk = warp == FA_TMA_WARP;
            const CUtensorMap* map = isk ? &tk : &tv;
            uint8_t* ring = isk ? sK : sV;
            uint64_t* full = isk ? k_full : v_full;
            uint64_t* empty = isk ? k_empty : v_empty;
            prefetch_tmap(map);
            for (int j = 0; j < nch; j++) {
                const int st = j & 1;
                if (!mbar_wait(&empty[st], ((uint32_t)(j >> 1) & 1) ^ 1, abort_flag)) {
                    cfi_set_error(a.err, 0xfa100 + st);
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full[st], KVBYTES);
#pragma unroll
                for (int b = 0; b < DB; b++)
                    tma_load_4d(ring + st * KVBYTES + b * BLK_KV, map, 64 * b, (jb + j) * FA_BN, kvh, seq, &full[st]);
            }
        }
        __syncwarp();
    } else if (warp == FA_MMA_WARP) {
        // ================= MMA issue =================
        if (lane == 0 && nch > 0) {
            const uint32_t id_s = idesc_f16(FA_BM, FA_BN, 0);
            const uint32_t id_o = idesc_f16(FA_BM, D, 0) | (1u << 16);  // B (V) MN-major
            bool ok = mbar_wait(q_ready, 0, abort_flag);
            for (int j = 0; ok && j <= nch; j++) {
                if (j < nch) {
                    const int st = j & 1;
                    ok = mbar_wait(&k_full[st], (uint32_t)(j >> 1) & 1, abort_flag);
                    if (ok && j >= 2) ok = mbar_wait(&s_empty[st], (uint32_t)((j >> 1) - 1) & 1, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t qa = smem_u32(sQ), kb = smem_u32(sK + st * KVBYTES);
#pragma unroll
                    for (int kk = 0; kk < D / 16; kk++) {
                        const uint32_t off_q = (kk >> 2) * BLK_Q + (kk & 3) * 32, off_k = (kk >> 2) * BLK_KV + (kk & 3) * 32;
                        mma_f16(tmem + st * FA_BN, sw128_kmajor_desc(qa + off_q), sw128_kmajor_desc(kb + off_k), id_s,
                                kk > 0 ? 1u : 0u);
                    }
                    mma_commit(&s_full[st]);
                    mma_commit(&k_empty[st]);
                }
                if (j >= 1) {
                    const int jp = j - 1, st = jp & 1, pb = jp % NPB;
                    ok = mbar_wait(&p_full[pb], (uint32_t)(jp / NPB) & 1, abort_flag);
                    if (ok) ok = mbar_wait(&v_full[st], (uint32_t)(jp >> 1) & 1, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t pa = smem_u32(sP + pb * PBYTES), vb = smem_u32(sV + st * KVBYTES);
#pragma unroll
                    for (int kk = 0; kk < FA_BN / 16; kk++) {
                        const uint32_t off_p = (kk >> 2) * BLK_Q + (kk & 3) * 32;
                        mma_f16(tmem + 256, sw128_kmajor_desc(pa + off_p), sw128_mnmajor_desc(vb + kk * 16 * 128, BLK_KV),
                                id_o, (jp > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit(&pv_done[pb]);
                    mma_commit(&v_empty[st]);
                }
            }
            if (!ok) {
                cfi_set_error(a.err, 0xfa200);
                *abort_flag = 1;
            }
        }
        __syncwarp();
    } else {
        // ================= softmax warps: (row, key half) per thread =================
        // scores are kept in log2 units: Q is scaled by scale * log2(e) and the mask by log2(e),
        // so every softmax weight is one ex2
        const float qscale = a.scale * FA_LOG2E;
        {
            // this half of the row: every load issued before any conversion or store
            const float* qrow = reinterpret_cast<const float*>(a.q + (size_t)seq * a.nb03 + (size_t)head * a.nb02 +
                                                               (size_t)(qvalid ? q : 0) * a.nb01) + DQ * h;
            float f[DQ];
            if (qvalid && (reinterpret_cast<uintptr_t>(qrow) & 15) == 0) {
#pragma unroll
                for (int i = 0; i < DQ / 4; i++) {
                    const float4 t = __ldg(reinterpret_cast<const float4*>(qrow) + i);
                    f[4 * i] = t.x;
                    f[4 * i + 1] = t.y;
                    f[4 * i + 2] = t.z;
                    f[4 * i + 3] = t.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < DQ; i++) f[i] = qvalid ? __ldg(qrow + i) : 0.0f;
            }
#pragma unroll
            for (int gi = 0; gi < DQ / 8; gi++) {
                const int g = h * (DQ / 8) + gi, b = g / 8, c = g % 8;  // 8-dim group of this quarter
                const float* e = f + 8 * gi;
                st_chunk16(sQ + b * BLK_Q, r, c, pack_h2(e[0] * qscale, e[1] * qscale), pack_h2(e[2] * qscale, e[3] * qscale),
                           pack_h2(e[4] * qscale, e[5] * qscale), pack_h2(e[6] * qscale, e[7] * qscale));
            }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_ready);

        const bool mvec = mrow && ((reinterpret_cast<uintptr_t>(a.mask) | (uintptr_t)a.nb31 | (uintptr_t)a.nb33) & 15) == 0;
        const uint32_t trow = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        const int quad_bar = 1 + (warp & 3);  // the four warps (key quarters) of this TMEM quadrant
        // this thread's DQ output columns in TMEM: ld / st of 16 or 32 columns
        auto o_ld = [&](uint32_t (&v)[DQ]) {
            if constexpr (DQ == 16) tmem_ld16(trow + 256 + DQ * h, v); else tmem_ld32(trow + 256 + DQ * h, v);
        };
        auto o_st = [&](const uint32_t (&v)[DQ]) {
            if constexpr (DQ == 16) tmem_st16(trow + 256 + DQ * h, v); else tmem_st32(trow + 256 + DQ * h, v);
        };
        // Online softmax with lazy rescaling: P = 2^(s - m_used) with m_used the row max at the last
        // rescale; O and l are rescaled only when the chunk's max exceeds m_used by more than
        // FA_RESCALE_LOG2 (P then stays below 2^FA_RESCALE_LOG2, far inside fp16), so most chunks
        // neither touch O nor wait for the previous PV product.  With two P buffers, chunk j's P
        // is written while the PV product of chunk j-1 runs.
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < nch; j++) {
            const int st = j & 1, key0 = (jb + j) * FA_BN + FA_KQ * h;
            // this quarter's 32 mask values, loaded before waiting on the scores (none without a
            // mask row); `full`: all 32 keys exist, so no per-key range test
            const bool full = key0 + FA_KQ <= a.ne11;
            float mk[FA_KQ];
            if (!mrow) {
#pragma unroll
                for (int c = 0; c < FA_KQ; c++) mk[c] = 0.0f;
            } else if (mvec) {
#pragma unroll
                for (int t = 0; t < FA_KQ / 8; t++) {
                    uint4 w = make_uint4(0, 0, 0, 0);
                    if (key0 + 8 * t < a.ne11) w = __ldg(reinterpret_cast<const uint4*>(mrow + key0 + 8 * t));
                    const __half2* hp = reinterpret_cast<const __half2*>(&w);
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const float2 f = __half22float2(hp[e]);
                        mk[8 * t + 2 * e] = f.x;
                        mk[8 * t + 2 * e + 1] = f.y;
                    }
                }
            } else {
#pragma unroll
                for (int c = 0; c < FA_KQ; c++)
                    mk[c] = key0 + c < a.ne11 ? __half2float(__ushort_as_half(mrow[key0 + c])) : 0.0f;
            }
            // tcgen05.ld / st are warp-collective: every decision before them is warp-uniform
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[st], (uint32_t)(j >> 1) & 1, abort_flag))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[FA_KQ];
            {
                uint32_t v[32];
                tmem_ld32(trow + st * FA_BN + FA_KQ * h, v);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i++) sv[i] = __uint_as_float(v[i]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[st]);
            float mx8[8];
#pragma unroll
            for (int i = 0; i < 8; i++) mx8[i] = -INFINITY;
            if (full) {
#pragma unroll
                for (int c = 0; c < FA_KQ; c++) {
                    sv[c] = fmaf(mk[c], FA_LOG2E, sv[c]);
                    mx8[c & 7] = fmaxf(mx8[c & 7], sv[c]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < FA_KQ; c++) {
                    sv[c] = key0 + c < a.ne11 ? fmaf(mk[c], FA_LOG2E, sv[c]) : -INFINITY;
                    mx8[c & 7] = fmaxf(mx8[c & 7], sv[c]);
                }
            }
            const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                   fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            // the row max over the four key quarters
            xmax[st][h][r] = mx;
            named_bar_sync(quad_bar, 32 * FA_NQ);
            const float m_chunk = fmaxf(fmaxf(xmax[st][0][r], xmax[st][1][r]), fmaxf(xmax[st][2][r], xmax[st][3][r]));
            // all four quarters of a row see the same values, so they take the same decision
            const bool grow = m_chunk > m_used + FA_RESCALE_LOG2 || (m_used == -INFINITY && m_chunk != -INFINITY);
            float alpha = 1.0f;
            if (grow) {
                alpha = m_used == -INFINITY ? 0.0f : ex2_approx(m_used - m_chunk);
                m_used = m_chunk;
            }
            if (j >= 1 && __any_sync(0xffffffffu, grow)) {
                // O holds products up to chunk j-1: wait for the last one, then rescale this quarter
                if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[(j - 1) % NPB], (uint32_t)((j - 1) / NPB) & 1, abort_flag))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t v[DQ];
                o_ld(v);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < DQ; i++) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                o_st(v);
                tmem_st_wait();
            }
            // every key so far masked: m_used is -inf and so is every score, and 2^(-inf - 0) = 0
            const float msub = m_used == -INFINITY ? 0.0f : m_used;
            uint32_t ph[FA_KQ / 2];
            float ps8[8];
#pragma unroll
            for (int i = 0; i < 8; i++) ps8[i] = 0.0f;
#pragma unroll
            for (int c = 0; c < FA_KQ; c += 2) {
                const float p0 = ex2_approx(sv[c] - msub), p1 = ex2_approx(sv[c + 1] - msub);
                const __half2 hh = __floats2half2_rn(p0, p1);
                ps8[(c >> 1) & 7] += p0 + p1;
                ph[c / 2] = *reinterpret_cast<const uint32_t*>(&hh);
            }
            const float psum = ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
            l = l * alpha + psum;
            // P buffer j % NPB was last read by the PV product of chunk j - NPB
            const int pb = j % NPB;
            if (j >= NPB && !__all_sync(0xffffffffu, mbar_wait(&pv_done[pb], (uint32_t)((j - NPB) / NPB) & 1, abort_flag))) {
                ok = false;
                break;
            }
            // keys 32 h .. 32 h + 31: 64-key block h / 2, 16-byte chunks 4 (h & 1) .. 4 (h & 1) + 3
            uint8_t* pblk = sP + pb * PBYTES + (h >> 1) * BLK_Q;
#pragma unroll
            for (int c = 0; c < 4; c++)
                st_chunk16(pblk, r, 4 * (h & 1) + c, ph[4 * c], ph[4 * c + 1], ph[4 * c + 2], ph[4 * c + 3]);
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[pb]);
        }
        if (ok && nch > 0) ok = mbar_wait(&pv_done[(nch - 1) % NPB], (uint32_t)((nch - 1) / NPB) & 1, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        xsum[h][r] = l;
        named_bar_sync(quad_bar, 32 * FA_NQ);
        tc_fence_after();
        if (!ok) {
            if (lane == 0) {
                cfi_set_error(a.err, 0xfa300 + warp);
                *abort_flag = 1;
            }
        } else {
            // every lane loads its TMEM row (collective); rows past the queries store nothing
            const float lt = (xsum[0][r] + xsum[1][r]) + (xsum[2][r] + xsum[3][r]);
            const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
            float* out = a.dst + (((size_t)seq * a.ne01 + (qvalid ? q : 0)) * a.ne02 + head) * D + DQ * h;
            uint32_t v[DQ];
            if (nch > 0) {
                o_ld(v);
                tmem_ld_wait();
            } else {
#pragma unroll
                for (int i = 0; i < DQ; i++) v[i] = 0u;
            }
            if (qvalid) {
#pragma unroll
                for (int i = 0; i < DQ; i += 4)
                    *reinterpret_cast<float4*>(out + i) =
                        make_float4(__uint_as_float(v[i]) * inv, __uint_as_float(v[i + 1]) * inv,
                                    __uint_as_float(v[i + 2]) * inv, __uint_as_float(v[i + 3]) * inv);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == FA_MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, FA_TMEM_COLS);
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

unsigned int* fa_err_ptr() {
    static CfiSymbolPtr<unsigned int> p;
    return p.get(g_fattn_error);
}

template <int D>
int launch_fa(const uint64_t* v, cudaStream_t stream) {
    PFN_encodeTiled enc = encode_fn();
    if (!enc) return (int)cudaErrorNotSupported;
    auto i32 = [&](int k) { return (int)(uint32_t)v[k]; };
    auto f32 = [&](int k) {
        const uint32_t b = (uint32_t)v[k];
        float f;
        memcpy(&f, &b, 4);
        return f;
    };
    const int ne01 = i32(15), ne02 = i32(16), ne03 = i32(17), ne11 = i32(22), ne12 = i32(23);
    const long long nb11 = i32(25), nb12 = i32(26), nb13 = (long long)v[27];
    const long long nb21 = i32(28), nb22 = i32(29), nb23 = (long long)v[30];
    CUtensorMap tk, tv;
    cuuint32_t box[4] = {64, FA_BN, 1, 1}, es[4] = {1, 1, 1, 1};
    {
        cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)ne11, (cuuint64_t)ne12, (cuuint64_t)ne03};
        cuuint64_t str[3] = {(cuuint64_t)nb11, (cuuint64_t)nb12, (cuuint64_t)nb13};
        if (enc(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, reinterpret_cast<void*>(v[1]), dims, str, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    {
        cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)ne11, (cuuint64_t)ne12, (cuuint64_t)ne03};
        cuuint64_t str[3] = {(cuuint64_t)nb21, (cuuint64_t)nb22, (cuuint64_t)nb23};
        if (enc(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, reinterpret_cast<void*>(v[2]), dims, str, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return (int)cudaErrorInvalidValue;
    }
    FaArgs a;
    a.q = reinterpret_cast<const uint8_t*>(v[0]);
    a.mask = reinterpret_cast<const uint8_t*>(v[3]);
    a.dst = reinterpret_cast<float*>(v[6]);
    a.scale = f32(8);
    a.ne01 = ne01;
    a.ne02 = ne02;
    a.ne03 = ne03;
    a.ne11 = ne11;
    a.ne12 = ne12;
    a.nb01 = i32(18);
    a.nb02 = i32(19);
    a.nb03 = i32(20);
    a.ne31 = i32(32);
    a.ne33 = std::max(1, i32(33));
    a.nb31 = i32(34);
    a.nb33 = (long long)v[36];
    a.nchunks = (ne11 + FA_BN - 1) / FA_BN;
    a.err = fa_err_ptr();
    constexpr size_t smem = fa_smem_bytes<D>();
    static CfiPerDeviceOnce attr;
    cfi_once_per_device(attr, [] { cudaFuncSetAttribute(cfi_fattn_tc<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); });
    const char* ep = getenv("CFI_PDL");
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned)((ne01 + FA_BM - 1) / FA_BM), (unsigned)ne02, (unsigned)ne03);
    c.blockDim = dim3(FA_THREADS, 1, 1);
    c.dynamicSmemBytes = smem;
    c.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = at;
    c.numAttrs = (ep && strcmp(ep, "0") == 0) ? 0 : 1;
    return (int)cudaLaunchKernelEx(&c, cfi_fattn_tc<D>, tk, tv, a);
}

}  // namespace

namespace cfi {
// mod.rs:27-54 plus this kernel's own needs: D 64/128, no sinks / ALiBi / softcap, GQA, at least
// 16 queries (below that ggml's split-KV kernel keeps decode), Q rows 4-byte aligned, K/V rows and
// strides 16-byte aligned (TMA), mask rows 2-byte aligned.
bool fattn_geometry_ok(uint32_t d, const uint64_t* v, int n) {
    if (n != 37 || (d != 64 && d != 128)) return false;
    auto u = [&](int k) { return (uint32_t)v[k]; };
    auto f_is_zero = [&](int k) { return (u(k) & 0x7fffffffu) == 0; };
    const uint32_t ne00 = u(14), ne01 = u(15), ne02 = u(16), ne03 = u(17), ne11 = u(22), ne12 = u(23);
    if (v[4] != 0 || !f_is_zero(9) || !f_is_zero(13)) return false;
    if (ne00 != d || ne01 < 16 || ne02 == 0 || ne03 == 0 || ne11 == 0 || ne12 == 0 || ne02 % ne12 || ne03 > 65535 || ne02 > 65535)
        return false;
    if ((v[0] | u(18) | u(19) | u(20)) % 4) return false;
    if ((v[1] | v[2] | u(25) | u(26) | v[27] | u(28) | u(29) | v[30]) % 16) return false;
    if (v[3] != 0 && ((v[3] | u(34) | v[36]) % 2 || u(33) == 0)) return false;
    if (v[6] % 16) return false;  // float4 stores of dst rows
    return true;
}

int fattn_launch(const cfi_plan& plan, void** args, void* stream) {
    std::vector<uint64_t> v = arg_values(plan, args);
    if (!fattn_geometry_ok(plan.aux, v.data(), (int)v.size())) return (int)cudaErrorInvalidValue;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return plan.aux == 64 ? launch_fa<64>(v.data(), s) : launch_fa<128>(v.data(), s);
}

int fattn_threads() { return FA_THREADS; }
int fattn_tile() { return FA_BM; }

unsigned int fattn_error_take() {
    unsigned int x = 0, z = 0;
    if (cudaMemcpyFromSymbol(&x, g_fattn_error, sizeof x) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaMemcpyToSymbol(g_fattn_error, &z, sizeof z);
    return x;
}
}  // namespace cfi
