// k_mmq_skinny.cu -- mul_mat_q for a few columns (ncols_dst <= 64: a batch of decode sequences):
// C[col][row] = sum_k W[row][k] X[col][k], W in Q4_K or Q8_0 blocks, X in ggml's q8_1_mmq layout.
//
// At 64 columns a product reads each weight byte once and each activation byte many times, and
// it is short: most of the matrices of a 1.5B model take a few microseconds at HBM rate.  So the
// kernel puts every load of a CTA in flight at its start and keeps nothing on the critical path
// that a load could hide:
//   * grid (CTAs over 16-row tiles, K splits), at most one CTA per SM.  A CTA copies the
//     activations of its K range (256-value chunks: two q8_1_mmq blocks of every column, each
//     block row of the batch one contiguous run) into shared memory once, by bulk copies, one
//     mbarrier per chunk; one warp per chunk turns that chunk's scales into float and releases
//     it on a second mbarrier, so a warp starts on its first chunk as soon as that chunk is in;
//   * the 8 warps form 8 / KP row groups of KP warps; row group r of CTA b takes tile
//     b * 8 / KP + r in round 0 and one tile gridDim.x * 8 / KP further in each later round; of
//     each tile, warp (r, part) takes the chunks part, part + KP, ...  Every warp streams its own
//     (tile, chunk) weight stages (16 rows x 144 bytes of Q4_K or 16 x 272 bytes of Q8_0, as
//     16-byte cp.async copies: the bulk-copy unit serves a few large copies far better than
//     hundreds of row-sized ones) through a private ring of mbarrier-tracked stages, so no warp
//     waits for another inside a tile;
//   * per 32-value sub-block and 8-column n-tile one mma.sync.m16n8k32 (u8/s8 x s8 -> s32) gives
//     the exact int32 block dots of 16 rows.  A comes from ldmatrix.x4 (Q4_K: a 32-byte nibble
//     group of 16 rows, masked 0x0F / 0xF0, the high nibbles' factor 16 taken out of the scale) or
//     4-byte shared loads (Q8_0's 34-byte blocks); B from one ldmatrix.x4 per two n-tiles.  The
//     MMA's accumulator input is 0x4B400000, so its int32 result read as a float is
//     1.5 * 2^23 + dot exactly (|dot| < 2^22 for these blocks) and one packed f32x2 subtract makes
//     two exact float dots; then acc += dot * (w_scale * x_scale) in packed f32x2 arithmetic,
//     w_scale = half(d * sc) (Q4_K) or d (Q8_0), ggml's mmq roundings;
//   * Q4_K's min term of a chunk, -sum_j half(dmin * m_j) * s_j, is one mma.sync.m16n8k8 tf32 per
//     n-tile (half values are exact in tf32), accumulated into the same registers;
//   * with KP > 1 the parts of a tile meet in shared memory at the end of each round (in part
//     order); with K splits the tile's partials go to the calling stream's workspace and the last
//     warp to finish a tile (a counter per tile) adds them in split order.  Both orders are fixed:
//     results do not depend on timing.
// Tolerance mode: the int32 block dots are exact, the fp32 sums are reassociated (agrees with the
// reference's order to about 1e-7 relative).  Every wait is bounded (error word, then the warp
// skips its remaining work and lets its copies in flight land).
#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "peer_sync.cuh"
#include "sm100_ptx.cuh"

#include <algorithm>
#include <stdlib.h>
#include <string.h>

namespace {

using namespace sm100;

constexpr int SK_TR = 16;  // rows per tile
constexpr int SK_MAX_NT = 8;                                // 8-column n-tiles (64 columns)
constexpr int SK_MAX_STAGES = 8;
constexpr int SK_DEFAULT_WARPS = 8;  // CTA size: 8 or 16 warps (CFI_MMQ_SKINNY_WARPS)
constexpr int SK_PART_FLOATS = SK_MAX_NT * 4 * 32;          // one tile's partial, lane-major
constexpr uint32_t SK_MAGIC = 0x4B400000u;                  // 1.5 * 2^23 as a float

template <uint32_t TY> __host__ __device__ constexpr uint32_t sk_chunk_bytes() { return TY == T_Q4_K ? 144u : 272u; }
// floats per (chunk, sub-block, t) row of xd: the 2 NT values of columns n * 8 + 2t + {0, 1},
// rounded to a multiple of 4 and padded by 4 (the four t rows of a 16-byte load hit different banks)
__host__ __device__ constexpr uint32_t sk_xdt(uint32_t nt) { return (2 * nt + 3) / 4 * 4 + 4; }

// Shared memory of a launch (bytes, each part a multiple of 16):
//   act  [kr][2 blocks][NC8 columns][144]     raw q8_1_mmq blocks
//   xd   [kr][8 sub-blocks][4 t][XDT]         float d of column n * 8 + 2t + e at n * 2 + e
//   xs   [kr][8][NC8 + 8]                     Q4_K: float s (padded rows: conflict-free tf32 B loads)
//   ring [W warps][stages][16 x chunk bytes]  weights
//   red  [slots][NT x 4][32]                  KP > 1: the parts of a tile (W - W / KP slots, or
//                                             one per row group when they are added in turn)
//   bars act[kr], scales[kr], ring[W][stages]
struct SkLayout {
    uint32_t act, xd, xs, ring, red, bars, total;
};
__host__ __device__ inline uint32_t sk_red_slots(uint32_t w, uint32_t kp, bool par) {
    return kp > 1 ? (par ? w - w / kp : w / kp) : 0;
}
__host__ __device__ inline SkLayout sk_layout(uint32_t ty, uint32_t nt, uint32_t kr, uint32_t stages, uint32_t kp,
                                              uint32_t w, bool par) {
    SkLayout l;
    const uint32_t nc8 = nt * 8, cb = ty == T_Q4_K ? 144u : 272u;
    l.act = 0;
    l.xd = l.act + kr * 2 * nc8 * 144;
    l.xs = l.xd + kr * 8 * 4 * sk_xdt(nt) * 4;
    l.ring = l.xs + (ty == T_Q4_K ? kr * 8 * (nc8 + 8) * 4 : 0);
    l.red = l.ring + w * stages * SK_TR * cb;
    l.bars = l.red + sk_red_slots(w, kp, par) * nt * 4 * 32 * 4;
    l.total = l.bars + (2 * kr + w * stages) * 8;
    return l;
}

constexpr int SK_MAX_GROUP = 4;  // products of one launch (they read the same activations)

struct SkArgs {
    // product i: weights x[i] (nrows[i] rows, stride_row_x[i] blocks apart), output dst[i]
    // (column c at c * stride_col_dst[i]); its 16-row tiles are tiles tile_begin[i] .. of the launch
    const uint8_t* x[SK_MAX_GROUP];
    float* dst[SK_MAX_GROUP];
    uint32_t nrows[SK_MAX_GROUP], stride_row_x[SK_MAX_GROUP], stride_col_dst[SK_MAX_GROUP];
    uint32_t tile_begin[SK_MAX_GROUP];
    uint32_t ngroup;
    const uint8_t* y;  // q8_1_mmq activations
    uint32_t ncols, ncols_y;
    uint32_t nchunks, kr, ksplits;  // 256-value chunks of K, chunks per K split, splits
    uint32_t kp, ntiles, stages;    // warps per row group, 16-row tiles, ring stages per warp
    uint32_t red_par;               // KP > 1: a slot per part (one barrier) or per row group (parts in turn)
    float* ws;                      // K splits: partials [tile][split][SK_PART_FLOATS]
    unsigned int* counters;         // K splits: per tile
    unsigned int* err;
    // all-gather over peer memory (world > 1): every output also at its address + delta[r] on
    // every other rank r; after the launch's last store its last CTA signals the peers and waits
    // for theirs (world == 1: local stores only)
    CfiPeerDev pr;
};

// The product a launch tile belongs to (constant indices only: no local copy of the arguments).
struct SkProd {
    const uint8_t* x;
    float* dst;
    uint32_t nrows, srx, scd, tile;  // tile: the tile's index within its product
};
CFI_DEV SkProd sk_prod(const SkArgs& a, uint32_t tile) {
    SkProd p = {a.x[0], a.dst[0], a.nrows[0], a.stride_row_x[0], a.stride_col_dst[0], tile};
#pragma unroll
    for (int i = 1; i < SK_MAX_GROUP; i++)
        if ((uint32_t)i < a.ngroup && tile >= a.tile_begin[i])
            p = {a.x[i], a.dst[i], a.nrows[i], a.stride_row_x[i], a.stride_col_dst[i], tile - a.tile_begin[i]};
    return p;
}

// A warp's outputs of one tile (m16n8 accumulator layout: lane (g, t) holds rows g, g + 8 of
// columns 2t, 2t + 1 of each 8-column tile n) into dst and, for an all-gather over peer memory,
// into every peer's copy (plain stores over NVLink).
// Ranks in turn from this one, so the ranks' first stores go to different GPUs.  (`a` is the
// kernel's __grid_constant__ parameter: the offsets are read from the parameter space with a
// run-time index, without a local copy of the arguments.)
template <int NT>
CFI_DEV void sk_store(const SkArgs& a, const SkProd& pr, const float (&out)[NT][4], int g, int t) {
#pragma unroll 1
    for (int i = 0; i < a.pr.world; i++) {
        const int r = a.pr.rank + i < a.pr.world ? a.pr.rank + i : a.pr.rank + i - a.pr.world;
        float* d = reinterpret_cast<float*>(reinterpret_cast<char*>(pr.dst) + a.pr.delta[r]);
#pragma unroll
        for (int n = 0; n < NT; n++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const uint32_t row = pr.tile * SK_TR + g + 8 * (e >> 1), col = n * 8 + 2 * t + (e & 1);
                if (row < pr.nrows && col < a.ncols) d[(size_t)col * pr.scd + row] = out[n][e];
            }
    }
}

// 16-byte global -> shared copy on the LSU path (L2 only), and an arrival on `bar` once every
// copy this thread issued before it has landed (the arrival does not count toward the barrier's
// expected arrivals beyond those it was initialised with)
CFI_DEV void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
CFI_DEV void cp_async_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
CFI_DEV void ldsm_x4v(uint32_t a, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a)
                 : "memory");
}
CFI_DEV void ldsm_x2v(uint32_t a, uint32_t (&r)[2]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(a) : "memory");
}
// 64-bit pairs of fp32 (sm_100 packed arithmetic): lo in bits 0..31
CFI_DEV uint64_t pk2(uint32_t lo, uint32_t hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
    return d;
}
CFI_DEV uint64_t pk2f(float lo, float hi) { return pk2(__float_as_uint(lo), __float_as_uint(hi)); }
CFI_DEV void upk2(uint64_t v, float& lo, float& hi) {
    uint32_t a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(a), "=r"(b) : "l"(v));
    lo = __uint_as_float(a);
    hi = __uint_as_float(b);
}
CFI_DEV uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
CFI_DEV uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
CFI_DEV void fma2(uint64_t& c, uint64_t a, uint64_t b) { asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c) : "l"(a), "l"(b)); }

// d = 1.5 * 2^23 + A B (int32), as two packed pairs (rows g and g + 8 of columns 2t, 2t + 1)
template <bool U8>
CFI_DEV void mma_i8_magic(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, uint64_t& d01, uint64_t& d23) {
    uint32_t d0, d1, d2, d3;
    if (U8)
        asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%10, %10, %10, %10};"
            : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(SK_MAGIC));
    else
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%10, %10, %10, %10};"
            : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(SK_MAGIC));
    d01 = pk2(d0, d1);
    d23 = pk2(d2, d3);
}
CFI_DEV void mma_tf32_p(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, uint64_t& c01, uint64_t& c23) {
    float c0, c1, c2, c3;
    upk2(c01, c0, c1);
    upk2(c23, c2, c3);
    asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c0), "+f"(c1), "+f"(c2), "+f"(c3)
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    c01 = pk2f(c0, c1);
    c23 = pk2f(c2, c3);
}

// The sub-block j of one chunk for every n-tile: acc[n] += dot(A, B_n) * (w * x_n).
// yq: shared address of this lane's ldmatrix row of B (n-tile pair 0) for sub-block j;
// xq: this lane's xd row of (chunk, j, t).
template <bool U8, int NT>
CFI_DEV void sk_subblock(const uint32_t (&af)[4], uint64_t w0, uint64_t w1, uint32_t yq, const float* xq,
                         uint64_t (&acc)[NT][2]) {
    const uint64_t mg = pk2f(12582912.0f, 12582912.0f);
#pragma unroll
    for (int p = 0; p < (NT + 1) / 2; p++) {
        const uint4 x4 = *reinterpret_cast<const uint4*>(xq + 4 * p);
        uint32_t b[4];
        if (2 * p + 1 < NT) {
            ldsm_x4v(yq + p * 16 * MMQ_BLOCK_BYTES, b);
        } else {
            uint32_t b2[2];
            ldsm_x2v(yq + p * 16 * MMQ_BLOCK_BYTES, b2);
            b[0] = b2[0];
            b[1] = b2[1];
            b[2] = b[3] = 0;
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int n = 2 * p + h;
            if (n >= NT) break;
            uint64_t d01, d23;
            mma_i8_magic<U8>(af, b[2 * h], b[2 * h + 1], d01, d23);
            const uint64_t x01 = h ? pk2(x4.z, x4.w) : pk2(x4.x, x4.y);
            fma2(acc[n][0], sub2(d01, mg), mul2(w0, x01));
            fma2(acc[n][1], sub2(d23, mg), mul2(w1, x01));
        }
    }
}

template <uint32_t TY, int NT, int W>
__global__ void __launch_bounds__(W * 32, 1) cfi_mmq_skinny(const __grid_constant__ SkArgs a) {
    constexpr uint32_t CB = sk_chunk_bytes<TY>(), WB = SK_TR * CB, NC8 = NT * 8;
    constexpr uint32_t XSP = NC8 + 8, XDT = sk_xdt(NT);
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_abort;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const uint32_t KP = a.kp, RW = W / KP, rw = warp / KP, kp = warp % KP;
    // 16 warps: the sub-block loops stay rolled so a thread fits the 128 registers of a full SM
    constexpr int UNR = W >= 16 ? 1 : 4;
    const uint32_t S = a.stages, kr = a.kr;
    const SkLayout L = sk_layout(TY, NT, kr, S, KP, W, a.red_par != 0);
    uint8_t* act = smem + L.act;
    float* xd = reinterpret_cast<float*>(smem + L.xd);
    float* xs = reinterpret_cast<float*>(smem + L.xs);
    uint8_t* ring = smem + L.ring + (size_t)warp * S * WB;
    float* red = reinterpret_cast<float*>(smem + L.red);
    uint64_t* abar = reinterpret_cast<uint64_t*>(smem + L.bars);  // activations of chunk ci landed
    uint64_t* sbar = abar + kr;                                      // ... and their float scales written
    uint64_t* rbar = sbar + kr + warp * S;
    volatile int* abort_flag = &s_abort;

    // this CTA's K range and this warp's tiles and chunks
    const uint32_t c0 = blockIdx.y * kr, nck = min(a.nchunks, c0 + kr) - c0;
    const uint32_t nq = nck > kp ? (nck - kp + KP - 1) / KP : 0;  // chunks of this warp per tile
    const uint32_t tstride = gridDim.x * RW, tile0 = blockIdx.x * RW + rw, tile00 = blockIdx.x * RW;
    const uint32_t rounds_w = tile0 < a.ntiles ? (a.ntiles - tile0 + tstride - 1) / tstride : 0;
    const uint32_t rounds = tile00 < a.ntiles ? (a.ntiles - tile00 + tstride - 1) / tstride : 0;  // row group 0: the most
    const uint32_t steps = rounds_w * nq;

    if (tid == 0) {
        s_abort = 0;
        for (uint32_t i = 0; i < kr; i++) {
            mbar_init(abar + i, 1);
            mbar_init(sbar + i, 32);
        }
        for (uint32_t i = 0; i < W * S; i++) mbar_init(sbar + kr + i, 32);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();  // weights, activations, workspace: everything after the previous kernel

    const uint32_t xbytes = TY == T_Q4_K ? 144u : 34u;  // bytes of one ggml block of a row
    // weights of step s into ring slot s % S: 16 rows x CB bytes as 16-byte cp.async copies, lane
    // L taking segments L, L + 32, ...; each lane's arrival (noinc: the barrier counts 32) fires
    // when its own copies have landed
    auto issue = [&](uint32_t s) {
        const uint32_t tile = tile0 + (s / nq) * tstride, chunk = c0 + kp + (s % nq) * KP;
        const SkProd pr = sk_prod(a, tile);
        uint8_t* st = ring + (s % S) * WB;
#pragma unroll
        for (uint32_t k = 0; k < (WB / 16 + 31) / 32; k++) {
            const uint32_t seg = lane + 32 * k;
            if (seg < WB / 16) {
                const uint32_t r = seg / (CB / 16), off = (seg % (CB / 16)) * 16;
                const uint32_t row = min(pr.tile * SK_TR + r, pr.nrows - 1);  // rows past the end: a copy of the last
                const uint8_t* src = pr.x + (size_t)row * pr.srx * xbytes + (size_t)chunk * CB + off;
                cp_async16(st + r * CB + off, src);
            }
        }
        cp_async_arrive_noinc(rbar + s % S);
    };
    // activations of the K range (warp 0, chunk by chunk), then every warp's first stages
    if (warp == 0) {
        for (uint32_t ci = 0; ci < nck; ci++) {
            if (lane == 0) mbar_arrive_expect_tx(abar + ci, 2 * a.ncols * MMQ_BLOCK_BYTES);
            __syncwarp();
            if (lane < 2) {
                const uint8_t* src = a.y + ((size_t)(c0 + ci) * 2 + lane) * a.ncols_y * MMQ_BLOCK_BYTES;
                bulk_g2s(act + ((ci * 2 + lane) * NC8) * MMQ_BLOCK_BYTES, src, a.ncols * MMQ_BLOCK_BYTES, abar + ci);
            }
        }
    }
    uint32_t issued = min(S, steps);
    for (uint32_t s = 0; s < issued; s++) issue(s);

    // float scales of chunks warp, warp + 8, ...: xd = d (and xs = s for Q4_K) of every
    // (sub-block, column), from the 16-byte headers of the chunk's 2 x NC8 blocks
    bool failed = false;  // warp-uniform: a wait gave up (or another warp's did), skip the rest
    auto fail = [&](uint32_t code) {
        failed = true;
        if (lane == 0) {
            cfi_set_error(a.err, code);
            s_abort = 1;
        }
    };
    for (uint32_t ci = warp; ci < nck; ci += W) {
        if (!failed && !__all_sync(0xffffffffu, mbar_wait(abar + ci, 0, abort_flag))) fail(0x5c0000u);
        if (!failed) {
            for (uint32_t hb = lane; hb < 2 * NC8; hb += 32) {  // (block half, column)
                const uint32_t h = hb / NC8, c = hb % NC8;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (c < a.ncols) v = *reinterpret_cast<const uint4*>(act + ((ci * 2 + h) * NC8 + c) * MMQ_BLOCK_BYTES);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                const uint32_t tt = (c % 8) / 2, col = (c / 8) * 2 + (c & 1);
#pragma unroll
                for (int gg = 0; gg < 4; gg++) {
                    const uint32_t j = 4 * h + gg;
                    if (TY == T_Q4_K) {
                        xd[((ci * 8 + j) * 4 + tt) * XDT + col] = h2f_bits((uint16_t)(w[gg] & 0xffffu));
                        xs[(ci * 8 + j) * XSP + c] = h2f_bits((uint16_t)(w[gg] >> 16));
                    } else {
                        xd[((ci * 8 + j) * 4 + tt) * XDT + col] = __uint_as_float(w[gg]);
                    }
                }
            }
        }
        mbar_arrive(sbar + ci);  // every lane: its own stores are released to the chunk's readers
    }

    const uint32_t sact = smem_u32(act);
    const uint32_t lrow = (lane & 7) + 8 * ((lane >> 3) & 1), lbyte = 16 * (lane >> 4);  // A ldmatrix row / half
    // B ldmatrix rows: lanes 0-15 column n * 8 + (lane & 7) of n-tile 2p, 16-31 of 2p + 1; bytes
    // 16 * ((lane >> 3) & 1) of the sub-block
    const uint32_t ybrow = ((lane & 7) + 8 * (lane >> 4)) * MMQ_BLOCK_BYTES + 16 * ((lane >> 3) & 1) + 16;
    uint32_t ready = 0;  // chunks of the K range whose activations this warp has seen released
    uint32_t s = 0, drain_from = 0;
    for (uint32_t r = 0; r < rounds; r++) {
        const bool has = r < rounds_w;
        const uint32_t tile = tile0 + r * tstride;
        uint64_t acc[NT][2];
#pragma unroll
        for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = 0;
        for (uint32_t q = 0; has && q < nq; q++, s++) {
            const uint32_t slot = s % S, ci = kp + q * KP;  // chunk within the K range
            if (failed) continue;
            bool got = true;
            if (!(ready >> ci & 1)) {
                got = mbar_wait(sbar + ci, 0, abort_flag) && mbar_wait(abar + ci, 0, abort_flag);
                ready |= 1u << ci;
            }
            got = __all_sync(0xffffffffu, got && mbar_wait(rbar + slot, (s / S) & 1, abort_flag));
            if (!got) {
                fail(0x5c0000u | ((s + 1) & 0xffffu));
                drain_from = s;
                continue;
            }
            const uint8_t* st = ring + slot * WB;
            const uint32_t sw = smem_u32(st);
            const uint32_t yb = sact + ci * 2 * NC8 * MMQ_BLOCK_BYTES + ybrow;
            const float* xdc = xd + (ci * 8 * 4 + t) * XDT;
            if (TY == T_Q4_K) {
                const uint4 h0 = *reinterpret_cast<const uint4*>(st + g * CB);
                const uint4 h1 = *reinterpret_cast<const uint4*>(st + (g + 8) * CB);
                float dd[2];
                uint32_t scw[2][2];  // [row][sub-blocks 0-3, 4-7]: 6-bit scales, one per byte
                uint32_t am[4];
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const uint4 hd = h ? h1 : h0;
                    dd[h] = h2f_bits((uint16_t)(hd.x & 0xffffu));
                    const float dmin = h2f_bits((uint16_t)(hd.x >> 16));
                    scw[h][0] = hd.y & 0x3F3F3F3Fu;
                    scw[h][1] = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
                    const uint32_t mlo = hd.z & 0x3F3F3F3Fu;
                    const uint32_t mhi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
                    // tf32 A of the min term: -half(dmin * m) at (row, sub-block t) and (row, t + 4)
                    am[h] = __float_as_uint(-__half2float(__float2half_rn(dmin * (float)((mlo >> (8 * t)) & 0xffu))));
                    am[h + 2] = __float_as_uint(-__half2float(__float2half_rn(dmin * (float)((mhi >> (8 * t)) & 0xffu))));
                }
#pragma unroll UNR
                for (int c4 = 0; c4 < 4; c4++) {  // nibble group c4: sub-blocks 2 c4 (low) and 2 c4 + 1 (high)
                    uint32_t raw[4];
                    ldsm_x4v(sw + lrow * CB + 16 + 32 * c4 + lbyte, raw);
#pragma unroll
                    for (int hi = 0; hi < 2; hi++) {
                        const int j = 2 * c4 + hi;
                        const uint32_t msk = hi ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
                        const uint32_t af[4] = {raw[0] & msk, raw[1] & msk, raw[2] & msk, raw[3] & msk};
                        float w2[2];
#pragma unroll
                        for (int h = 0; h < 2; h++) {  // half(d * sc), ggml's rounding; odd sub-blocks / 16
                            const uint32_t sc = ((c4 < 2 ? scw[h][0] : scw[h][1]) >> (8 * (j & 3))) & 0xffu;
                            const float v = __half2float(__float2half_rn(dd[h] * (float)sc));
                            w2[h] = hi ? v * 0.0625f : v;
                        }
                        sk_subblock<true, NT>(af, pk2f(w2[0], w2[0]), pk2f(w2[1], w2[1]),
                                              yb + (j / 4) * NC8 * MMQ_BLOCK_BYTES + 32 * (j % 4), xdc + j * 4 * XDT, acc);
                    }
                }
                const float* xsc = xs + ci * 8 * XSP + g;
#pragma unroll
                for (int n = 0; n < NT; n++)
                    mma_tf32_p(am, __float_as_uint(xsc[t * XSP + n * 8]), __float_as_uint(xsc[(t + 4) * XSP + n * 8]),
                               acc[n][0], acc[n][1]);
            } else {
                // Q8_0: block j of a row at j * 34 (d) and j * 34 + 2 (quants); rows g and g + 8
#pragma unroll UNR
                for (int j2 = 0; j2 < 4; j2++) {
#pragma unroll
                    for (int odd = 0; odd < 2; odd++) {
                        const int j = 2 * j2 + odd;
                        uint32_t af[4];
                        float wd[2];
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const uint8_t* rb = st + (g + 8 * h) * CB + 34 * j;
                            wd[h] = h2f_bits(*reinterpret_cast<const uint16_t*>(rb));
                            const uint8_t* o = rb + 2 + 4 * t;  // quants 4t .. 4t + 3, and 16 + 4t ..
                            if (!odd) {                         // 2-byte aligned: shift two words together
                                const uint32_t* wp = reinterpret_cast<const uint32_t*>(o - 2);
                                af[h] = __funnelshift_r(wp[0], wp[1], 16);
                                af[h + 2] = __funnelshift_r(wp[4], wp[5], 16);
                            } else {
                                const uint32_t* wp = reinterpret_cast<const uint32_t*>(o);
                                af[h] = wp[0];
                                af[h + 2] = wp[4];
                            }
                        }
                        sk_subblock<false, NT>(af, pk2f(wd[0], wd[0]), pk2f(wd[1], wd[1]),
                                               yb + (j / 4) * NC8 * MMQ_BLOCK_BYTES + 32 * (j % 4), xdc + j * 4 * XDT, acc);
                    }
                }
            }
            __syncwarp();  // every lane is done with the slot before it is refilled
            if (s + S < steps) {
                issue(s + S);
                issued = s + S + 1;
            }
        }
        float out[NT][4];
#pragma unroll
        for (int n = 0; n < NT; n++) {
            upk2(acc[n][0], out[n][0], out[n][1]);
            upk2(acc[n][1], out[n][2], out[n][3]);
        }
        // ---- the parts of the tile (KP > 1) ----
        if (KP > 1 && a.red_par) {  // a slot per part, added in part order after one barrier
            float* mine = red + (rw * (KP - 1) + kp - 1) * (NT * 4 * 32);
            if (has && kp > 0) {
#pragma unroll
                for (int n = 0; n < NT; n++)
#pragma unroll
                    for (int e = 0; e < 4; e++) mine[(n * 4 + e) * 32 + lane] = out[n][e];
            }
            __syncthreads();
            if (has && kp == 0) {
                for (uint32_t k2 = 1; k2 < KP; k2++) {
                    const float* o = red + (rw * (KP - 1) + k2 - 1) * (NT * 4 * 32);
#pragma unroll
                    for (int n = 0; n < NT; n++)
#pragma unroll
                        for (int e = 0; e < 4; e++) out[n][e] += o[(n * 4 + e) * 32 + lane];
                }
            }
        } else if (KP > 1) {  // one slot per row group: parts KP - 1, ..., 1 add into it in turn
            float* slot = red + rw * (NT * 4 * 32);
            for (uint32_t k2 = KP - 1; k2 >= 1; k2--) {
                if (has && kp == k2) {
#pragma unroll
                    for (int n = 0; n < NT; n++)
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            float* q = slot + (n * 4 + e) * 32 + lane;
                            *q = k2 == KP - 1 ? out[n][e] : *q + out[n][e];
                        }
                }
                __syncthreads();
            }
            if (has && kp == 0) {
#pragma unroll
                for (int n = 0; n < NT; n++)
#pragma unroll
                    for (int e = 0; e < 4; e++) out[n][e] += slot[(n * 4 + e) * 32 + lane];
            }
        }
        if (has && kp == 0 && !failed) {
            const SkProd pr = sk_prod(a, tile);
            if (a.ksplits == 1) {
                sk_store<NT>(a, pr, out, g, t);
            } else {
                // K splits: this split's partial, then the last warp of the tile adds them in order
                float* part = a.ws + ((size_t)tile * a.ksplits + blockIdx.y) * SK_PART_FLOATS;
#pragma unroll
                for (int n = 0; n < NT; n++)
#pragma unroll
                    for (int e = 0; e < 4; e++) part[(n * 4 + e) * 32 + lane] = out[n][e];
                __threadfence();
                __syncwarp();
                unsigned int prev = 0;
                if (lane == 0) prev = atomicAdd(&a.counters[tile], 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == a.ksplits - 1) {
                    __threadfence();
                    // split by split (each split's 4 NT loads in flight together), in split order
                    const float* base = a.ws + (size_t)tile * a.ksplits * SK_PART_FLOATS + lane;
#pragma unroll
                    for (int n = 0; n < NT; n++)
#pragma unroll
                        for (int e = 0; e < 4; e++) out[n][e] = 0.0f;
                    for (uint32_t sp = 0; sp < a.ksplits; sp++) {
                        float v[NT][4];
#pragma unroll
                        for (int n = 0; n < NT; n++)
#pragma unroll
                            for (int e = 0; e < 4; e++) v[n][e] = __ldcg(base + (size_t)sp * SK_PART_FLOATS + (n * 4 + e) * 32);
#pragma unroll
                        for (int n = 0; n < NT; n++)
#pragma unroll
                            for (int e = 0; e < 4; e++) out[n][e] += v[n][e];
                    }
                    sk_store<NT>(a, pr, out, g, t);
                    if (lane == 0) a.counters[tile] = 0u;
                }
            }
        }
        if (KP > 1) __syncthreads();  // red is rewritten next round
    }
    if (failed) {
        // let this warp's copies still in flight land before the CTA exits (bounded as a whole);
        // warp 0 issued the activations
        const uint64_t deadline = globaltimer() + WAIT_LIMIT_NS;
        for (uint32_t k = drain_from; k < issued; k++)
            while (!mbar_try_wait(rbar + k % S, (k / S) & 1) && globaltimer() < deadline) {
            }
        if (warp == 0)
            for (uint32_t ci = 0; ci < nck; ci++)
                while (!mbar_try_wait(abar + ci, 0) && globaltimer() < deadline) {
                }
    }
    if (a.pr.world > 1) {
        // this CTA's stores (the peers' copies included; ordered before thread 0 by the CTA
        // barrier) made visible to the system, then its share of the launch's signal to every
        // peer; CTA 0 then waits for every peer's whole signal, so the launch completes once
        // every rank's rows are here (a CTA that gave up signals too: its error is in the error
        // word, and the peers do not wait out their limit)
        __syncthreads();
        if (tid == 0) {
            const bool first = blockIdx.x == 0 && blockIdx.y == 0;
            peer_signal_cta(a.pr, gridDim.x * gridDim.y, first);
            if (first) peer_wait_all(a.pr, a.err);
        }
    }
}

template <uint32_t TY, int W>
const void* sk_kernel_w(int nt) {
    switch (nt) {
    case 1: return reinterpret_cast<const void*>(&cfi_mmq_skinny<TY, 1, W>);
    case 2: return reinterpret_cast<const void*>(&cfi_mmq_skinny<TY, 2, W>);
    case 3: return reinterpret_cast<const void*>(&cfi_mmq_skinny<TY, 3, W>);
    case 4: return reinterpret_cast<const void*>(&cfi_mmq_skinny<TY, 4, W>);
    case 5: return reinterpret_cast<const void*>(&cfi_mmq_skinny<TY, 5, W>);
    case 6: return reinterpret_cast<const void*>(&cfi_mmq_skinny<TY, 6, W>);
    case 7: return reinterpret_cast<const void*>(&cfi_mmq_skinny<TY, 7, W>);
    case 8: return reinterpret_cast<const void*>(&cfi_mmq_skinny<TY, 8, W>);
    default: return nullptr;
    }
}
const void* sk_kernel(uint32_t ty, int nt, int w) {
    if (ty == T_Q4_K) return w == 16 ? sk_kernel_w<T_Q4_K, 16>(nt) : sk_kernel_w<T_Q4_K, 8>(nt);
    return w == 16 ? sk_kernel_w<T_Q8_0, 16>(nt) : sk_kernel_w<T_Q8_0, 8>(nt);
}

struct SkPlan {
    uint32_t kr, ksplits, kp, nx, stages;
    bool par;
    size_t smem;
};

// Work split of one product over CTAs of w warps: K splits only where the K range's activations
// do not fit in shared memory; then the row-group shape KP (warps per tile) and the CTA count that
// give the fewest chunks per warp (ties: smaller KP, fewer parts to combine); then as many ring
// stages as fit, and a slot per part for the tile's parts when those fit too.
bool sk_plan(uint32_t ty, uint32_t nt, uint32_t nchunks, uint32_t ntiles, int sms, size_t smem_max, uint32_t w,
             SkPlan& p) {
    uint32_t kr_max = 0;
    for (uint32_t kr = 1; kr <= std::min(nchunks, 32u); kr++) {  // <= 32: a warp's mask of released chunks
        if (sk_layout(ty, nt, kr, 2, 1, w, false).total > smem_max) break;
        kr_max = kr;
    }
    if (kr_max == 0) return false;
    p.kp = 1;
    p.nx = 1;
    const char* ek = getenv("CFI_MMQ_SKINNY_SPLITS");
    uint32_t ks = (nchunks + kr_max - 1) / kr_max;
    if (ek && atoi(ek) >= 1) ks = std::max(ks, std::min<uint32_t>((uint32_t)atoi(ek), nchunks));
    p.kr = (nchunks + ks - 1) / ks;
    p.ksplits = (nchunks + p.kr - 1) / p.kr;
    const uint32_t per_split = std::max(1u, (uint32_t)sms / p.ksplits);
    // CFI_MMQ_SKINNY_KP (1, 2, 4, 8, 16 up to the warp count) fixes the row-group shape instead
    // (tests of each form)
    const char* ekp = getenv("CFI_MMQ_SKINNY_KP");
    const uint32_t kp_only = ekp ? (uint32_t)atoi(ekp) : 0u;
    double best = 1e30;
    bool any = false;
    for (uint32_t kp = 1; kp <= w; kp *= 2) {
        if (kp_only && kp != kp_only) continue;
        if (sk_layout(ty, nt, p.kr, 1, kp, w, false).total > smem_max) continue;
        const uint32_t rw = w / kp;
        const uint32_t nx = std::min(per_split, (ntiles + rw - 1) / rw);
        const uint32_t rounds = (ntiles + nx * rw - 1) / (nx * rw);
        const double cost = (double)rounds * ((p.kr + kp - 1) / kp) + (kp > 1 ? 0.25 * rounds : 0.0);
        if (cost < best - 1e-9) {
            best = cost;
            p.kp = kp;
            p.nx = nx;
            any = true;
        }
    }
    if (!any) return false;
    const uint32_t rw = w / p.kp;
    const uint32_t rounds = (ntiles + p.nx * rw - 1) / (p.nx * rw);
    const uint32_t steps = rounds * ((p.kr + p.kp - 1) / p.kp);  // most steps of one warp
    p.stages = 1;
    for (uint32_t st = 1; st <= (uint32_t)SK_MAX_STAGES && st <= std::max(1u, steps); st++)
        if (sk_layout(ty, nt, p.kr, st, p.kp, w, false).total <= smem_max) p.stages = st;
    p.par = sk_layout(ty, nt, p.kr, p.stages, p.kp, w, true).total <= smem_max;
    p.smem = sk_layout(ty, nt, p.kr, p.stages, p.kp, w, p.par).total;
    return p.smem <= smem_max;
}

struct SkDev {
    int sms = 0;
    size_t smem_max = 0;
};

SkDev sk_dev() {
    static SkDev devs[CFI_MAX_DEVICES];
    static CfiPerDeviceOnce once[CFI_MAX_DEVICES];
    const int dev = cfi_device_index();
    cfi_once_per_device(once[dev], [&] {
        int sms = 148, optin = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        devs[dev].sms = sms;
        devs[dev].smem_max = optin > 1024 ? (size_t)optin - 1024 : 0;  // the kernel's static shared words
    });
    return devs[dev];
}

}  // namespace

bool cfi_mmq_skinny_applies(uint32_t ty, const void* x, const void* y, uint32_t K, uint32_t ncols_dst,
                            uint32_t stride_row_x, uint32_t planes) {
    if (ty != T_Q4_K && ty != T_Q8_0) return false;
    const char* e = getenv("CFI_MMQ_SKINNY");
    if (e && strcmp(e, "0") == 0) return false;
    if (planes != 1 || ncols_dst == 0 || ncols_dst > 8u * SK_MAX_NT || K == 0 || K % 256) return false;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15)) return false;
    // every row's chunks must start 16-byte aligned for the bulk copies
    if (ty == T_Q8_0 && stride_row_x % 8) return false;
    return true;
}

int cfi_mmq_skinny_group_launch(uint32_t ty, int n, const void* const* x, const void* y, float* const* dst,
                                const uint32_t* nrows, const uint32_t* stride_row_x, const uint32_t* stride_col_dst,
                                uint32_t K, uint32_t ncols_dst, uint32_t ncols_y, unsigned int* err, cudaStream_t stream,
                                bool pdl, const CfiPeerDev* peers) {
    const int nt = (int)((ncols_dst + 7) / 8);
    const char* ew = getenv("CFI_MMQ_SKINNY_WARPS");
    const int w = ew && atoi(ew) == 16 ? 16 : (ew && atoi(ew) == 8 ? 8 : SK_DEFAULT_WARPS);
    const void* fn = sk_kernel(ty, nt, w);
    if (!fn || n < 1 || n > SK_MAX_GROUP || ncols_dst > ncols_y || K == 0 || K % 256 || (reinterpret_cast<uintptr_t>(y) & 15))
        return (int)cudaErrorInvalidValue;
    const SkDev dv = sk_dev();
    SkArgs a = {};
    uint32_t tiles = 0;
    for (int i = 0; i < n; i++) {
        if (nrows[i] == 0 || (reinterpret_cast<uintptr_t>(x[i]) & 15) || (ty == T_Q8_0 && stride_row_x[i] % 8))
            return (int)cudaErrorInvalidValue;
        a.x[i] = static_cast<const uint8_t*>(x[i]);
        a.dst[i] = dst[i];
        a.nrows[i] = nrows[i];
        a.stride_row_x[i] = stride_row_x[i];
        a.stride_col_dst[i] = stride_col_dst[i];
        a.tile_begin[i] = tiles;
        tiles += (nrows[i] + SK_TR - 1) / SK_TR;
    }
    a.ngroup = (uint32_t)n;
    a.y = static_cast<const uint8_t*>(y);
    a.ncols = ncols_dst;
    a.ncols_y = ncols_y;
    a.nchunks = K / 256;
    a.ntiles = tiles;
    a.err = err;
    if (peers) {
        a.pr = *peers;
    } else {
        a.pr.world = 1;  // rank 0, delta[0] = 0: local stores
    }
    SkPlan p;
    if (!sk_plan(ty, (uint32_t)nt, a.nchunks, a.ntiles, dv.sms, dv.smem_max, (uint32_t)w, p))
        return (int)cudaErrorInvalidValue;
    if (a.pr.world > 1 && (size_t)p.nx * p.ksplits >= CFI_PEER_UNIT) return (int)cudaErrorInvalidValue;  // signal units
    if (p.ksplits > 1) {
        int e1 = 0, e2 = 0;
        a.ws = static_cast<float*>(
            cfi_stream_buffer(CFI_BUF_SKINNY_WS, (size_t)a.ntiles * p.ksplits * SK_PART_FLOATS * 4, stream, &e1));
        a.counters = static_cast<unsigned int*>(cfi_stream_buffer(CFI_BUF_COUNTERS, (size_t)a.ntiles * 4, stream, &e2));
        if (!a.ws || !a.counters) return e1 ? e1 : (e2 ? e2 : (int)cudaErrorMemoryAllocation);
    }
    a.kr = p.kr;
    a.ksplits = p.ksplits;
    a.kp = p.kp;
    a.stages = p.stages;
    a.red_par = p.par ? 1u : 0u;
    static CfiPerDeviceOnce attr[2][2][SK_MAX_NT + 1];
    cfi_once_per_device(attr[ty == T_Q4_K][w == 16][nt], [&] {
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dv.smem_max);
    });
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3(p.nx, p.ksplits, 1);
    c.blockDim = dim3(w * 32, 1, 1);
    c.dynamicSmemBytes = p.smem;
    c.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = at;
    c.numAttrs = pdl ? 1 : 0;
    void* args[] = {&a};
    return (int)cudaLaunchKernelExC(&c, fn, args);
}

int cfi_mmq_skinny_launch(uint32_t ty, const void* x, const void* y, float* dst, uint32_t K, uint32_t nrows,
                          uint32_t ncols_dst, uint32_t ncols_y, uint32_t stride_row_x, uint32_t stride_col_dst,
                          unsigned int* err, cudaStream_t stream, bool pdl) {
    return cfi_mmq_skinny_group_launch(ty, 1, &x, y, &dst, &nrows, &stride_row_x, &stride_col_dst, K, ncols_dst, ncols_y,
                                       err, stream, pdl);
}
