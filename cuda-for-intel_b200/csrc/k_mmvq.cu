// k_mmvq.cu -- decode GEMV y = W x for quantized W (sm_100a), the native mul_mat_vec_q.
//
// Parameter list: ggml-cuda's mul_mat_vec_q<type, ncols_dst> (x, y, ids, dst, u32 ncols_x, uint3
// nchannels_y, u32 stride_row_x, stride_col_y, stride_col_dst, uint3 channel_ratio, u32
// stride_channel_x/y/dst, uint3 sample_ratio, u32 stride_sample_x/y/dst; cuda-for-intel
// src/subst/mod.rs:214-218) plus one trailing u32 `nrows` appended by the router, as the
// reference's decode-fast variant does (src/subst/mod.rs:529-536).
//
// Arithmetic: one warp per weight row; lane l takes the 32-value group l (Q8_0) or sub-block l%8
// of superblock l/8 (Q4_K), stepping 32 groups (4 superblocks) at a time, one fp32 accumulator per
// lane and column, then the 32-lane xor butterfly.  That is the reference's whole-group decode
// model with one warp per row and one accumulator (src/subst/refs.rs:435-497, `wide`), and every
// per-lane float operation uses explicit-rounding intrinsics in the reference's order
// (refs.rs:386-433), so each output column equals cfo_mmvq_fast(warps=1, unroll=1, wide) bit for
// bit; the integer block dot products are exact dp4a sums.
//
// Memory path (B200): a persistent grid, each CTA owning a contiguous range of rows of one
// channel/sample plane.  Before waiting on the previous kernel (programmatic dependent launch)
// every CTA asks L2 for its rows with bulk prefetches (cp.async.bulk.prefetch.L2), so the HBM
// stream of this GEMV overlaps the tail of whatever ran before it; prefetching into L2 cannot
// expose stale data (all reads still happen after griddepcontrol.wait, through the coherent L2).
// The CTA then lets its own dependents launch, waits, stages the q8_1 activations in shared
// memory once (block-major, split so lane-consecutive blocks are bank-conflict free) and each
// warp computes R rows at a time with every global load of an iteration issued before its math:
//   * Q8_0 (34-byte blocks, 2-byte aligned): the warp copies 32 blocks of each row into its own
//     shared buffer with 16-byte coalesced loads (ragged head/tail as halfwords: no byte outside
//     the row is read) and lane l takes block l;
//   * Q4_K (144-byte superblocks, 16-byte aligned): three 16-byte loads per lane straight from
//     global memory (L2).
#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "sm100_ptx.cuh"
#include "decode_epi.cuh"
#include "q81_block.cuh"
#include "mma_sync.cuh"
#include "../../include/cfi_glue.h"

#include <algorithm>

namespace {

using namespace sm100;

constexpr int NW = CFI_MMVQ_WARPS;   // warps per CTA
constexpr int WBUF_ROW = 1120;       // Q8_0: one 32-block chunk of a row + alignment slack + read-ahead

template <uint32_t TY> __host__ __device__ constexpr uint32_t block_bytes() {
    return TY == T_Q4_K ? Q4_K_BYTES : TY == T_Q6_K ? Q6_K_BYTES : TY == T_Q4_0 ? Q4_0_BYTES : Q8_0_BYTES;
}
template <uint32_t TY> __host__ __device__ constexpr uint32_t block_values() { return (TY == T_Q4_K || TY == T_Q6_K) ? QK_K : 32; }
__host__ __device__ inline uint32_t block_bytes_of(uint32_t ty) {
    return ty == T_Q4_K ? Q4_K_BYTES : ty == T_Q6_K ? Q6_K_BYTES : ty == T_Q4_0 ? Q4_0_BYTES : Q8_0_BYTES;
}
__host__ __device__ inline uint32_t block_values_of(uint32_t ty) { return (ty == T_Q4_K || ty == T_Q6_K) ? QK_K : 32; }
template <uint32_t TY, int NCOLS> __host__ __device__ constexpr int rows_per_warp() {
    return TY == T_Q4_K ? (NCOLS == 1 ? 2 : 1) : (NCOLS <= 2 ? 2 : 1);
}

CFI_DEV void l2_prefetch(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Activation stage: ya[c][b] = qs words 0..3, yb[c][b] = qs words 4..7, ym[c][b] = {d (fp32
// bits), aux}; 40 bytes per block and column.  aux: the sum of the 32 int8 quants (Q4_K); the
// block's s as fp32 bits (Q4_0); the sums of quants 0..15 and 16..31 as two int16 (Q6_K).
struct YStage {
    uint32_t ya, yb, ym;  // shared-space byte addresses
    uint32_t nb32;
};

template <uint32_t TY = T_Q4_K>
CFI_DEV YStage stage_y(uint8_t* smem, int ncols, const uint8_t* y0, size_t y_base, uint32_t stride_col_y, uint32_t nb32) {
    uint4* ya = reinterpret_cast<uint4*>(smem);
    uint4* yb = ya + (size_t)ncols * nb32;
    uint2* ym = reinterpret_cast<uint2*>(yb + (size_t)ncols * nb32);
    for (uint32_t idx = threadIdx.x; idx < (uint32_t)ncols * nb32; idx += blockDim.x) {
        const uint32_t c = idx / nb32, b = idx - c * nb32;
        const uint32_t* w = reinterpret_cast<const uint32_t*>(y0 + (y_base + (size_t)c * stride_col_y + b) * Q8_1_BYTES);
        uint32_t q[9];
#pragma unroll
        for (int i = 0; i < 9; i++) q[i] = __ldg(w + i);
        uint32_t aux;
        if (TY == T_Q4_0) {
            aux = __float_as_uint(h2f_bits((uint16_t)(q[0] >> 16)));
        } else if (TY == T_Q6_K) {
            int lo = 0, hi = 0;
#pragma unroll
            for (int i = 1; i < 5; i++) lo = dp4a(0x01010101, (int)q[i], lo);
#pragma unroll
            for (int i = 5; i < 9; i++) hi = dp4a(0x01010101, (int)q[i], hi);
            aux = ((uint32_t)lo & 0xffffu) | ((uint32_t)hi << 16);
        } else {
            int sm = 0;
#pragma unroll
            for (int i = 1; i < 9; i++) sm = dp4a(0x01010101, (int)q[i], sm);
            aux = (uint32_t)sm;
        }
        ya[idx] = make_uint4(q[1], q[2], q[3], q[4]);
        yb[idx] = make_uint4(q[5], q[6], q[7], q[8]);
        ym[idx] = make_uint2(__float_as_uint(h2f_bits((uint16_t)(q[0] & 0xffffu))), aux);
    }
    return YStage{smem_u32(ya), smem_u32(yb), smem_u32(ym), nb32};
}

// The activation stage of a GEMV that absorbed a deferred quantize_q8_1, built by a cluster of
// CTAs together: CTA `rank` of the cluster quantizes blocks rank, rank + cs, ... (one 8-thread
// group per 32-value block of x, q81_block.cuh: the quantizer's arithmetic) and stores each one
// into the stage of every CTA of the cluster (distributed shared memory), so the stage holds
// exactly what stage_y would have read from the quantizer's output.  The first cluster also
// stores every block, padding blocks (b >= nb32) included, to vy.  Ends with a cluster barrier:
// no CTA leaves while a peer may still store into its shared memory.  The kernel arrives at the
// cluster barrier on entry (mmvq_stream_body); the wait here completes that phase.
template <uint32_t TY>
CFI_DEV YStage stage_y_q81(uint8_t* smem, int ncols, const CfiFuseQ& f, uint32_t nb32) {
    uint4* ya = reinterpret_cast<uint4*>(smem);
    uint4* yb = ya + (size_t)ncols * nb32;
    uint2* ym = reinterpret_cast<uint2*>(yb + (size_t)ncols * nb32);
    const uint32_t cs = cluster_nctarank(), rank = cluster_ctarank();
    const bool writer = blockIdx.x < cs;  // the first cluster
    cluster_wait();  // every CTA of the cluster has started (arrived at kernel entry)
    const uint32_t total = (uint32_t)ncols * f.nbq;
    const uint32_t j = threadIdx.x & 7, groups = blockDim.x / 8;
    for (uint32_t base = 0; base * cs < total; base += groups) {
        const uint32_t idx = (base + threadIdx.x / 8) * cs + rank;
        const uint32_t c = idx / f.nbq, b = idx - c * f.nbq;
        const bool need = idx < total && (b < nb32 || writer);  // uniform over the 8-thread group
        const unsigned mask = __ballot_sync(0xffffffffu, need);
        if (!need) continue;
        const Q81Part p = q81_quantize4(q81_load4(f.x + (size_t)c * f.s01, (int64_t)b * 32 + 4 * j, f.ne00), mask);
        uint32_t qw;
        memcpy(&qw, &p.q, 4);
        // aux word of the stage (stage_y): quant sums as exact integer adds over the group
        int part = dp4a(0x01010101, (int)qw, 0);
        part += __shfl_xor_sync(mask, part, 1);
        part += __shfl_xor_sync(mask, part, 2);          // words 0-3 on threads 0-3, 4-7 on 4-7
        const int other = __shfl_xor_sync(mask, part, 4);
        uint32_t aux;
        if (TY == T_Q4_0)
            aux = __float_as_uint(h2f_bits((uint16_t)(p.ds >> 16)));
        else if (TY == T_Q6_K)
            aux = ((uint32_t)part & 0xffffu) | ((uint32_t)other << 16);
        else
            aux = (uint32_t)(part + other);
        if (writer) {
            uint8_t* blk = f.vy + (size_t)idx * Q8_1_BYTES;
            *reinterpret_cast<uint32_t*>(blk + 4 + 4 * j) = qw;
            if (j == 0) *reinterpret_cast<uint32_t*>(blk) = p.ds;
        }
        if (b < nb32) {
            const uint32_t s = c * nb32 + b;
            const uint32_t wa = j < 4 ? smem_u32(ya + s) + 4 * j : smem_u32(yb + s) + 4 * (j - 4);
            const uint32_t ma = smem_u32(ym + s);
            const uint32_t dbits = __float_as_uint(h2f_bits((uint16_t)(p.ds & 0xffffu)));
            for (uint32_t t = 0; t < cs; t++) {
                st_cluster_u32(mapa_shared(wa, t), qw);
                if (j == 0) st_cluster_v2(mapa_shared(ma, t), dbits, aux);
            }
        }
    }
    __syncwarp();
    cluster_sync();
    return YStage{smem_u32(ya), smem_u32(yb), smem_u32(ym), nb32};
}

CFI_DEV size_t y_bytes(int ncols, uint32_t nb32) { return ((size_t)ncols * nb32 * 40 + 127) & ~(size_t)127; }

// 8-word integer dot in two independent dp4a chains (exact: integer adds commute).
CFI_DEV int dot8(const int (&w)[8], uint4 a, uint4 b) {
    int s0 = dp4a(w[0], (int)a.x, 0), s1 = dp4a(w[1], (int)a.y, 0);
    s0 = dp4a(w[2], (int)a.z, s0);
    s1 = dp4a(w[3], (int)a.w, s1);
    s0 = dp4a(w[4], (int)b.x, s0);
    s1 = dp4a(w[5], (int)b.y, s1);
    s0 = dp4a(w[6], (int)b.z, s0);
    s1 = dp4a(w[7], (int)b.w, s1);
    return s0 + s1;
}

// Q4_K lane state of one superblock: nibble words of sub-block g, its 6-bit scale and min, d, dmin.
struct Q4K {
    int v[8];
    int sc, m;
    float dx, dmin;
};

// get_scale_min_k4 without data-dependent selects (sh = 8 * (g & 3)).
CFI_DEV Q4K q4k_decode(uint4 h, uint4 q0, uint4 q1, int g, uint32_t sh, uint32_t nsh) {
    Q4K r;
    r.dx = h2f_bits((uint16_t)(h.x & 0xffffu));
    r.dmin = h2f_bits((uint16_t)(h.x >> 16));
    const uint32_t a = h.y >> sh, b = h.z >> sh, c = h.w >> sh;
    if (g < 4) {
        r.sc = (int)(a & 63u);
        r.m = (int)(b & 63u);
    } else {
        r.sc = (int)((c & 15u) | ((a >> 2) & 0x30u));
        r.m = (int)(((c >> 4) & 15u) | ((b >> 2) & 0x30u));
    }
    r.v[0] = (int)((q0.x >> nsh) & 0x0F0F0F0Fu);
    r.v[1] = (int)((q0.y >> nsh) & 0x0F0F0F0Fu);
    r.v[2] = (int)((q0.z >> nsh) & 0x0F0F0F0Fu);
    r.v[3] = (int)((q0.w >> nsh) & 0x0F0F0F0Fu);
    r.v[4] = (int)((q1.x >> nsh) & 0x0F0F0F0Fu);
    r.v[5] = (int)((q1.y >> nsh) & 0x0F0F0F0Fu);
    r.v[6] = (int)((q1.z >> nsh) & 0x0F0F0F0Fu);
    r.v[7] = (int)((q1.w >> nsh) & 0x0F0F0F0Fu);
    return r;
}

template <int NCOLS>
CFI_DEV void store_row(const float (&acc)[NCOLS], uint32_t lane, float* dst_row, uint32_t stride_col_dst) {
#pragma unroll
    for (int c = 0; c < NCOLS; c++) {
        const float v = warp_sum(acc[c]);
        if (lane == 0) dst_row[(size_t)c * stride_col_dst] = v;
    }
}

template <uint32_t TY, int NCOLS>
__global__ void __launch_bounds__(NW * 32)
    cfi_mmvq_rows(const void* __restrict__ vx, const void* __restrict__ vy, const int32_t* __restrict__ ids,
             float* __restrict__ dst, uint32_t ncols_x, uint3 nchannels_y, uint32_t stride_row_x,
             uint32_t stride_col_y, uint32_t stride_col_dst, uint3 channel_ratio, uint32_t stride_channel_x,
             uint32_t stride_channel_y, uint32_t stride_channel_dst, uint3 sample_ratio, uint32_t stride_sample_x,
             uint32_t stride_sample_y, uint32_t stride_sample_dst, uint32_t nrows, uint32_t /*chunk_rows*/,
             uint32_t /*nstages*/) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int R = rows_per_warp<TY, NCOLS>();
    constexpr uint32_t BB = block_bytes<TY>();
    const uint32_t nb32 = ncols_x / 32;
    const uint32_t nb = TY == T_Q4_K ? ncols_x / QK_K : ncols_x / QK8_0;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t channel_dst = blockIdx.y, sample_dst = blockIdx.z;
    const bool use_ids = NCOLS == 1 && ids != nullptr;
    const uint32_t sample_x = fastdiv(sample_dst, sample_ratio);
    const uint32_t rbeg = (uint32_t)((uint64_t)blockIdx.x * nrows / gridDim.x);
    const uint32_t rend = (uint32_t)((uint64_t)(blockIdx.x + 1) * nrows / gridDim.x);

    // ---- L2 prefetch of this CTA's rows (the ids table may come from the previous kernel: skip) ----
    if (!use_ids && threadIdx.x == 0 && rend > rbeg) {
        const uint32_t channel_x = fastdiv(channel_dst, channel_ratio);
        const uint8_t* plane = static_cast<const uint8_t*>(vx) + ((size_t)sample_x * stride_sample_x + (size_t)channel_x * stride_channel_x) * BB;
        const uintptr_t s = reinterpret_cast<uintptr_t>(plane + (size_t)rbeg * stride_row_x * BB);
        const uintptr_t e = reinterpret_cast<uintptr_t>(plane + ((size_t)(rend - 1) * stride_row_x + nb) * BB);
        uintptr_t a0 = (s + 15) & ~(uintptr_t)15;
        const uintptr_t a1 = e & ~(uintptr_t)15;
        while (a0 < a1) {
            const uint32_t n = (uint32_t)min((uintptr_t)(1u << 20), a1 - a0);
            l2_prefetch(reinterpret_cast<const void*>(a0), n);
            a0 += n;
        }
    }
    pdl_launch_dependents();
    pdl_wait();

    const uint32_t channel_x = use_ids ? (uint32_t)ids[channel_dst] : fastdiv(channel_dst, channel_ratio);
    const uint32_t channel_y = use_ids ? fastmodulo(channel_dst, nchannels_y) : channel_dst;
    const size_t y_base = (size_t)sample_dst * stride_sample_y + (size_t)channel_y * stride_channel_y;
    const YStage y = stage_y(smem, NCOLS, static_cast<const uint8_t*>(vy), y_base, stride_col_y, nb32);
    __syncthreads();

    const uint8_t* plane = static_cast<const uint8_t*>(vx) + ((size_t)sample_x * stride_sample_x + (size_t)channel_x * stride_channel_x) * BB;
    float* dplane = dst + (size_t)sample_dst * stride_sample_dst + (size_t)channel_dst * stride_channel_dst;

    if constexpr (TY == T_Q4_K) {
        const int g = (int)(lane & 7);
        const uint32_t sh = 8u * (uint32_t)(g & 3), nsh = 4u * (uint32_t)(g & 1);
        for (uint32_t r0 = rbeg + warp * R; r0 < rend; r0 += NW * R) {
            const uint8_t* rp[R];
#pragma unroll
            for (int j = 0; j < R; j++) rp[j] = plane + (size_t)min(r0 + j, rend - 1) * stride_row_x * BB;
            float acc[R][NCOLS];
#pragma unroll
            for (int j = 0; j < R; j++)
#pragma unroll
                for (int c = 0; c < NCOLS; c++) acc[j][c] = 0.0f;
            uint32_t ya = y.ya + lane * 16, yb = y.yb + lane * 16, ym = y.ym + lane * 8;
            for (uint32_t sb = lane >> 3; sb < nb; sb += 4, ya += 512, yb += 512, ym += 256) {
                uint4 h[R], q0[R], q1[R];
#pragma unroll
                for (int j = 0; j < R; j++) {
                    const uint4* b4 = reinterpret_cast<const uint4*>(rp[j] + (size_t)sb * Q4_K_BYTES);
                    h[j] = __ldg(b4);
                    q0[j] = __ldg(b4 + 1 + 2 * (g >> 1));
                    q1[j] = __ldg(b4 + 2 + 2 * (g >> 1));
                }
                Q4K wl[R];
#pragma unroll
                for (int j = 0; j < R; j++) wl[j] = q4k_decode(h[j], q0[j], q1[j], g, sh, nsh);
#pragma unroll
                for (int c = 0; c < NCOLS; c++) {
                    const uint4 a0 = lds128(ya + c * nb32 * 16), a1 = lds128(yb + c * nb32 * 16);
                    const uint2 m2 = lds64(ym + c * nb32 * 8);
                    const float d8 = __uint_as_float(m2.x);
#pragma unroll
                    for (int j = 0; j < R; j++) {
                        const int sumi = dot8(wl[j].v, a0, a1);
                        const float a = __fmul_rn(d8, (float)(sumi * wl[j].sc));
                        const float bm = __fmul_rn(d8, (float)((int)m2.y * wl[j].m));
                        acc[j][c] = __fadd_rn(acc[j][c], __fsub_rn(__fmul_rn(wl[j].dx, a), __fmul_rn(wl[j].dmin, bm)));
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < R; j++)
                if (r0 + j < rend) store_row<NCOLS>(acc[j], lane, dplane + r0 + j, stride_col_dst);
        }
    } else {
        // per-warp row buffers: R rows x (32 blocks + slack)
        uint8_t* wbuf = smem + y_bytes(NCOLS, nb32) + (size_t)warp * R * WBUF_ROW;
        const uint32_t wbuf_s = smem_u32(wbuf);
        for (uint32_t r0 = rbeg + warp * R; r0 < rend; r0 += NW * R) {
            float acc[R][NCOLS];
#pragma unroll
            for (int j = 0; j < R; j++)
#pragma unroll
                for (int c = 0; c < NCOLS; c++) acc[j][c] = 0.0f;
            for (uint32_t b0 = 0; b0 < nb; b0 += 32) {
                const uint32_t n = min(32u, nb - b0);
                uint32_t off[R];
                // copy 32 blocks of each row: all 16-byte loads of the R rows first, then the stores
                uint4 v[R][3];
                uint16_t hh[R];
                uint32_t nvec[R], nhead[R], ntail[R], a0o[R], a1o[R];
#pragma unroll
                for (int j = 0; j < R; j++) {
                    const uint32_t row = min(r0 + j, rend - 1);
                    const uintptr_t cs = reinterpret_cast<uintptr_t>(plane + (size_t)row * stride_row_x * BB) + (uintptr_t)b0 * Q8_0_BYTES;
                    const uintptr_t ce = cs + (uintptr_t)n * Q8_0_BYTES;
                    const uintptr_t base = cs & ~(uintptr_t)15;
                    const uintptr_t a0 = (cs + 15) & ~(uintptr_t)15, a1 = ce & ~(uintptr_t)15;
                    nvec[j] = (uint32_t)((a1 - a0) >> 4);
                    off[j] = (uint32_t)(cs - base);
                    a0o[j] = (uint32_t)(a0 - base);
                    a1o[j] = (uint32_t)(a1 - base);
#pragma unroll
                    for (int k = 0; k < 3; k++) {
                        const uint32_t idx = lane + 32u * k;
                        v[j][k] = idx < nvec[j] ? __ldg(reinterpret_cast<const uint4*>(a0) + idx) : make_uint4(0, 0, 0, 0);
                    }
                    nhead[j] = (uint32_t)((a0 - cs) >> 1);
                    ntail[j] = (uint32_t)((ce - a1) >> 1);
                    hh[j] = 0;
                    if (lane < nhead[j])
                        hh[j] = __ldg(reinterpret_cast<const unsigned short*>(cs) + lane);
                    else if (lane >= 8 && lane - 8 < ntail[j])
                        hh[j] = __ldg(reinterpret_cast<const unsigned short*>(a1) + (lane - 8));
                }
#pragma unroll
                for (int j = 0; j < R; j++) {
#pragma unroll
                    for (int k = 0; k < 3; k++) {
                        const uint32_t idx = lane + 32u * k;
                        if (idx < nvec[j]) *reinterpret_cast<uint4*>(wbuf + j * WBUF_ROW + a0o[j] + 16 * idx) = v[j][k];
                    }
                    if (lane < nhead[j])
                        reinterpret_cast<uint16_t*>(wbuf + j * WBUF_ROW + off[j])[lane] = hh[j];
                    else if (lane >= 8 && lane - 8 < ntail[j])
                        reinterpret_cast<uint16_t*>(wbuf + j * WBUF_ROW + a1o[j])[lane - 8] = hh[j];
                }
                __syncwarp();
                if (lane < n) {
                    const uint32_t b = b0 + lane;
                    int wq[R][8];
                    float dx[R];
#pragma unroll
                    for (int j = 0; j < R; j++) {
                        const uint32_t blk = wbuf_s + j * WBUF_ROW + off[j] + lane * Q8_0_BYTES;
                        dx[j] = h2f_bits((uint16_t)lds16(blk));
                        const uint32_t qo = blk + 2, shq = (qo & 3u) * 8, wa = qo & ~3u;
                        uint32_t prev = lds32(wa);
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const uint32_t nxt = lds32(wa + 4 * (i + 1));
                            wq[j][i] = (int)__funnelshift_r(prev, nxt, shq);
                            prev = nxt;
                        }
                    }
#pragma unroll
                    for (int c = 0; c < NCOLS; c++) {
                        const uint4 a0 = lds128(y.ya + (c * nb32 + b) * 16), a1 = lds128(y.yb + (c * nb32 + b) * 16);
                        const float d8 = __uint_as_float(lds32(y.ym + (c * nb32 + b) * 8));
#pragma unroll
                        for (int j = 0; j < R; j++)
                            acc[j][c] = __fmaf_rn(__fmul_rn(dx[j], d8), (float)dot8(wq[j], a0, a1), acc[j][c]);
                    }
                }
                __syncwarp();
            }
#pragma unroll
            for (int j = 0; j < R; j++)
                if (r0 + j < rend) store_row<NCOLS>(acc[j], lane, dplane + r0 + j, stride_col_dst);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Streaming kernel (ncols_dst 1 and 2): weights staged through shared memory by bulk copies.
//
// Launch order with programmatic dependent launch: before waiting on its predecessor a CTA only
// asks L2 for its weight rows (a hint, never a read) and lets its own dependents launch, so a
// chain of GEMVs (with the quantizer between them, which also triggers first) keeps several
// grids resident and the HBM stream of later launches overlaps the work of earlier ones.  After
// the wait the CTA copies its rows L2 -> shared memory in chunks (cp.async.bulk, up to four
// stages, 16-byte-aligned interior of every row; Q8_0's ragged 2-byte ends by plain loads) while
// it stages the q8_1 activations, and computes chunk k while later chunks land.  Where a CTA
// refills its stages, each warp takes its rows of a chunk as soon as the chunk has landed and
// counts itself out of the stage; the last warp out refills it (no CTA-wide barrier per chunk).
//
// Arithmetic (per output column, bit-exact to the one-warp decode-fast model of the reference,
// src/subst/refs.rs:435-497): model lane l accumulates the 32-value groups l, l+32, l+64, ... of
// its row in that order and the 32 lane sums are combined by the xor butterfly 16, 8, 4, 2, 1.
//   * Q4_K: 16 threads per row; thread j computes model lanes 2j and 2j+1, which read the low and
//     high nibbles of the same 32 bytes, so each 32-byte chunk is loaded once; the butterfly
//     becomes xor 8, 4, 2, 1 across the 16 threads for both lanes, then lane 2j + lane 2j+1.  The
//     high-nibble dot is taken on the bytes masked with 0xF0 (unsigned x signed dp4a, 16x the
//     nibble dot, exact) and shifted back.
//   * Q8_0: one warp per row, lane l = model lane l.
// R rows per team are computed together so their loads and butterflies interleave.
constexpr uint32_t ST_MAX_STAGES = 4;
constexpr int DIRECT_U = 4;  // 16-byte pieces per thread and chunk of the direct fill

// Shared-memory layout of one stage.  Dense rows (stride_row_x == blocks per row) are copied as
// one contiguous range, row k of the chunk at (address of its first row & 15) + k * row_bytes;
// strided rows are copied one by one at k * pitch + (row address & 15).
__host__ __device__ inline uint32_t st_pitch(uint32_t row_bytes) { return ((row_bytes + 15u) & ~15u) + 16u; }
__host__ __device__ inline uint32_t st_row_stride(uint32_t row_bytes, bool dense) { return dense ? row_bytes : st_pitch(row_bytes); }
__host__ __device__ inline uint32_t st_stage_bytes(uint32_t chunk_rows, uint32_t row_bytes, bool dense) {
    return (chunk_rows * st_row_stride(row_bytes, dense) + 16u + 127u) & ~127u;
}

static __device__ unsigned int g_mmvq_error;
static __device__ int g_mmvq_abort;  // never set: the bounded waits end on their time limit

CFI_DEV int dp4a_us(uint32_t a, uint32_t b, int c) {  // unsigned bytes of a x signed bytes of b
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
CFI_DEV int dot8m(const uint32_t (&q)[8], uint32_t mask, uint4 a, uint4 b) {
    int s0 = dp4a_us(q[0] & mask, a.x, 0), s1 = dp4a_us(q[1] & mask, a.y, 0);
    s0 = dp4a_us(q[2] & mask, a.z, s0);
    s1 = dp4a_us(q[3] & mask, a.w, s1);
    s0 = dp4a_us(q[4] & mask, b.x, s0);
    s1 = dp4a_us(q[5] & mask, b.y, s1);
    s0 = dp4a_us(q[6] & mask, b.z, s0);
    s1 = dp4a_us(q[7] & mask, b.w, s1);
    return s0 + s1;
}
// get_scale_min_k4 for sub-block g of a superblock header (scales in words h.y, h.z, h.w)
CFI_DEV void q4k_scale_min(uint4 h, uint32_t g, int& sc, int& m) {
    const uint32_t sh = 8u * (g & 3u);
    const uint32_t a = h.y >> sh, b = h.z >> sh, c = h.w >> sh;
    if (g < 4) {
        sc = (int)(a & 63u);
        m = (int)(b & 63u);
    } else {
        sc = (int)((c & 15u) | ((a >> 2) & 0x30u));
        m = (int)(((c >> 4) & 15u) | ((b >> 2) & 0x30u));
    }
}
CFI_DEV float q4k_term(float dx, float dmin, float d8, int sumi, int sc, int sumy, int m, float acc) {
    const float a = __fmul_rn(d8, (float)(sumi * sc));
    const float b = __fmul_rn(d8, (float)(sumy * m));
    return __fadd_rn(acc, __fsub_rn(__fmul_rn(dx, a), __fmul_rn(dmin, b)));
}

// Rows of one chunk.  Each pass holds the weights of R rows per team in registers and streams
// the activations column by column, so a column's q8_1 block is read once per R rows.
CFI_DEV int dot8u(const uint32_t (&q)[8], uint4 a, uint4 b) {
    int s0 = dp4a_us(q[0], a.x, 0), s1 = dp4a_us(q[1], a.y, 0);
    s0 = dp4a_us(q[2], a.z, s0);
    s1 = dp4a_us(q[3], a.w, s1);
    s0 = dp4a_us(q[4], b.x, s0);
    s1 = dp4a_us(q[5], b.y, s1);
    s0 = dp4a_us(q[6], b.z, s0);
    s1 = dp4a_us(q[7], b.w, s1);
    return s0 + s1;
}

// Q4_K: 2 rows per team and pass (each activation block read once per 2 rows); the nibble words
// are masked once per row for up to 4 columns, per column beyond (register budget)
template <int NCOLS> constexpr int q4k_rows() { return 2; }
template <int NCOLS> constexpr bool q4k_hoist() { return NCOLS <= 4; }

template <int NCOLS>
CFI_DEV void q4k_chunk(uint32_t sbase, uint32_t rstride, uint32_t r0, uint32_t r1, const YStage& y, uint32_t tid,
                       float* dplane, uint32_t stride_col_dst) {
    constexpr int R = q4k_rows<NCOLS>();
    constexpr uint32_t NTEAM = NW * 32 / 16;
    const uint32_t j = tid & 15, team = tid >> 4, c4 = j & 3;
    const uint32_t G = y.nb32;
    for (uint32_t p0 = r0; p0 < r1; p0 += NTEAM * R) {
        float acc[R][NCOLS][2];
#pragma unroll
        for (int k = 0; k < R; k++)
#pragma unroll
            for (int c = 0; c < NCOLS; c++) acc[k][c][0] = acc[k][c][1] = 0.0f;
        for (uint32_t g0 = 2 * j; g0 < G; g0 += 32) {
            const uint32_t sbo = (g0 >> 3) * Q4_K_BYTES;
            constexpr bool H = q4k_hoist<NCOLS>();
            uint32_t ql[R][8], qh[R][H ? 8 : 1];  // low nibbles (or raw words), high nibbles in place (16 x value)
            int sc0[R], mn0[R], sc1[R], mn1[R];
            float dx[R], dmin[R];
#pragma unroll
            for (int k = 0; k < R; k++) {
                const uint32_t r = min(p0 + team + NTEAM * k, r1 - 1);
                const uint32_t a = sbase + (r - r0) * rstride + sbo;
                const uint4 h = lds128(a), q0 = lds128(a + 16 + 32 * c4), q1 = lds128(a + 32 + 32 * c4);
                dx[k] = h2f_bits((uint16_t)(h.x & 0xffffu));
                dmin[k] = h2f_bits((uint16_t)(h.x >> 16));
                const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    if constexpr (H) {
                        ql[k][i] = qw[i] & 0x0F0F0F0Fu;
                        qh[k][i] = qw[i] & 0xF0F0F0F0u;
                    } else {
                        ql[k][i] = qw[i];
                    }
                }
                q4k_scale_min(h, 2 * c4, sc0[k], mn0[k]);
                q4k_scale_min(h, 2 * c4 + 1, sc1[k], mn1[k]);
            }
#pragma unroll
            for (int c = 0; c < NCOLS; c++) {
                const uint32_t o = c * G + g0;
                const uint4 ya0 = lds128(y.ya + o * 16), yb0 = lds128(y.yb + o * 16);
                const uint4 ya1 = lds128(y.ya + o * 16 + 16), yb1 = lds128(y.yb + o * 16 + 16);
                const uint2 m0 = lds64(y.ym + o * 8), m1 = lds64(y.ym + o * 8 + 8);
#pragma unroll
                for (int k = 0; k < R; k++) {
                    int lo, hi;
                    if constexpr (H) {
                        lo = dot8u(ql[k], ya0, yb0);
                        hi = dot8u(qh[k], ya1, yb1) >> 4;
                    } else {
                        lo = dot8m(ql[k], 0x0F0F0F0Fu, ya0, yb0);
                        hi = dot8m(ql[k], 0xF0F0F0F0u, ya1, yb1) >> 4;
                    }
                    acc[k][c][0] = q4k_term(dx[k], dmin[k], __uint_as_float(m0.x), lo, sc0[k], (int)m0.y, mn0[k], acc[k][c][0]);
                    acc[k][c][1] = q4k_term(dx[k], dmin[k], __uint_as_float(m1.x), hi, sc1[k], (int)m1.y, mn1[k], acc[k][c][1]);
                }
            }
        }
        // model butterfly: lanes 2j and 2j+1 pair with 2(j^8), 2(j^4), 2(j^2), 2(j^1) (+0/+1), then with each other
#pragma unroll
        for (int k = 0; k < R; k++) {
            const uint32_t r = p0 + team + NTEAM * k;
#pragma unroll
            for (int c = 0; c < NCOLS; c++) {
                float a0 = acc[k][c][0], a1 = acc[k][c][1];
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) {
                    a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, o));
                    a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, o));
                }
                if (j == 0 && r < r1) dplane[(size_t)c * stride_col_dst + r] = __fadd_rn(a0, a1);
            }
        }
    }
}

template <int NCOLS>
CFI_DEV void q80_chunk(uint32_t sbase, uint32_t rstride, bool dense, uint32_t r0, uint32_t r1, const YStage& y,
                       uint32_t lane, uint32_t warp, uintptr_t plane, uint32_t stride_row_x, float* dplane,
                       uint32_t stride_col_dst) {
    constexpr int R = NCOLS == 1 ? 4 : 2;
    const uint32_t nb = y.nb32;
    for (uint32_t p0 = r0; p0 < r1; p0 += NW * R) {
        float acc[R][NCOLS];
        uint32_t rb[R];
#pragma unroll
        for (int k = 0; k < R; k++) {
            const uint32_t r = min(p0 + warp + NW * k, r1 - 1);
            const uintptr_t rs = plane + (uintptr_t)(dense ? r0 : r) * stride_row_x * Q8_0_BYTES;
            rb[k] = sbase + (r - r0) * rstride + (uint32_t)(rs & 15);
#pragma unroll
            for (int c = 0; c < NCOLS; c++) acc[k][c] = 0.0f;
        }
        for (uint32_t b = lane; b < nb; b += 32) {
            int wq[R][8];
            float dx[R];
#pragma unroll
            for (int k = 0; k < R; k++) {
                const uint32_t blk = rb[k] + b * Q8_0_BYTES;
                dx[k] = h2f_bits((uint16_t)lds16(blk));
                const uint32_t qo = blk + 2, shq = (qo & 3u) * 8, wa = qo & ~3u;
                uint32_t prev = lds32(wa);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const uint32_t nxt = lds32(wa + 4 * (i + 1));
                    wq[k][i] = (int)__funnelshift_r(prev, nxt, shq);
                    prev = nxt;
                }
            }
#pragma unroll
            for (int c = 0; c < NCOLS; c++) {
                const uint4 ya = lds128(y.ya + (c * nb + b) * 16), yb = lds128(y.yb + (c * nb + b) * 16);
                const float d8 = __uint_as_float(lds32(y.ym + (c * nb + b) * 8));
#pragma unroll
                for (int k = 0; k < R; k++)
                    acc[k][c] = __fmaf_rn(__fmul_rn(dx[k], d8), (float)dot8(wq[k], ya, yb), acc[k][c]);
            }
        }
#pragma unroll
        for (int k = 0; k < R; k++) {
            const uint32_t r = p0 + warp + NW * k;
#pragma unroll
            for (int c = 0; c < NCOLS; c++) {
                float v = acc[k][c];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
                if (lane == 0 && r < r1) dplane[(size_t)c * stride_col_dst + r] = v;
            }
        }
    }
}

// 8 consecutive words starting at the 2-byte-aligned shared address a.
CFI_DEV void lds8w(uint32_t a, uint32_t (&w)[8]) {
    const uint32_t sh = (a & 3u) * 8, wa = a & ~3u;
    uint32_t prev = lds32(wa);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t nxt = lds32(wa + 4 * (i + 1));
        w[i] = __funnelshift_r(prev, nxt, sh);
        prev = nxt;
    }
}

// Q4_0 (never `wide` in the reference: refs.rs vec_dot Q4_0, two threads per block): model lane l
// takes words kqs = 2 (l & 1), kqs + 1 of block l / 2 + 16 i; one warp per row.
template <int NCOLS>
CFI_DEV void q40_chunk(uint32_t sbase, uint32_t rstride, bool dense, uint32_t r0, uint32_t r1, const YStage& y,
                       uint32_t lane, uint32_t warp, uintptr_t plane, uint32_t stride_row_x, float* dplane,
                       uint32_t stride_col_dst) {
    constexpr int R = NCOLS == 1 ? 4 : 2;
    const uint32_t nb = y.nb32, kqs = 2 * (lane & 1);
    for (uint32_t p0 = r0; p0 < r1; p0 += NW * R) {
        float acc[R][NCOLS];
        uint32_t rb[R];
#pragma unroll
        for (int k = 0; k < R; k++) {
            const uint32_t r = min(p0 + warp + NW * k, r1 - 1);
            const uintptr_t rs = plane + (uintptr_t)(dense ? r0 : r) * stride_row_x * Q4_0_BYTES;
            rb[k] = sbase + (r - r0) * rstride + (uint32_t)(rs & 15);
#pragma unroll
            for (int c = 0; c < NCOLS; c++) acc[k][c] = 0.0f;
        }
        for (uint32_t b = lane >> 1; b < nb; b += 16) {
            uint32_t v0[R], v1[R];
            float d4[R];
#pragma unroll
            for (int k = 0; k < R; k++) {
                const uint32_t blk = rb[k] + b * Q4_0_BYTES;
                d4[k] = h2f_bits((uint16_t)lds16(blk));
                const uint32_t qo = blk + 2 + 4 * kqs, sh = (qo & 3u) * 8, wa = qo & ~3u;
                const uint32_t w0 = lds32(wa), w1 = lds32(wa + 4), w2 = lds32(wa + 8);
                v0[k] = __funnelshift_r(w0, w1, sh);
                v1[k] = __funnelshift_r(w1, w2, sh);
            }
#pragma unroll
            for (int c = 0; c < NCOLS; c++) {
                const uint32_t o = c * nb + b;
                const uint2 ua = lds64(y.ya + o * 16 + 4 * kqs), ub = lds64(y.yb + o * 16 + 4 * kqs);
                const uint2 m = lds64(y.ym + o * 8);
                const float d8 = __uint_as_float(m.x), s8 = __uint_as_float(m.y);
#pragma unroll
                for (int k = 0; k < R; k++) {
                    int sumi = dp4a((int)(v0[k] & 0x0F0F0F0Fu), (int)ua.x, 0);
                    sumi = dp4a((int)((v0[k] >> 4) & 0x0F0F0F0Fu), (int)ub.x, sumi);
                    sumi = dp4a((int)(v1[k] & 0x0F0F0F0Fu), (int)ua.y, sumi);
                    sumi = dp4a((int)((v1[k] >> 4) & 0x0F0F0F0Fu), (int)ub.y, sumi);
                    const float inner = __fmaf_rn(d8, (float)sumi, __fmul_rn(s8, -4.0f));
                    acc[k][c] = __fmaf_rn(d4[k], inner, acc[k][c]);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < R; k++) {
            const uint32_t r = p0 + warp + NW * k;
#pragma unroll
            for (int c = 0; c < NCOLS; c++) {
                float v = acc[k][c];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
                if (lane == 0 && r < r1) dplane[(size_t)c * stride_col_dst + r] = v;
            }
        }
    }
}

// Q6_K (wide, refs.rs vec_dot_wide Q6_K): model lane l takes 32-value group g = l & 7 (half
// h = g / 4, quarter sub = g % 4) of superblock l / 8 + 4 i; one warp per row.  6-bit quants are
// the low or high nibble of ql plus 2 bits of qh; per 16 values an int8 scale.
template <int NCOLS>
CFI_DEV void q6k_chunk(uint32_t sbase, uint32_t rstride, bool dense, uint32_t r0, uint32_t r1, const YStage& y,
                       uint32_t lane, uint32_t warp, uintptr_t plane, uint32_t stride_row_x, float* dplane,
                       uint32_t stride_col_dst) {
    constexpr int R = NCOLS == 1 ? 2 : 1;
    const uint32_t nb32 = y.nb32, nsb = nb32 / 8;
    const uint32_t g = lane & 7, h = g >> 2, sub = g & 3;
    for (uint32_t p0 = r0; p0 < r1; p0 += NW * R) {
        float acc[R][NCOLS];
        uint32_t rb[R];
#pragma unroll
        for (int k = 0; k < R; k++) {
            const uint32_t r = min(p0 + warp + NW * k, r1 - 1);
            const uintptr_t rs = plane + (uintptr_t)(dense ? r0 : r) * stride_row_x * Q6_K_BYTES;
            rb[k] = sbase + (r - r0) * rstride + (uint32_t)(rs & 15);
#pragma unroll
            for (int c = 0; c < NCOLS; c++) acc[k][c] = 0.0f;
        }
        for (uint32_t sb = lane >> 3; sb < nsb; sb += 4) {
            uint32_t q[R][8];
            int sc0[R], sc1[R];
            float dx[R];
#pragma unroll
            for (int k = 0; k < R; k++) {
                const uint32_t blk = rb[k] + sb * Q6_K_BYTES;
                dx[k] = h2f_bits((uint16_t)lds16(blk + 208));
                const uint32_t scw = lds16(blk + 192 + 8 * h + 2 * sub);
                sc0[k] = (int)(int8_t)(scw & 0xffu);
                sc1[k] = (int)(int8_t)(scw >> 8);
                uint32_t ql[8], qh[8];
                lds8w(blk + 64 * h + 32 * (sub & 1), ql);
                lds8w(blk + 128 + 32 * h, qh);
                const uint32_t lsh = 4 * (sub >> 1), hsh = 2 * sub;
#pragma unroll
                for (int i = 0; i < 8; i++) q[k][i] = ((ql[i] >> lsh) & 0x0F0F0F0Fu) | (((qh[i] >> hsh) & 0x03030303u) << 4);
            }
#pragma unroll
            for (int c = 0; c < NCOLS; c++) {
                const uint32_t o = c * nb32 + sb * 8 + g;
                const uint4 ya = lds128(y.ya + o * 16), yb = lds128(y.yb + o * 16);
                const uint2 m = lds64(y.ym + o * 8);
                const float d8 = __uint_as_float(m.x);
                const int su0 = (int)(int16_t)(m.y & 0xffffu), su1 = (int)(int16_t)(m.y >> 16);
#pragma unroll
                for (int k = 0; k < R; k++) {
                    int s0 = dp4a((int)q[k][0], (int)ya.x, 0);
                    s0 = dp4a((int)q[k][1], (int)ya.y, s0);
                    s0 = dp4a((int)q[k][2], (int)ya.z, s0);
                    s0 = dp4a((int)q[k][3], (int)ya.w, s0);
                    int s1 = dp4a((int)q[k][4], (int)yb.x, 0);
                    s1 = dp4a((int)q[k][5], (int)yb.y, s1);
                    s1 = dp4a((int)q[k][6], (int)yb.z, s1);
                    s1 = dp4a((int)q[k][7], (int)yb.w, s1);
                    const int tot = (s0 - (su0 << 5)) * sc0[k] + (s1 - (su1 << 5)) * sc1[k];
                    acc[k][c] = __fmaf_rn(__fmul_rn(dx[k], d8), (float)tot, acc[k][c]);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < R; k++) {
            const uint32_t r = p0 + warp + NW * k;
#pragma unroll
            for (int c = 0; c < NCOLS; c++) {
                float v = acc[k][c];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
                if (lane == 0 && r < r1) dplane[(size_t)c * stride_col_dst + r] = v;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Tensor-core Q4_K GEMV for 3..8 columns (tolerance mode: the int32 block dots are exact, the fp32
// scale arithmetic is reassociated; outputs agree with the reference's fp32 order to about 1e-7
// relative).  The bit-exact decode-fast kernels above stay selectable (CFI_MMVQ_EXACT=1).
//
// y[r, c] = sum_sb d[r,sb] * sum_j d8[c,j] * sc[r,j] * sumi[r,c,j]  -  dmin[r,sb] * sum_j m[r,j] * dsum[c,j]
// with j the 32-value sub-blocks of superblock sb, sumi the exact int8 block dot and dsum = d8 * sumq.
//   * sumi: one mma.sync.m16n8k32 (u8 x s8 -> s32) per sub-block gives it for 16 weight rows and
//     all 8 columns; the A fragments of a 32-byte nibble chunk (two sub-blocks) come from one
//     ldmatrix.x4 of 16 rows, masked with 0x0F (low sub-block) or 0xF0 (high: 16 x sumi, the 1/16
//     folded into that sub-block's staged d8);
//   * the min term of a superblock is a 16 x 8 x 8 product (m over its 8 sub-blocks times dsum):
//     two mma.sync.m16n8k8 tf32 with m exact and dsum split into tf32 hi + lo parts (~2^-21
//     relative), accumulated in fp32;
//   * the scale term stays on the CUDA cores: t += d8' * float(sumi * sc) per sub-block, then
//     acc += d * t - dmin * m-term once per superblock.
// Layouts in shared memory:
//   * weights: the streaming kernel's stages, one row per pitch with pitch / 16 odd, so the eight
//     16-byte rows of an ldmatrix phase hit eight different bank groups;
//   * activations, per superblock: for each sub-block 8 columns x 32 qs bytes stored as words
//     (0,4,1,5,2,6,3,7), so lane (n = lane / 4, t = lane % 4) loads its B fragment (words t and
//     t + 4 of column n) with one 8-byte load, then the 8 columns' d8'; then dsum hi and lo as
//     [sub-block][column] floats; columns >= NCOLS are zero;
//   * work: (16-row tile, superblock) items of a chunk spread over the 8 warps, the partial tiles
//     summed across warps through shared memory in warp order (deterministic).
// ---------------------------------------------------------------------------------------------
constexpr uint32_t MMA_SUB_BYTES = 288;                   // 8 columns x 32 qs bytes + 8 x d8'
constexpr uint32_t MMA_SB_BYTES = 8 * MMA_SUB_BYTES + 512;  // + dsum hi / lo [8 sub-blocks][8 columns]
constexpr uint32_t MMA_MAX_CHUNK = 32;                    // rows per chunk: at most two 16-row tiles
constexpr uint32_t MMA_RED_BYTES = NW * 2 * 128 * 4;

__host__ __device__ inline uint32_t mma_pitch(uint32_t row_bytes) {
    const uint32_t p = (row_bytes + 15u) & ~15u;
    return ((p >> 4) & 1u) ? p : p + 16u;
}
__host__ __device__ inline uint32_t mma_stage_bytes(uint32_t chunk_rows, uint32_t row_bytes) {
    return (chunk_rows * mma_pitch(row_bytes) + 127u) & ~127u;
}
__host__ __device__ inline size_t mma_y_bytes(uint32_t nb32) { return ((size_t)(nb32 / 8) * MMA_SB_BYTES + 127) & ~(size_t)127; }


template <int NCOLS>
CFI_DEV YStage stage_y_mma(uint8_t* smem, const uint8_t* y0, size_t y_base, uint32_t stride_col_y, uint32_t nb32) {
    for (uint32_t idx = threadIdx.x; idx < 8u * nb32; idx += blockDim.x) {
        const uint32_t c = idx / nb32, b = idx - c * nb32, sb = b >> 3, j = b & 7;
        uint8_t* sbp = smem + (size_t)sb * MMA_SB_BYTES;
        uint8_t* g = sbp + j * MMA_SUB_BYTES;
        uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
        float d8 = 0.0f, ds = 0.0f;
        if (c < (uint32_t)NCOLS) {
            const uint32_t* w = reinterpret_cast<const uint32_t*>(y0 + (y_base + (size_t)c * stride_col_y + b) * Q8_1_BYTES);
            uint32_t q[9];
#pragma unroll
            for (int i = 0; i < 9; i++) q[i] = __ldg(w + i);
            int sum = 0;
#pragma unroll
            for (int i = 1; i < 9; i++) sum = dp4a(0x01010101, (int)q[i], sum);
            lo = make_uint4(q[1], q[5], q[2], q[6]);
            hi = make_uint4(q[3], q[7], q[4], q[8]);
            d8 = h2f_bits((uint16_t)(q[0] & 0xffffu));
            ds = d8 * (float)sum;
        }
        *reinterpret_cast<uint4*>(g + c * 32) = lo;
        *reinterpret_cast<uint4*>(g + c * 32 + 16) = hi;
        // odd sub-blocks are the high nibbles, whose MMA sums carry a factor 16
        reinterpret_cast<float*>(g + 256)[c] = (j & 1) ? d8 * 0.0625f : d8;
        const uint32_t dh = tf32_bits(ds);
        const uint32_t dl = tf32_bits(ds - __uint_as_float(dh));
        reinterpret_cast<uint32_t*>(sbp + 8 * MMA_SUB_BYTES)[j * 8 + c] = dh;
        reinterpret_cast<uint32_t*>(sbp + 8 * MMA_SUB_BYTES + 256)[j * 8 + c] = dl;
    }
    return YStage{smem_u32(smem), 0, 0, nb32};
}


// Rows [r0, r1) of one chunk (at most MMA_MAX_CHUNK), staged at sbase with row pitch rstride.
template <int NCOLS>
CFI_DEV void q4k_chunk_mma(uint32_t sbase, uint32_t rstride, uint32_t r0, uint32_t r1, const YStage& y, uint32_t red,
                           uint32_t tid, float* dplane, uint32_t stride_col_dst) {
    const uint32_t lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const uint32_t nrows = r1 - r0, ntile = (nrows + 15) / 16, nsb = y.nb32 / 8;
    float acc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
    // this lane's ldmatrix row within a tile (matrices: rows 0-7 / 8-15 x bytes 0-15 / 16-31)
    const uint32_t lrow = (lane & 7) + 8 * ((lane >> 3) & 1), lbyte = 16 * (lane >> 4);
    const uint32_t mshift = 8 * t;
    for (uint32_t item = warp; item < ntile * nsb; item += NW) {
        const uint32_t tile = item >= nsb ? 1u : 0u, sb = item - tile * nsb;
        const uint32_t arow = min(tile * 16 + lrow, nrows - 1);
        const uint32_t aaddr = sbase + arow * rstride + sb * Q4_K_BYTES + 16 + lbyte;
        float dx[2], dmin[2];
        uint32_t scw[2][2], am[4];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t row = min(tile * 16 + g + 8 * h, nrows - 1);
            const uint4 hd = lds128(sbase + row * rstride + sb * Q4_K_BYTES);
            dx[h] = h2f_bits((uint16_t)(hd.x & 0xffffu));
            dmin[h] = h2f_bits((uint16_t)(hd.x >> 16));
            // get_scale_min_k4 for all 8 sub-blocks, four bytes at a time
            scw[h][0] = hd.y & 0x3F3F3F3Fu;
            scw[h][1] = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
            const uint32_t m_lo = hd.z & 0x3F3F3F3Fu;
            const uint32_t m_hi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
            // tf32 A fragment of the min term: (row g + 8h, sub-block t) and (.., t + 4)
            am[h] = __float_as_uint((float)((m_lo >> mshift) & 0xffu));
            am[h + 2] = __float_as_uint((float)((m_hi >> mshift) & 0xffu));
        }
        const uint32_t ysb = y.ya + sb * MMA_SB_BYTES;
        float tm[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        {
            const uint32_t dsh = ysb + 8 * MMA_SUB_BYTES + (t * 8 + g) * 4;
            mma_tf32(am, lds32(dsh), lds32(dsh + 128), tm);
            mma_tf32(am, lds32(dsh + 256), lds32(dsh + 384), tm);
        }
        float tsc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int c = 0; c < 4; c++) {
            uint32_t raw[4];
            ldsm_x4(aaddr + 32 * c, raw);
#pragma unroll
            for (int hn = 0; hn < 2; hn++) {
                const int j = 2 * c + hn;  // sub-block of the superblock
                const uint32_t msk = hn ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
                const uint32_t a[4] = {raw[0] & msk, raw[1] & msk, raw[2] & msk, raw[3] & msk};
                const uint32_t gb = ysb + j * MMA_SUB_BYTES;
                const uint2 bw = lds64(gb + g * 32 + t * 8);
                int s4[4];
                mma_u8s8(a, bw.x, bw.y, s4);
                const uint2 dd = lds64(gb + 256 + t * 8);  // d8' of columns 2t, 2t + 1
                const float d80 = __uint_as_float(dd.x), d81 = __uint_as_float(dd.y);
                const uint32_t sh = 8u * (uint32_t)(j & 3);
                const int sc0 = (int)((scw[0][j >> 2] >> sh) & 0xffu), sc1 = (int)((scw[1][j >> 2] >> sh) & 0xffu);
                tsc[0] = __fmaf_rn(d80, (float)(s4[0] * sc0), tsc[0]);
                tsc[1] = __fmaf_rn(d81, (float)(s4[1] * sc0), tsc[1]);
                tsc[2] = __fmaf_rn(d80, (float)(s4[2] * sc1), tsc[2]);
                tsc[3] = __fmaf_rn(d81, (float)(s4[3] * sc1), tsc[3]);
            }
        }
        // the two tiles of a chunk are unrolled so acc stays in registers
#pragma unroll
        for (int T = 0; T < 2; T++)
            if (tile == (uint32_t)T)
#pragma unroll
                for (int i = 0; i < 4; i++)
                    acc[T][i] = __fmaf_rn(dx[i >> 1], tsc[i], __fmaf_rn(-dmin[i >> 1], tm[i], acc[T][i]));
    }
    // partial tiles of every warp, then the sum over warps in warp order
#pragma unroll
    for (int T = 0; T < 2; T++)
        if ((uint32_t)T < ntile)
#pragma unroll
            for (int i = 0; i < 4; i++)
                asm volatile("st.shared.f32 [%0], %1;" ::"r"(red + (((warp * 2 + T) * 4 + i) * 32 + lane) * 4), "f"(acc[T][i]));
    __syncthreads();
    for (uint32_t e = tid; e < ntile * 128; e += NW * 32) {
        const uint32_t T = e >> 7, rr = (e >> 3) & 15, cc = e & 7;
        if (cc >= (uint32_t)NCOLS || T * 16 + rr >= nrows) continue;
        const uint32_t i = ((rr >> 3) << 1) | (cc & 1), ln = 4 * (rr & 7) + (cc >> 1);
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) {
            float p;
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(p) : "r"(red + (((w * 2 + T) * 4 + i) * 32 + ln) * 4));
            v += p;
        }
        dplane[(size_t)cc * stride_col_dst + r0 + T * 16 + rr] = v;
    }
}

#define MMVQ_STREAM_PARAMS                                                                                           \
    const void *__restrict__ vx, const void *__restrict__ vy, const int32_t *__restrict__ ids, float *__restrict__ dst,     \
        uint32_t ncols_x, uint3 nchannels_y, uint32_t stride_row_x, uint32_t stride_col_y, uint32_t stride_col_dst,        \
        uint3 channel_ratio, uint32_t stride_channel_x, uint32_t stride_channel_y, uint32_t stride_channel_dst,            \
        uint3 sample_ratio, uint32_t stride_sample_x, uint32_t stride_sample_y, uint32_t stride_sample_dst, uint32_t nrows, \
        uint32_t chunk_rows, uint32_t nst
#define MMVQ_STREAM_ARGS                                                                                              \
    vx, vy, ids, dst, ncols_x, nchannels_y, stride_row_x, stride_col_y, stride_col_dst, channel_ratio, stride_channel_x, \
        stride_channel_y, stride_channel_dst, sample_ratio, stride_sample_x, stride_sample_y, stride_sample_dst, nrows,  \
        chunk_rows, nst

template <uint32_t TY, int NCOLS, bool FQ = false, bool DIRECT = false, bool MMA = false>
CFI_DEV void mmvq_stream_body(MMVQ_STREAM_PARAMS, const CfiFuseQ* fq = nullptr) {
    // nst bit 8 (CFI_CTX_CONST_WEIGHTS): the weights are not written by any kernel, so their
    // first stages are fetched before waiting on the previous kernel (programmatic dependent
    // launch), overlapping its tail; only the activations (and an ids table) wait
    const bool early = (nst & 0x100u) != 0 && !(NCOLS == 1 && ids != nullptr);
    // nst bit 9: the L2 hint for the CTA's whole row range is given in the early form too, so HBM
    // streams the rows ahead of the shared-memory stages (which then copy from L2)
    const bool hint_early = (nst & 0x200u) != 0;
    const uint32_t nst_word = nst;
    nst &= 0xffu;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[ST_MAX_STAGES];
    constexpr uint32_t BB = block_bytes<TY>();
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t nb = ncols_x / block_values<TY>();
    const uint32_t nb32 = ncols_x / 32;
    const uint32_t row_bytes = nb * BB;
    // the tensor-core kernel copies row by row at its bank-conflict-free pitch
    const bool dense = stride_row_x == nb && !MMA;
    const uint32_t rstride = MMA ? mma_pitch(row_bytes) : st_row_stride(row_bytes, dense);
    const uint32_t stage_bytes = MMA ? mma_stage_bytes(chunk_rows, row_bytes) : st_stage_bytes(chunk_rows, row_bytes, dense);
    const uint32_t channel_dst = blockIdx.y, sample_dst = blockIdx.z;
    const bool use_ids = NCOLS == 1 && ids != nullptr;
    const uint32_t sample_x = fastdiv(sample_dst, sample_ratio);
    const uint32_t rbeg = (uint32_t)((uint64_t)blockIdx.x * nrows / gridDim.x);
    const uint32_t rend = (uint32_t)((uint64_t)(blockIdx.x + 1) * nrows / gridDim.x);
    const uint32_t nchunks = (rend - rbeg + chunk_rows - 1) / chunk_rows;
    // a CTA that refills its stages runs the per-warp pipeline below, unless nst bit 10 asks for
    // the CTA-wide chunk loop (as a CTA whose chunks all fit its stages does)
    const bool warp_pipe = !MMA && (nst_word & 0x400u) == 0 && nchunks > nst;
    if constexpr (FQ) cluster_arrive_relaxed();  // completed in stage_y_q81

    // per-warp pipeline (every kernel but the tensor-core one, whose chunk ends in a cross-warp
    // sum): a stage's barrier completes on the filling warp's two arrivals (bulk bytes announced;
    // its ragged-end stores done) and the bulk bytes; done[s] counts the warps through the stage
    __shared__ uint32_t done[ST_MAX_STAGES];
    if (tid == 0) {
        for (uint32_t s = 0; s < nst; s++) {
            mbar_init(&full[s], warp_pipe ? 2 : 1);
            done[s] = 0;
        }
        fence_mbar_init();
        // L2 hint for this CTA's rows (the ids table may come from the previous kernel: skip)
        if (!use_ids && (!early || hint_early) && rend > rbeg) {
            const uint32_t channel_x = fastdiv(channel_dst, channel_ratio);
            const uint8_t* pl = static_cast<const uint8_t*>(vx) +
                                ((size_t)sample_x * stride_sample_x + (size_t)channel_x * stride_channel_x) * BB;
            uintptr_t a0 = (reinterpret_cast<uintptr_t>(pl + (size_t)rbeg * stride_row_x * BB) + 15) & ~(uintptr_t)15;
            const uintptr_t a1 = reinterpret_cast<uintptr_t>(pl + (size_t)(rend - 1) * stride_row_x * BB + row_bytes) & ~(uintptr_t)15;
            while (a0 < a1) {
                const uint32_t n = (uint32_t)min((uintptr_t)(1u << 20), a1 - a0);
                l2_prefetch(reinterpret_cast<const void*>(a0), n);
                a0 += n;
            }
        }
    }
    // operand addresses of this CTA's plane (an ids table is read only after the wait)
    size_t y_base = 0;
    uintptr_t plane = 0;
    float* dplane = nullptr;
    auto resolve = [&]() {
        const uint32_t channel_x = use_ids ? (uint32_t)ids[channel_dst] : fastdiv(channel_dst, channel_ratio);
        const uint32_t channel_y = use_ids ? fastmodulo(channel_dst, nchannels_y) : channel_dst;
        y_base = (size_t)sample_dst * stride_sample_y + (size_t)channel_y * stride_channel_y;
        plane = reinterpret_cast<uintptr_t>(vx) + ((size_t)sample_x * stride_sample_x + (size_t)channel_x * stride_channel_x) * BB;
        dplane = dst + (size_t)sample_dst * stride_sample_dst + (size_t)channel_dst * stride_channel_dst;
    };

    // copies one byte range [b0, b1) (2-byte aligned) to shared memory at st + (x - (b0 & ~15)):
    // the 16-byte-aligned interior by one bulk copy (issued by `issuer`), the ragged ends as
    // halfwords by threads base .. base + 15.  Returns the bulk byte count.
    auto range_bytes = [](uintptr_t b0, uintptr_t b1) -> uint32_t {
        const uintptr_t a0 = (b0 + 15) & ~(uintptr_t)15, a1 = b1 & ~(uintptr_t)15;
        return a1 > a0 ? (uint32_t)(a1 - a0) : 0u;
    };
    auto range_copy = [&](uint8_t* st, uintptr_t b0, uintptr_t b1, uint64_t* bar, bool issuer, uint32_t hw) {
        const uintptr_t base = b0 & ~(uintptr_t)15;
        uintptr_t a0 = (b0 + 15) & ~(uintptr_t)15, a1 = b1 & ~(uintptr_t)15;
        if (a1 <= a0) a0 = a1 = b1;
        if (issuer && a1 > a0) bulk_g2s(st + (a0 - base), reinterpret_cast<const void*>(a0), (uint32_t)(a1 - a0), bar);
        if (TY != T_Q4_K && hw < 16) {  // Q8_0, Q4_0, Q6_K rows are 2-byte aligned: at most 7 halfwords per end
            const uintptr_t src = hw < 8 ? b0 + 2 * hw : a1 + 2 * (hw - 8);
            if (hw < 8 ? src < a0 : src < b1)
                *reinterpret_cast<uint16_t*>(st + (src - base)) = __ldg(reinterpret_cast<const unsigned short*>(src));
        }
    };
    auto fill = [&](uint32_t ch, uint32_t s) {
        const uint32_t r0 = rbeg + ch * chunk_rows, r1 = min(r0 + chunk_rows, rend);
        uint8_t* st = smem + s * stage_bytes;
        if (dense) {
            const uintptr_t b0 = plane + (uintptr_t)r0 * nb * BB, b1 = plane + (uintptr_t)r1 * nb * BB;
            if (tid == 0) mbar_arrive_expect_tx(&full[s], range_bytes(b0, b1));
            range_copy(st, b0, b1, &full[s], tid == 0, tid);
        } else {
            if (tid == 0) {
                uint32_t tx = 0;
                for (uint32_t r = r0; r < r1; r++) {
                    const uintptr_t rs = plane + (uintptr_t)r * stride_row_x * BB;
                    tx += range_bytes(rs, rs + row_bytes);
                }
                mbar_arrive_expect_tx(&full[s], tx);
            }
            __syncthreads();
            for (uint32_t idx = tid; idx < (r1 - r0) * 16; idx += NW * 32) {
                const uint32_t k = idx / 16;
                const uintptr_t rs = plane + (uintptr_t)(r0 + k) * stride_row_x * BB;
                range_copy(st + k * rstride, rs, rs + row_bytes, &full[s], (idx & 15) == 0, idx & 15);
            }
        }
    };
    // the same fill by one whole warp (the per-warp pipeline): lane 0 announces the bytes and
    // issues the bulk copies, lanes store the ragged ends, then lane 0 arrives for them
    auto fill_w = [&](uint32_t ch, uint32_t s) {
        const uint32_t r0 = rbeg + ch * chunk_rows, r1 = min(r0 + chunk_rows, rend);
        uint8_t* st = smem + s * stage_bytes;
        if (dense) {
            const uintptr_t b0 = plane + (uintptr_t)r0 * nb * BB, b1 = plane + (uintptr_t)r1 * nb * BB;
            if (lane == 0) mbar_arrive_expect_tx(&full[s], range_bytes(b0, b1));
            range_copy(st, b0, b1, &full[s], lane == 0, lane);
        } else {
            if (lane == 0) {
                uint32_t tx = 0;
                for (uint32_t r = r0; r < r1; r++) {
                    const uintptr_t rs = plane + (uintptr_t)r * stride_row_x * BB;
                    tx += range_bytes(rs, rs + row_bytes);
                }
                mbar_arrive_expect_tx(&full[s], tx);
            }
            __syncwarp();
            for (uint32_t idx = lane; idx < (r1 - r0) * 16; idx += 32) {
                const uint32_t k = idx / 16;
                const uintptr_t rs = plane + (uintptr_t)(r0 + k) * stride_row_x * BB;
                range_copy(st + k * rstride, rs, rs + row_bytes, &full[s], (idx & 15) == 0, idx & 15);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
    };
    auto stage_act = [&](uint8_t* at) -> YStage {
        if constexpr (MMA)
            return stage_y_mma<NCOLS>(at, static_cast<const uint8_t*>(vy), y_base, stride_col_y, nb32);
        else if constexpr (FQ)
            return stage_y_q81<TY>(at, NCOLS, *fq, nb32);
        else
            return stage_y<TY>(at, NCOLS, static_cast<const uint8_t*>(vy), y_base, stride_col_y, nb32);
    };
    // the tensor-core kernel's cross-warp partials follow its activation stage
    const uint32_t red = MMA ? smem_u32(smem + nst * stage_bytes + mma_y_bytes(nb32)) : 0u;
    auto compute = [&](uint32_t sb, uint32_t r0, uint32_t r1, const YStage& y) {
        if constexpr (MMA)
            q4k_chunk_mma<NCOLS>(sb, rstride, r0, r1, y, red, tid, dplane, stride_col_dst);
        else if constexpr (TY == T_Q4_K)
            q4k_chunk<NCOLS>(sb, rstride, r0, r1, y, tid, dplane, stride_col_dst);
        else if constexpr (TY == T_Q6_K)
            q6k_chunk<NCOLS>(sb, rstride, dense, r0, r1, y, lane, warp, plane, stride_row_x, dplane, stride_col_dst);
        else if constexpr (TY == T_Q4_0)
            q40_chunk<NCOLS>(sb, rstride, dense, r0, r1, y, lane, warp, plane, stride_row_x, dplane, stride_col_dst);
        else
            q80_chunk<NCOLS>(sb, rstride, dense, r0, r1, y, lane, warp, plane, stride_row_x, dplane, stride_col_dst);
    };

    if constexpr (DIRECT) {
        // Direct fill (dense rows; the host sizes a chunk to at most DIRECT_U x 16 bytes per
        // thread): every thread loads its 16-byte pieces of the chunk's byte range into
        // registers with plain global loads -- all of them in flight at once, served from L2
        // after the prefetch above -- and stores them into the stage, two stages alternating,
        // so chunk k+1 is in flight while chunk k is computed.  Same stage layout as the bulk
        // copies: the range from its first 16-byte boundary, ragged ends as halfwords.
        uint4 reg[DIRECT_U];
        uint32_t hwv = 0;
        auto piece = [&](uint32_t ch, uintptr_t& b0, uintptr_t& b1, uintptr_t& a0, uintptr_t& a1) {
            const uint32_t r0 = rbeg + ch * chunk_rows, r1 = min(r0 + chunk_rows, rend);
            b0 = plane + (uintptr_t)r0 * row_bytes;
            b1 = plane + (uintptr_t)r1 * row_bytes;
            a0 = (b0 + 15) & ~(uintptr_t)15;
            a1 = b1 & ~(uintptr_t)15;
            if (a1 <= a0) a0 = a1 = b1;
        };
        auto load = [&](uint32_t ch) {
            uintptr_t b0, b1, a0, a1;
            piece(ch, b0, b1, a0, a1);
#pragma unroll
            for (int u = 0; u < DIRECT_U; u++) {
                const uintptr_t src = a0 + 16u * (tid + NW * 32u * u);
                reg[u] = src < a1 ? __ldg(reinterpret_cast<const uint4*>(src)) : make_uint4(0, 0, 0, 0);
            }
            if (TY != T_Q4_K && tid < 16) {  // 2-byte aligned rows: at most 7 halfwords per end
                const uintptr_t src = tid < 8 ? b0 + 2 * tid : a1 + 2 * (tid - 8);
                if (tid < 8 ? src < a0 : src < b1) hwv = __ldg(reinterpret_cast<const unsigned short*>(src));
            }
        };
        auto store = [&](uint32_t ch, uint8_t* st) {
            uintptr_t b0, b1, a0, a1;
            piece(ch, b0, b1, a0, a1);
            const uintptr_t base = b0 & ~(uintptr_t)15;
#pragma unroll
            for (int u = 0; u < DIRECT_U; u++) {
                const uintptr_t src = a0 + 16u * (tid + NW * 32u * u);
                if (src < a1) *reinterpret_cast<uint4*>(st + (src - base)) = reg[u];
            }
            if (TY != T_Q4_K && tid < 16) {
                const uintptr_t src = tid < 8 ? b0 + 2 * tid : a1 + 2 * (tid - 8);
                if (tid < 8 ? src < a0 : src < b1) *reinterpret_cast<uint16_t*>(st + (src - base)) = (uint16_t)hwv;
            }
        };
        if (early) {
            resolve();
            if (nchunks > 0) load(0);
        }
        pdl_launch_dependents();
        pdl_wait();
        if (!early) {
            resolve();
            if (nchunks > 0) load(0);
        }
        const YStage y = stage_act(smem + 2 * stage_bytes);
        for (uint32_t ch = 0; ch < nchunks; ch++) {
            uint8_t* st = smem + (ch & 1) * stage_bytes;
            store(ch, st);
            __syncthreads();
            if (ch + 1 < nchunks) load(ch + 1);
            const uint32_t r0 = rbeg + ch * chunk_rows;
            compute(smem_u32(st), r0, min(r0 + chunk_rows, rend), y);
        }
        return;
    } else {
    auto first_fills = [&]() {
        if (!warp_pipe) {
            for (uint32_t ch = 0; ch < nst && ch < nchunks; ch++) fill(ch, ch);
        } else if (warp == 0) {
            for (uint32_t ch = 0; ch < nst && ch < nchunks; ch++) fill_w(ch, ch);
        }
    };
    if (early) {
        __syncthreads();  // the barrier inits precede the fills' waits in other threads
        resolve();
        first_fills();
    }
    pdl_launch_dependents();
    pdl_wait();
    __syncthreads();
    if (!early) {
        resolve();
        first_fills();
    }
    const YStage y = stage_act(smem + nst * stage_bytes);
    __syncthreads();

    if (warp_pipe) {
        // each warp takes its rows of every chunk as soon as the chunk has landed; the last warp
        // through a stage refills it (no CTA-wide barrier between chunks)
        for (uint32_t ch = 0; ch < nchunks; ch++) {
            const uint32_t s = ch % nst;
            if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (ch / nst) & 1, &g_mmvq_abort))) {
                if (lane == 0) cfi_set_error(&g_mmvq_error, 0x4d560000u | ch);
                return;
            }
            const uint32_t r0 = rbeg + ch * chunk_rows, r1 = min(r0 + chunk_rows, rend);
            compute(smem_u32(smem + s * stage_bytes), r0, r1, y);
            __syncwarp();
            uint32_t prev = 0;
            if (lane == 0) prev = atomicAdd(&done[s], 1u);
            prev = __shfl_sync(0xffffffffu, prev, 0);
            if (prev == NW - 1) {
                // every warp has read the stage: reset its count (ordered before the next
                // chunk's readers by the fill's arrivals) and refill it
                if (lane == 0) done[s] = 0u;
                if (ch + nst < nchunks) fill_w(ch + nst, s);
            }
        }
        return;
    }

    for (uint32_t ch = 0; ch < nchunks; ch++) {
        const uint32_t s = ch % nst;
        const bool ok = __syncthreads_and(mbar_wait(&full[s], (ch / nst) & 1, &g_mmvq_abort));
        if (!ok) {
            if (tid == 0) cfi_set_error(&g_mmvq_error, 0x4d560000u | ch);
            return;
        }
        const uint32_t r0 = rbeg + ch * chunk_rows, r1 = min(r0 + chunk_rows, rend);
        compute(smem_u32(smem + s * stage_bytes), r0, r1, y);
        __syncthreads();
        if (ch + nst < nchunks) fill(ch + nst, s);
    }
    }
}

template <uint32_t TY, int NCOLS>
__global__ void __launch_bounds__(NW * 32) cfi_mmvq_stream(MMVQ_STREAM_PARAMS) {
    mmvq_stream_body<TY, NCOLS>(MMVQ_STREAM_ARGS);
}

// The tensor-core Q4_K GEMV (3..8 columns).
template <int NCOLS>
__global__ void __launch_bounds__(NW * 32) cfi_mmvq_mma(MMVQ_STREAM_PARAMS) {
    mmvq_stream_body<T_Q4_K, NCOLS, false, false, true>(MMVQ_STREAM_ARGS);
}

// The direct-fill GEMV (nst == 0 from the host): 4 CTAs per SM for one or two columns.
template <int NCOLS> constexpr int direct_min_ctas() { return NCOLS <= 2 ? 4 : 2; }
template <uint32_t TY, int NCOLS>
__global__ void __launch_bounds__(NW * 32, direct_min_ctas<NCOLS>()) cfi_mmvq_direct(MMVQ_STREAM_PARAMS) {
    mmvq_stream_body<TY, NCOLS, false, true>(MMVQ_STREAM_ARGS);
}

// GEMV that absorbed the quantize_q8_1 launched before it (single channel/sample plane), on the
// direct-fill and on the bulk-copy layout.
template <uint32_t TY, int NCOLS>
__global__ void __launch_bounds__(NW * 32, direct_min_ctas<NCOLS>()) cfi_mmvq_direct_q81(MMVQ_STREAM_PARAMS, const CfiFuseQ fq) {
    mmvq_stream_body<TY, NCOLS, true, true>(MMVQ_STREAM_ARGS, &fq);
}
template <uint32_t TY, int NCOLS>
__global__ void __launch_bounds__(NW * 32) cfi_mmvq_stream_q81(MMVQ_STREAM_PARAMS, const CfiFuseQ fq) {
    mmvq_stream_body<TY, NCOLS, true, false>(MMVQ_STREAM_ARGS, &fq);
}

// Q8_0 GEMV (one column) followed, in its last CTA to finish, by one fused decode step on the
// output (decode_epi.cuh).  Every CTA counts itself done after its rows are stored (fence, then
// the device counter); the last one runs the step over the whole output and resets the counter.
template <int EPI>
__global__ void __launch_bounds__(NW * 32) cfi_mmvq_epi(MMVQ_STREAM_PARAMS, const DecodeEpi e) {
    mmvq_stream_body<T_Q8_0, 1>(MMVQ_STREAM_ARGS);
    __shared__ int last;
    __syncthreads();
    __threadfence();
    if (threadIdx.x == 0) last = atomicAdd(e.counter, 1u) == gridDim.x * gridDim.y * gridDim.z - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    extern __shared__ __align__(128) uint8_t smem[];
    if (EPI == EPI_ADD_RMSNORM_Q81)
        epi_add_rmsnorm_q81(e.x, dst, e.w, e.q, e.n, e.eps, reinterpret_cast<float*>(smem));
    else if (EPI == EPI_SWIGLU_Q81)
        epi_swiglu_q81(dst, e.q, e.n, threadIdx.x >> 5, NW);
    else
        epi_qkv_rope_store(dst, e.bias, e.q_out, e.kc, e.vc, e.pos, e.nq, e.nkv, e.head_dim, e.n_ctx, e.theta_scale,
                           threadIdx.x, NW * 32);
    __syncthreads();
    if (threadIdx.x == 0) *e.counter = 0u;
}

template <uint32_t TY>
const void* pick(uint32_t ncols, bool stream) {
    switch (ncols) {
    case 1: return stream ? reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 1>) : reinterpret_cast<const void*>(&cfi_mmvq_rows<TY, 1>);
    case 2: return stream ? reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 2>) : reinterpret_cast<const void*>(&cfi_mmvq_rows<TY, 2>);
    case 3: return stream ? reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 3>) : reinterpret_cast<const void*>(&cfi_mmvq_rows<TY, 3>);
    case 4: return stream ? reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 4>) : reinterpret_cast<const void*>(&cfi_mmvq_rows<TY, 4>);
    case 5: return stream ? reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 5>) : reinterpret_cast<const void*>(&cfi_mmvq_rows<TY, 5>);
    case 6: return stream ? reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 6>) : reinterpret_cast<const void*>(&cfi_mmvq_rows<TY, 6>);
    case 7: return stream ? reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 7>) : reinterpret_cast<const void*>(&cfi_mmvq_rows<TY, 7>);
    case 8: return stream ? reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 8>) : reinterpret_cast<const void*>(&cfi_mmvq_rows<TY, 8>);
    default: return nullptr;
    }
}

template <uint32_t TY>
const void* pick_stream(uint32_t ncols) {
    switch (ncols) {
    case 1: return reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 1>);
    case 2: return reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 2>);
    case 3: return reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 3>);
    case 4: return reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 4>);
    case 5: return reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 5>);
    case 6: return reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 6>);
    case 7: return reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 7>);
    case 8: return reinterpret_cast<const void*>(&cfi_mmvq_stream<TY, 8>);
    default: return nullptr;
    }
}

template <uint32_t TY>
const void* pick_direct(uint32_t ncols) {
    switch (ncols) {
    case 1: return reinterpret_cast<const void*>(&cfi_mmvq_direct<TY, 1>);
    case 2: return reinterpret_cast<const void*>(&cfi_mmvq_direct<TY, 2>);
    case 3: return reinterpret_cast<const void*>(&cfi_mmvq_direct<TY, 3>);
    case 4: return reinterpret_cast<const void*>(&cfi_mmvq_direct<TY, 4>);
    case 5: return reinterpret_cast<const void*>(&cfi_mmvq_direct<TY, 5>);
    case 6: return reinterpret_cast<const void*>(&cfi_mmvq_direct<TY, 6>);
    case 7: return reinterpret_cast<const void*>(&cfi_mmvq_direct<TY, 7>);
    case 8: return reinterpret_cast<const void*>(&cfi_mmvq_direct<TY, 8>);
    default: return nullptr;
    }
}

// fused kernels exist for up to 4 columns (the router absorbs a quantize only there)
template <uint32_t TY>
const void* pick_q81(uint32_t ncols, bool direct) {
    switch (ncols) {
    case 1: return direct ? reinterpret_cast<const void*>(&cfi_mmvq_direct_q81<TY, 1>) : reinterpret_cast<const void*>(&cfi_mmvq_stream_q81<TY, 1>);
    case 2: return direct ? reinterpret_cast<const void*>(&cfi_mmvq_direct_q81<TY, 2>) : reinterpret_cast<const void*>(&cfi_mmvq_stream_q81<TY, 2>);
    case 3: return direct ? reinterpret_cast<const void*>(&cfi_mmvq_direct_q81<TY, 3>) : reinterpret_cast<const void*>(&cfi_mmvq_stream_q81<TY, 3>);
    case 4: return direct ? reinterpret_cast<const void*>(&cfi_mmvq_direct_q81<TY, 4>) : reinterpret_cast<const void*>(&cfi_mmvq_stream_q81<TY, 4>);
    default: return nullptr;
    }
}

}  // namespace

const void* cfi_native_mmvq_mma(uint32_t ty, uint32_t ncols) {
    if (ty != T_Q4_K) return nullptr;
    switch (ncols) {
    case 3: return reinterpret_cast<const void*>(&cfi_mmvq_mma<3>);
    case 4: return reinterpret_cast<const void*>(&cfi_mmvq_mma<4>);
    case 5: return reinterpret_cast<const void*>(&cfi_mmvq_mma<5>);
    case 6: return reinterpret_cast<const void*>(&cfi_mmvq_mma<6>);
    case 7: return reinterpret_cast<const void*>(&cfi_mmvq_mma<7>);
    case 8: return reinterpret_cast<const void*>(&cfi_mmvq_mma<8>);
    default: return nullptr;
    }
}

bool cfi_mmvq_mma_layout(uint32_t ncols_x, uint32_t nrows, uint32_t grid_x, uint32_t ctas_per_sm, uint32_t chunk_target,
                         uint32_t stage_budget, uint32_t max_stages, uint32_t* chunk_rows, uint32_t* nstages,
                         size_t* smem) {
    if (ncols_x == 0 || ncols_x % QK_K) return false;
    const uint32_t row_bytes = ncols_x / QK_K * Q4_K_BYTES;
    const uint32_t per_cta = (nrows + grid_x - 1) / grid_x;
    uint32_t c = std::min(std::min(std::max(1u, chunk_target), MMA_MAX_CHUNK), std::max(1u, per_cta));
    while (c > 1 && mma_stage_bytes(c, row_bytes) > stage_budget) c--;
    const uint32_t chunks = (per_cta + c - 1) / c;
    uint32_t nst = std::max(1u, std::min(std::min(max_stages, ST_MAX_STAGES), chunks));
    // the grid's CTAs per SM must fit side by side (228 KB of shared memory per SM, 1 KB of it
    // reserved per CTA)
    const size_t fixed = mma_y_bytes(ncols_x / 32) + MMA_RED_BYTES;
    const size_t cap = std::min((size_t)cfi_mmvq_max_smem_bytes(), (size_t)233472 / std::max(1u, ctas_per_sm) - 1024 - 128);
    // long rows: fewer stages, then shorter chunks, until the CTA fits
    while (nst > 1 && (size_t)nst * mma_stage_bytes(c, row_bytes) + fixed > cap) nst--;
    while (c > 1 && (size_t)nst * mma_stage_bytes(c, row_bytes) + fixed > cap) c--;
    *chunk_rows = c;
    *nstages = nst;
    *smem = (size_t)nst * mma_stage_bytes(c, row_bytes) + fixed;
    return *smem <= cap;
}

const void* cfi_native_mmvq_direct(uint32_t ty, uint32_t ncols) {
    if (ty == T_Q8_0) return pick_direct<T_Q8_0>(ncols);
    if (ty == T_Q4_K) return pick_direct<T_Q4_K>(ncols);
    if (ty == T_Q6_K) return pick_direct<T_Q6_K>(ncols);
    if (ty == T_Q4_0) return pick_direct<T_Q4_0>(ncols);
    return nullptr;
}

const void* cfi_native_mmvq_q81(uint32_t ty, uint32_t ncols, bool direct) {
    if (ty == T_Q8_0) return pick_q81<T_Q8_0>(ncols, direct);
    if (ty == T_Q4_K) return pick_q81<T_Q4_K>(ncols, direct);
    if (ty == T_Q6_K) return pick_q81<T_Q6_K>(ncols, direct);
    if (ty == T_Q4_0) return pick_q81<T_Q4_0>(ncols, direct);
    return nullptr;
}

// Q6_K and Q4_0 have the streaming kernel only (`stream` is ignored for them).
const void* cfi_native_mmvq(uint32_t ty, uint32_t ncols, bool stream) {
    if (ty == T_Q8_0) return pick<T_Q8_0>(ncols, stream);
    if (ty == T_Q4_K) return pick<T_Q4_K>(ncols, stream);
    if (ty == T_Q6_K) return pick_stream<T_Q6_K>(ncols);
    if (ty == T_Q4_0) return pick_stream<T_Q4_0>(ncols);
    return nullptr;
}

bool cfi_mmvq_stream_only(uint32_t ty) { return ty == T_Q6_K || ty == T_Q4_0; }

bool cfi_mmvq_streams(uint32_t ncols) { return ncols >= 1 && ncols <= 8; }

void cfi_mmvq_stream_layout(uint32_t ty, uint32_t ncols, uint32_t ncols_x, uint32_t nrows, uint32_t grid_x,
                            uint32_t stride_row_x, uint32_t chunk_target, uint32_t stage_budget, uint32_t max_stages,
                            uint32_t ctas_per_sm, uint32_t* chunk_rows, uint32_t* nstages, size_t* smem) {
    const uint32_t nb = ncols_x / block_values_of(ty);
    const uint32_t row_bytes = nb * block_bytes_of(ty);
    const bool dense = stride_row_x == nb;
    const uint32_t per_cta = (nrows + grid_x - 1) / grid_x;
    uint32_t c = std::min(std::max(1u, chunk_target), std::max(1u, per_cta));
    while (c > 1 && st_stage_bytes(c, row_bytes, dense) > stage_budget) c--;
    const uint32_t chunks = (per_cta + c - 1) / c;
    uint32_t nst = std::max(1u, std::min(std::min(max_stages, ST_MAX_STAGES), chunks));
    // the grid holds ctas_per_sm CTAs per SM: each fits its share of the SM's 228 KB (1 KB of it
    // reserved per CTA, and the kernel's static words), so the grid runs in one wave
    const size_t ys = ((size_t)ncols * (ncols_x / 32) * 40 + 127) & ~(size_t)127;
    const size_t cap = std::min((size_t)cfi_mmvq_max_smem_bytes(), (size_t)233472 / std::max(1u, ctas_per_sm) - 1024 - 128);
    // long rows: fewer stages, then shorter chunks, until the CTA fits
    while (nst > 1 && (size_t)nst * st_stage_bytes(c, row_bytes, dense) + ys > cap) nst--;
    while (c > 1 && (size_t)nst * st_stage_bytes(c, row_bytes, dense) + ys > cap) c--;
    *chunk_rows = c;
    *nstages = nst;
    *smem = (size_t)nst * st_stage_bytes(c, row_bytes, dense) + ys;
}

bool cfi_mmvq_direct_layout(uint32_t ty, uint32_t ncols, uint32_t ncols_x, uint32_t nrows, uint32_t grid_x,
                            uint32_t stride_row_x, uint32_t* chunk_rows, size_t* smem) {
    const uint32_t nb = ncols_x / block_values_of(ty);
    const uint32_t row_bytes = nb * block_bytes_of(ty);
    const uint32_t cap = (uint32_t)DIRECT_U * 16u * (uint32_t)(NW * 32);
    if (stride_row_x != nb || row_bytes == 0 || row_bytes > cap) return false;
    const uint32_t per_cta = (nrows + grid_x - 1) / grid_x;
    const uint32_t c = std::max(1u, std::min(per_cta, cap / row_bytes));
    *chunk_rows = c;
    const size_t ys = ((size_t)ncols * (ncols_x / 32) * 40 + 127) & ~(size_t)127;
    *smem = 2 * (size_t)st_stage_bytes(c, row_bytes, true) + ys;
    return true;
}

size_t cfi_mmvq_smem_bytes(uint32_t ty, uint32_t ncols, uint32_t ncols_x) {
    const size_t ys = ((size_t)ncols * (ncols_x / 32) * 40 + 127) & ~(size_t)127;
    const int r = ty == T_Q4_K ? (ncols == 1 ? 2 : 1) : (ncols <= 2 ? 2 : 1);
    const size_t wb = ty == T_Q8_0 ? (size_t)NW * r * WBUF_ROW : 0;
    return ys + wb;
}

int cfi_mmvq_max_smem_bytes() { return 200 * 1024; }

// Reads and clears the error word of the GEMV's bounded waits (folded into cfi_device_error).
unsigned int cfi_mmvq_error_take() {
    unsigned int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_mmvq_error, sizeof v) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaMemcpyToSymbol(g_mmvq_error, &z, sizeof z);
    return v;
}

// ---- GEMV + fused decode step (include/cfi_glue.h) ----

namespace {
template <int EPI>
int launch_epi(const void* w, const void* xq, float* y, int rows, int k, DecodeEpi e, size_t epi_smem, void* stream) {
    if (rows <= 0 || k <= 0 || k % 32 || (reinterpret_cast<uintptr_t>(w) & 1) || (reinterpret_cast<uintptr_t>(xq) & 3))
        return (int)cudaErrorInvalidValue;
    CfiGlueSlot sl;  // the calling stream's counters
    const int rc = cfi_glue_slot(static_cast<cudaStream_t>(stream), &sl);
    if (rc) return rc;
    e.counter = sl.epi_count + EPI;
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t nb = (uint32_t)k / 32, grid = std::max(1u, std::min((uint32_t)rows, 2u * (uint32_t)sms));
    uint32_t chunk = 0, nst = 0;
    size_t smem = 0;
    cfi_mmvq_stream_layout(T_Q8_0, 1, (uint32_t)k, (uint32_t)rows, grid, nb, 32, 48 * 1024, 3, 2, &chunk, &nst, &smem);
    smem = std::max(smem, epi_smem);
    // the largest dynamic shared memory set so far for this kernel, per device
    static std::mutex attr_mu;
    static size_t attr_set[CFI_MAX_DEVICES] = {};
    if (smem > 48 * 1024) {
        const int d = cfi_device_index();
        std::lock_guard<std::mutex> lk(attr_mu);
        if (d < 0 || attr_set[d] < smem) {
            if (cudaFuncSetAttribute(cfi_mmvq_epi<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
                return (int)cudaErrorInvalidValue;
            if (d >= 0) attr_set[d] = smem;
        }
    }
    const uint3 none = make_uint3(0, 0, 0), fd1 = make_uint3(1, 0, 1);  // fastdiv triple of 1 (ggml's)
    const char* ep = getenv("CFI_PDL");
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3(grid, 1, 1);
    c.blockDim = dim3(NW * 32, 1, 1);
    c.dynamicSmemBytes = smem;
    c.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = at;
    c.numAttrs = (ep && strcmp(ep, "0") == 0) ? 0 : 1;
    const uint32_t r = (uint32_t)rows;
    return (int)cudaLaunchKernelEx(&c, cfi_mmvq_epi<EPI>, w, xq, (const int32_t*)nullptr, y, (uint32_t)k, none, nb, nb, r,
                                   fd1, r * nb, nb, r, fd1, r * nb, nb, r, r, chunk, nst, e);
}
}  // namespace

extern "C" int cfi_fused_mmvq_add_rmsnorm_q8_1(const void* w, const void* xq, float* y, int rows, int k, float* x,
                                               const float* norm_w, void* out_q8_1, float eps, void* stream) {
    if (rows % 32 || rows > 8192) return (int)cudaErrorInvalidValue;
    DecodeEpi e = {};
    e.x = x;
    e.w = norm_w;
    e.q = static_cast<uint8_t*>(out_q8_1);
    e.n = rows;
    e.eps = eps;
    return launch_epi<EPI_ADD_RMSNORM_Q81>(w, xq, y, rows, k, e, (size_t)rows * 4, stream);
}

extern "C" int cfi_fused_mmvq_swiglu_q8_1(const void* w, const void* xq, float* y, int rows, int k, void* out_q8_1,
                                          void* stream) {
    if (rows % 64) return (int)cudaErrorInvalidValue;
    DecodeEpi e = {};
    e.q = static_cast<uint8_t*>(out_q8_1);
    e.n = rows / 2;
    return launch_epi<EPI_SWIGLU_Q81>(w, xq, y, rows, k, e, 0, stream);
}

extern "C" int cfi_fused_mmvq_qkv_rope_store(const void* w, const void* xq, float* y, int k, const float* bias,
                                             float* q_out, void* kc, void* vc, const int32_t* pos, int nq, int nkv,
                                             int head_dim, int n_ctx, float theta, void* stream) {
    if (head_dim <= 0 || head_dim % 2 || nq % head_dim || nkv % head_dim) return (int)cudaErrorInvalidValue;
    DecodeEpi e = {};
    e.bias = bias;
    e.q_out = q_out;
    e.kc = static_cast<__half*>(kc);
    e.vc = static_cast<__half*>(vc);
    e.pos = pos;
    e.nq = nq;
    e.nkv = nkv;
    e.head_dim = head_dim;
    e.n_ctx = n_ctx;
    e.theta_scale = powf(theta, -2.0f / (float)head_dim);
    return launch_epi<EPI_QKV_ROPE_STORE>(w, xq, y, nq + 2 * nkv, k, e, 0, stream);
}
