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

namespace {

using namespace sm100;

constexpr int NW = CFI_MMVQ_WARPS;   // warps per CTA
constexpr int WBUF_ROW = 1120;       // Q8_0: one 32-block chunk of a row + alignment slack + read-ahead

template <uint32_t TY> __host__ __device__ constexpr uint32_t block_bytes() { return TY == T_Q4_K ? Q4_K_BYTES : Q8_0_BYTES; }
template <uint32_t TY, int NCOLS> __host__ __device__ constexpr int rows_per_warp() {
    return TY == T_Q4_K ? (NCOLS == 1 ? 2 : 1) : (NCOLS <= 2 ? 2 : 1);
}

CFI_DEV uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
CFI_DEV uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
CFI_DEV uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
CFI_DEV uint32_t lds16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
CFI_DEV void l2_prefetch(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Activation stage: ya[c][b] = qs words 0..3, yb[c][b] = qs words 4..7, ym[c][b] = {d (fp32
// bits), sum of the 32 int8 quants}; 40 bytes per block and column.
struct YStage {
    uint32_t ya, yb, ym;  // shared-space byte addresses
    uint32_t nb32;
};

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
        int s = 0;
#pragma unroll
        for (int i = 1; i < 9; i++) s = dp4a(0x01010101, (int)q[i], s);
        ya[idx] = make_uint4(q[1], q[2], q[3], q[4]);
        yb[idx] = make_uint4(q[5], q[6], q[7], q[8]);
        ym[idx] = make_uint2(__float_as_uint(h2f_bits((uint16_t)(q[0] & 0xffffu))), (uint32_t)s);
    }
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
    cfi_mmvq(const void* __restrict__ vx, const void* __restrict__ vy, const int32_t* __restrict__ ids,
             float* __restrict__ dst, uint32_t ncols_x, uint3 nchannels_y, uint32_t stride_row_x,
             uint32_t stride_col_y, uint32_t stride_col_dst, uint3 channel_ratio, uint32_t stride_channel_x,
             uint32_t stride_channel_y, uint32_t stride_channel_dst, uint3 sample_ratio, uint32_t stride_sample_x,
             uint32_t stride_sample_y, uint32_t stride_sample_dst, uint32_t nrows) {
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

template <uint32_t TY>
const void* pick(uint32_t ncols) {
    switch (ncols) {
    case 1: return reinterpret_cast<const void*>(&cfi_mmvq<TY, 1>);
    case 2: return reinterpret_cast<const void*>(&cfi_mmvq<TY, 2>);
    case 3: return reinterpret_cast<const void*>(&cfi_mmvq<TY, 3>);
    case 4: return reinterpret_cast<const void*>(&cfi_mmvq<TY, 4>);
    case 5: return reinterpret_cast<const void*>(&cfi_mmvq<TY, 5>);
    case 6: return reinterpret_cast<const void*>(&cfi_mmvq<TY, 6>);
    case 7: return reinterpret_cast<const void*>(&cfi_mmvq<TY, 7>);
    case 8: return reinterpret_cast<const void*>(&cfi_mmvq<TY, 8>);
    default: return nullptr;
    }
}

}  // namespace

const void* cfi_native_mmvq(uint32_t ty, uint32_t ncols) {
    if (ty == T_Q8_0) return pick<T_Q8_0>(ncols);
    if (ty == T_Q4_K) return pick<T_Q4_K>(ncols);
    return nullptr;
}

size_t cfi_mmvq_smem_bytes(uint32_t ty, uint32_t ncols, uint32_t ncols_x) {
    const size_t ys = ((size_t)ncols * (ncols_x / 32) * 40 + 127) & ~(size_t)127;
    const int r = ty == T_Q4_K ? (ncols == 1 ? 2 : 1) : (ncols <= 2 ? 2 : 1);
    const size_t wb = ty == T_Q8_0 ? (size_t)NW * r * WBUF_ROW : 0;
    return ys + wb;
}

int cfi_mmvq_max_smem_bytes() { return 200 * 1024; }
