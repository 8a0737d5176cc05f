// k_mmvq.cu -- decode GEMV y = W x for quantized W (sm_100a), the native mul_mat_vec_q.
//
// Parameter list: ggml-cuda's mul_mat_vec_q<type, ncols_dst> (x, y, ids, dst, u32 ncols_x, uint3
// nchannels_y, u32 stride_row_x, stride_col_y, stride_col_dst, uint3 channel_ratio, u32
// stride_channel_x/y/dst, uint3 sample_ratio, u32 stride_sample_x/y/dst; cuda-for-intel
// src/subst/mod.rs:214-218) plus one trailing u32 `nrows` appended by the router, as the
// reference's decode-fast variant does (src/subst/mod.rs:529-536).
//
// Work decomposition (B200): grid (row tiles, channels, samples), 8 warps per CTA.  Each CTA first
// stages the q8_1 activation blocks of its channel/sample into shared memory transposed
// (word-major, so lane b reading word i of block b is bank-conflict free), then every warp owns
// one weight row at a time:
//   * Q8_0 (34-byte blocks, 2-byte aligned): the warp copies 32 blocks (1088 B) of its row into a
//     private shared buffer with 16-byte coalesced loads (head/tail halfwords separately, so no
//     byte outside the row is touched), then lane l takes block l of the chunk;
//   * Q4_K (144-byte superblocks, 16-byte aligned): lane l takes sub-block l%8 of superblock l/8
//     (+4 per step) straight from global memory with 16-byte loads.
// This is the lane assignment of the reference's whole-group decode-fast model with one warp per
// row and one accumulator (src/subst/refs.rs:435-497, `wide`), and every per-lane float operation
// is written with explicit-rounding intrinsics in the reference's order (refs.rs:386-433), so each
// output column equals cfo_mmvq_fast(warps=1, unroll=1, wide) of that column bit for bit; the
// integer block dot products are exact dp4a sums.
#include "cfi_common.cuh"
#include "cfi_kernels.h"

namespace {

constexpr int WBUF_BYTES = 1120;  // 1088-byte chunk + alignment slack + funnel read-ahead

template <uint32_t TY> struct YStage {
    static constexpr int WORDS = (TY == T_Q4_K) ? 10 : 9;  // qs[8], d, (sum of quants)
};

CFI_DEV uint32_t byte_of(uint4 h, int k) {
    uint32_t w = k < 4 ? h.y : (k < 8 ? h.z : h.w);
    return (w >> (8 * (k & 3))) & 0xffu;
}

// ggml get_scale_min_k4 over the 12 scale bytes held in h.y, h.z, h.w.
CFI_DEV void scale_min_k4(int j, uint4 h, int& sc, int& m) {
    if (j < 4) {
        sc = byte_of(h, j) & 63;
        m = byte_of(h, j + 4) & 63;
    } else {
        sc = (byte_of(h, j + 4) & 0xF) | ((byte_of(h, j - 4) >> 6) << 4);
        m = (byte_of(h, j + 4) >> 4) | ((byte_of(h, j) >> 6) << 4);
    }
}

template <uint32_t TY, int NCOLS>
__global__ void __launch_bounds__(CFI_MMVQ_THREADS)
    cfi_mmvq(const void* __restrict__ vx, const void* __restrict__ vy, const int32_t* __restrict__ ids,
             float* __restrict__ dst, uint32_t ncols_x, uint3 nchannels_y, uint32_t stride_row_x,
             uint32_t stride_col_y, uint32_t stride_col_dst, uint3 channel_ratio, uint32_t stride_channel_x,
             uint32_t stride_channel_y, uint32_t stride_channel_dst, uint3 sample_ratio, uint32_t stride_sample_x,
             uint32_t stride_sample_y, uint32_t stride_sample_dst, uint32_t nrows) {
    extern __shared__ __align__(16) uint8_t smem[];
    const uint32_t nb32 = ncols_x / 32;
    uint32_t* ys = reinterpret_cast<uint32_t*>(smem);        // [NCOLS][8][nb32]
    float* yd = reinterpret_cast<float*>(ys + NCOLS * 8 * nb32);  // [NCOLS][nb32]
    int* ysum = reinterpret_cast<int*>(yd + NCOLS * nb32);     // [NCOLS][nb32] (Q4_K)
    const size_t stage_bytes = (size_t)NCOLS * nb32 * YStage<TY>::WORDS * 4;
    uint8_t* wbuf_all = smem + ((stage_bytes + 15) & ~(size_t)15);

    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t channel_dst = blockIdx.y, sample_dst = blockIdx.z;
    const bool use_ids = NCOLS == 1 && ids != nullptr;
    const uint32_t channel_x = use_ids ? (uint32_t)ids[channel_dst] : fastdiv(channel_dst, channel_ratio);
    const uint32_t channel_y = use_ids ? fastmodulo(channel_dst, nchannels_y) : channel_dst;
    const uint32_t sample_x = fastdiv(sample_dst, sample_ratio);
    const size_t y_base = (size_t)sample_dst * stride_sample_y + (size_t)channel_y * stride_channel_y;

    // ---- stage the activation blocks (word-major) ----
    const uint8_t* yb0 = static_cast<const uint8_t*>(vy);
    for (uint32_t idx = tid; idx < NCOLS * nb32; idx += CFI_MMVQ_THREADS) {
        const uint32_t c = idx / nb32, b = idx - c * nb32;
        const uint32_t* w = reinterpret_cast<const uint32_t*>(yb0 + (y_base + (size_t)c * stride_col_y + b) * Q8_1_BYTES);
        const uint32_t ds = __ldg(w);
        int s = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t q = __ldg(w + 1 + i);
            ys[(c * 8 + i) * nb32 + b] = q;
            if (TY == T_Q4_K) s = dp4a(0x01010101, (int)q, s);
        }
        yd[c * nb32 + b] = h2f_bits((uint16_t)(ds & 0xffffu));
        if (TY == T_Q4_K) ysum[c * nb32 + b] = s;
    }
    __syncthreads();

    constexpr uint32_t BB = TY == T_Q4_K ? Q4_K_BYTES : Q8_0_BYTES;
    const uint32_t nb = TY == T_Q4_K ? ncols_x / QK_K : ncols_x / QK8_0;  // x blocks per row
    const size_t x_off = (size_t)sample_x * stride_sample_x + (size_t)channel_x * stride_channel_x;
    const size_t dst_base = (size_t)sample_dst * stride_sample_dst + (size_t)channel_dst * stride_channel_dst;
    uint8_t* wbuf = wbuf_all + warp * WBUF_BYTES;

    for (uint32_t row = blockIdx.x * CFI_MMVQ_WARPS + warp; row < nrows; row += gridDim.x * CFI_MMVQ_WARPS) {
        const uint8_t* xrow = static_cast<const uint8_t*>(vx) + (x_off + (size_t)row * stride_row_x) * BB;
        float acc[NCOLS];
#pragma unroll
        for (int c = 0; c < NCOLS; c++) acc[c] = 0.0f;

        if constexpr (TY == T_Q8_0) {
            for (uint32_t b0 = 0; b0 < nb; b0 += 32) {
                const uint32_t n = min(32u, nb - b0);
                const uintptr_t cs = reinterpret_cast<uintptr_t>(xrow) + (uintptr_t)b0 * Q8_0_BYTES;
                const uintptr_t ce = cs + (uintptr_t)n * Q8_0_BYTES;
                const uintptr_t base = cs & ~(uintptr_t)15;
                const uintptr_t a0 = (cs + 15) & ~(uintptr_t)15, a1 = ce & ~(uintptr_t)15;
                const uint32_t nvec = (uint32_t)((a1 - a0) >> 4);
                for (uint32_t j = lane; j < nvec; j += 32) {
                    const uint4 v = __ldg(reinterpret_cast<const uint4*>(a0) + j);
                    *reinterpret_cast<uint4*>(wbuf + (a0 - base) + 16 * j) = v;
                }
                const uint32_t nhead = (uint32_t)((a0 - cs) >> 1), ntail = (uint32_t)((ce - a1) >> 1);
                if (lane < nhead) {
                    const uint16_t h = __ldg(reinterpret_cast<const unsigned short*>(cs) + lane);
                    reinterpret_cast<uint16_t*>(wbuf + (cs - base))[lane] = h;
                } else if (lane >= 8 && lane - 8 < ntail) {
                    const uint16_t h = __ldg(reinterpret_cast<const unsigned short*>(a1) + (lane - 8));
                    reinterpret_cast<uint16_t*>(wbuf + (a1 - base))[lane - 8] = h;
                }
                __syncwarp();
                if (lane < n) {
                    const uint32_t o = (uint32_t)(cs - base) + lane * Q8_0_BYTES;
                    const float dx = h2f_bits(reinterpret_cast<const uint16_t*>(wbuf)[o >> 1]);
                    const uint32_t qo = o + 2, qa = qo & ~3u, sh = (qo & 3u) * 8;
                    const uint32_t* W = reinterpret_cast<const uint32_t*>(wbuf) + (qa >> 2);
                    int wq[8];
                    uint32_t prev = W[0];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const uint32_t nxt = W[i + 1];
                        wq[i] = (int)__funnelshift_r(prev, nxt, sh);
                        prev = nxt;
                    }
                    const uint32_t b = b0 + lane;
#pragma unroll
                    for (int c = 0; c < NCOLS; c++) {
                        int sumi = 0;
#pragma unroll
                        for (int i = 0; i < 8; i++) sumi = dp4a(wq[i], (int)ys[(c * 8 + i) * nb32 + b], sumi);
                        acc[c] = __fmaf_rn(__fmul_rn(dx, yd[c * nb32 + b]), (float)sumi, acc[c]);
                    }
                }
                __syncwarp();
            }
        } else {  // Q4_K
            const int g = (int)(lane & 7);
            for (uint32_t sb = lane >> 3; sb < nb; sb += 4) {
                const uint4* blk = reinterpret_cast<const uint4*>(xrow + (size_t)sb * Q4_K_BYTES);
                const uint4 h = __ldg(blk);
                const uint4 q0 = __ldg(blk + 1 + 2 * (g >> 1));
                const uint4 q1 = __ldg(blk + 2 + 2 * (g >> 1));
                const float dx = h2f_bits((uint16_t)(h.x & 0xffffu));
                const float dmin = h2f_bits((uint16_t)(h.x >> 16));
                int sc, m;
                scale_min_k4(g, h, sc, m);
                const uint32_t nsh = 4 * (g & 1);
                const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                int v[8];
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = (int)((qw[i] >> nsh) & 0x0F0F0F0Fu);
                const uint32_t yb = sb * 8 + g;
#pragma unroll
                for (int c = 0; c < NCOLS; c++) {
                    int sumi = 0;
#pragma unroll
                    for (int i = 0; i < 8; i++) sumi = dp4a(v[i], (int)ys[(c * 8 + i) * nb32 + yb], sumi);
                    const float d8 = yd[c * nb32 + yb];
                    const float a = __fmul_rn(d8, (float)(sumi * sc));
                    const float bm = __fmul_rn(d8, (float)(ysum[c * nb32 + yb] * m));
                    acc[c] = __fadd_rn(acc[c], __fsub_rn(__fmul_rn(dx, a), __fmul_rn(dmin, bm)));
                }
            }
        }
#pragma unroll
        for (int c = 0; c < NCOLS; c++) {
            const float v = warp_sum(acc[c]);
            if (lane == 0) dst[dst_base + (size_t)c * stride_col_dst + row] = v;
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
    const size_t words = ty == T_Q4_K ? YStage<T_Q4_K>::WORDS : YStage<T_Q8_0>::WORDS;
    const size_t stage = (size_t)ncols * (ncols_x / 32) * words * 4;
    const size_t wbuf = ty == T_Q8_0 ? (size_t)CFI_MMVQ_WARPS * WBUF_BYTES : 0;
    return ((stage + 15) & ~(size_t)15) + wbuf;
}

int cfi_mmvq_max_smem_bytes() { return 200 * 1024; }
