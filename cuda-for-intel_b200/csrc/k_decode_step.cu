// k_decode_step.cu -- one whole Q8_0 decode token step (Qwen2-architecture model) in a single
// persistent, cooperative launch: the same op sequence as the fused glue chain of the decode
// driver (get_rows, add_rmsnorm_q8_1, QKV GEMV, qkv_rope_store, split attention, O GEMV,
// add_rmsnorm_q8_1, gate/up GEMV, swiglu_q8_1, down GEMV, ..., the head GEMV and the greedy
// argmax), with grid-wide barriers between the phases instead of kernel boundaries.
//
// Every phase computes exactly what the standalone kernel it replaces computes:
//   * the GEMVs follow the decode-fast model of mul_mat_vec_q<Q8_0, 1> (one warp per row, lane l
//     the 32-value blocks l, l + 32, ..., acc = fma(d_w * d_x, float(int8 dot), acc), the xor
//     butterfly 16..1), so each output equals the native GEMV's bit for bit;
//   * add_rmsnorm_q8_1, qkv_rope_store and swiglu_q8_1 call the same block-level device functions
//     as their kernels (decode_epi.cuh); the residual stream x lives in every CTA's shared memory
//     (each CTA applies the same operations to the same values, so the copies stay identical) and
//     each CTA quantizes its own copy of the normalised activations, so these steps need no
//     barrier;
//   * the attention splits over the same position ranges as cfi_fused_attention_q8_1 and
//     combines them in split order in the last CTA of each head.
// Values another CTA wrote during the launch are read through L2 (ld.global.cg); the weights,
// written by nothing, through the read-only path, and each CTA asks L2 for the rows of its next
// GEMV before it waits at the barrier in front of that GEMV.  Every barrier wait is bounded by
// %globaltimer: a CTA that gives up records an error code and raises the launch's abort flag, and
// every CTA then leaves at its next barrier.
#include "../../include/cfi_glue.h"
#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "decode_epi.cuh"
#include "sm100_ptx.cuh"

#include <math.h>
#include <string.h>

namespace {

constexpr int DS_THREADS = 256, DS_WARPS = DS_THREADS / 32;
constexpr int DS_MAX_HIDDEN = 1536, DS_MAX_FFN_BLOCKS = 384;  // the q8_1 stage: 12288 values
constexpr int DS_ATT_CHUNK = 128;                             // as cfi_fused_attention_q8_1

__device__ unsigned int g_ds_error;

struct DsArgs {
    CfiDecodeStep m;
    const CfiDecodeLayer* layers;  // device copy of the layer table
    unsigned int* sync;            // [0]: barrier count, [1]: abort flag (zeroed before the launch)
    float* att_part;
    unsigned int* att_count;
    float* amax_val;
    int* amax_idx;
    unsigned int* amax_count;
    int att_nsplit, att_chunk;
    float theta_scale, scale;
};

CFI_DEV unsigned int ld_acquire(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Barrier `k` (1, 2, ...) of the launch over all CTAs.  False when the launch is aborting.
CFI_DEV bool grid_sync(const DsArgs& a, unsigned int k) {
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile unsigned int* abort = a.sync + 1;
        // arrive: a release reduction (this CTA's writes, ordered before it by the CTA barrier
        // above, become visible to whoever acquires the count); wait: acquire loads
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.sync) : "memory");
        const unsigned int target = k * gridDim.x;
        if (ld_acquire(a.sync) < target) {
            const uint64_t t0 = sm100::globaltimer();
            for (uint32_t it = 1; ld_acquire(a.sync) < target; it++) {
                if ((it & 63) == 0) {
                    if (*abort) break;
                    if (sm100::globaltimer() - t0 > sm100::WAIT_LIMIT_NS) {
                        atomicCAS(&g_ds_error, 0u, 0xd5000000u | (k & 0xffffu));
                        *abort = 1u;
                        break;
                    }
                }
            }
        }
    }
    __syncthreads();
    return *reinterpret_cast<volatile unsigned int*>(a.sync + 1) == 0u;
}

CFI_DEV void l2_prefetch_range(const void* p, size_t bytes) {
    uintptr_t a0 = (reinterpret_cast<uintptr_t>(p) + 15) & ~(uintptr_t)15;
    const uintptr_t a1 = (reinterpret_cast<uintptr_t>(p) + bytes) & ~(uintptr_t)15;
    while (a0 < a1) {
        const uint32_t n = (uint32_t)min((uintptr_t)(1u << 20), a1 - a0);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a0), "r"(n) : "memory");
        a0 += n;
    }
}

// rows [r0, r1) of the CTA in a GEMV of `rows` rows
CFI_DEV void cta_rows(uint32_t rows, uint32_t& r0, uint32_t& r1) {
    r0 = (uint32_t)((uint64_t)blockIdx.x * rows / gridDim.x);
    r1 = (uint32_t)((uint64_t)(blockIdx.x + 1) * rows / gridDim.x);
}

CFI_DEV void prefetch_rows(const void* w, uint32_t rows, uint32_t k) {
    uint32_t r0, r1;
    cta_rows(rows, r0, r1);
    if (threadIdx.x == 0 && r1 > r0)
        l2_prefetch_range(static_cast<const uint8_t*>(w) + (size_t)r0 * (k / 32) * Q8_0_BYTES,
                          (size_t)(r1 - r0) * (k / 32) * Q8_0_BYTES);
}

// The 32 int8 quants of Q8_0 block b of a row (34-byte blocks, even block count per row) as 8
// words, and its d: nine aligned 4-byte loads (an even block starts 4-byte aligned and its last
// word reaches 2 bytes into the next block; an odd one starts 2 bytes into its first word).
CFI_DEV void q80_block(const uint8_t* row, uint32_t b, int (&w)[8], float& d) {
    const uint8_t* blk = row + (size_t)b * Q8_0_BYTES;
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(blk) & ~(uintptr_t)3);
    uint32_t v[9];
#pragma unroll
    for (int i = 0; i < 9; i++) v[i] = __ldg(wp + i);
    if ((b & 1) == 0) {
        d = h2f_bits((uint16_t)(v[0] & 0xffffu));
#pragma unroll
        for (int i = 0; i < 8; i++) w[i] = (int)__funnelshift_r(v[i], v[i + 1], 16);
    } else {
        d = h2f_bits((uint16_t)(v[0] >> 16));
#pragma unroll
        for (int i = 0; i < 8; i++) w[i] = (int)v[i + 1];
    }
}

CFI_DEV int dot8q(const int (&w)[8], const uint32_t* xq) {
    int s0 = __dp4a(w[0], (int)xq[0], 0), s1 = __dp4a(w[1], (int)xq[1], 0);
    s0 = __dp4a(w[2], (int)xq[2], s0);
    s1 = __dp4a(w[3], (int)xq[3], s1);
    s0 = __dp4a(w[4], (int)xq[4], s0);
    s1 = __dp4a(w[5], (int)xq[5], s1);
    s0 = __dp4a(w[6], (int)xq[6], s0);
    s1 = __dp4a(w[7], (int)xq[7], s1);
    return s0 + s1;
}

// y[r] = W[r] . x for the CTA's rows, x: q8_1 blocks (36 B: half d, half s, 32 int8) in shared
// memory.  Warp w of the CTA takes rows r0 + w, r0 + w + 8, ..., R at a time, and of a row the
// blocks lane, lane + 32, ... in groups of NBL: every weight load of a group (R rows x NBL
// blocks) is issued before its math, which then runs in block order per row.
template <int R, int NBL>
__device__ __noinline__ void gemv_rows_t(const void* wv, const uint8_t* xs, float* y, uint32_t rows, uint32_t k) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nb = k / 32;
    uint32_t r0, r1;
    cta_rows(rows, r0, r1);
    const uint8_t* W = static_cast<const uint8_t*>(wv);
    for (uint32_t rb = r0 + warp; rb < r1; rb += DS_WARPS * R) {
        float acc[R];
        const uint8_t* row[R];
#pragma unroll
        for (int j = 0; j < R; j++) {
            acc[j] = 0.0f;
            row[j] = W + (size_t)min(rb + DS_WARPS * j, r1 - 1) * nb * Q8_0_BYTES;
        }
        for (uint32_t b0 = 0; b0 < nb; b0 += 32 * NBL) {
            int wq[R][NBL][8];
            float dw[R][NBL];
#pragma unroll
            for (int j = 0; j < R; j++)
#pragma unroll
                for (int i = 0; i < NBL; i++) {
                    const uint32_t b = b0 + lane + 32 * i;
                    if (b < nb) q80_block(row[j], b, wq[j][i], dw[j][i]);
                }
#pragma unroll
            for (int i = 0; i < NBL; i++) {
                const uint32_t b = b0 + lane + 32 * i;
                if (b < nb) {
                    const uint32_t* xb = reinterpret_cast<const uint32_t*>(xs + (size_t)b * Q8_1_BYTES);
                    const float d8 = h2f_bits((uint16_t)(xb[0] & 0xffffu));
#pragma unroll
                    for (int j = 0; j < R; j++)
                        acc[j] = __fmaf_rn(__fmul_rn(dw[j][i], d8), (float)dot8q(wq[j][i], xb + 1), acc[j]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < R; j++) {
            float v = acc[j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (lane == 0 && rb + DS_WARPS * j < r1) y[rb + DS_WARPS * j] = v;
        }
    }
}

// short rows (<= 32 blocks): four rows per warp at a time; long rows: one row, five blocks per lane
CFI_DEV void gemv_rows(const void* wv, const uint8_t* xs, float* y, uint32_t rows, uint32_t k) {
    if (k / 32 <= 32)
        gemv_rows_t<4, 1>(wv, xs, y, rows, k);
    else
        gemv_rows_t<1, 5>(wv, xs, y, rows, k);
}

// q8_1 blocks another CTA wrote -> shared memory (through L2)
CFI_DEV void stage_q81(const void* src, uint8_t* dst, uint32_t nblocks) {
    const uint32_t* s = static_cast<const uint32_t*>(src);
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    for (uint32_t i = threadIdx.x; i < nblocks * (Q8_1_BYTES / 4); i += DS_THREADS) d[i] = __ldcg(s + i);
}

// Split attention for query head h and position range `split` (cfi_fused_attention_q8_1's
// attention_q81 body, with every value written during this launch read through L2); the last
// CTA of the head combines the ranges in order and writes the head's q8_1 blocks.
__device__ __noinline__ void attention_unit(const DsArgs& a, const CfiDecodeLayer& lay, int h, int split, float* sc, float* red,
                            float* qs, float* o, int* last) {
    const CfiDecodeStep& m = a.m;
    const int head_dim = m.head_dim, n_ctx = m.n_ctx, nsplit = a.att_nsplit, chunk = a.att_chunk;
    const int kvh = h / (m.n_head / m.n_kv_head);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int npos = min(__ldcg(m.pos) + 1, n_ctx);
    const int j0 = split * chunk, j1 = min(npos, j0 + chunk);
    const __half* K = static_cast<const __half*>(lay.kc) + (size_t)kvh * n_ctx * head_dim;
    const __half* V = static_cast<const __half*>(lay.vc) + (size_t)kvh * head_dim * n_ctx;
    if (tid < head_dim) qs[tid] = __ldcg(m.qr + (size_t)h * head_dim + tid);
    __syncthreads();
    float mx = -INFINITY;
    const int nv = head_dim / 8;
    for (int jj = tid; j0 + jj < j1; jj += 256) {
        const uint4* kr = reinterpret_cast<const uint4*>(K + (size_t)(j0 + jj) * head_dim);
        uint4 kv[16];
#pragma unroll
        for (int e = 0; e < 16; e++)
            if (e < nv) kv[e] = __ldcg(kr + e);
        float acc = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; e++) {
            if (e < nv) {
                const __half2* hp = reinterpret_cast<const __half2*>(&kv[e]);
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const float2 f = __half22float2(hp[t]);
                    acc = __fmaf_rn(qs[8 * e + 2 * t], f.x, acc);
                    acc = __fmaf_rn(qs[8 * e + 2 * t + 1], f.y, acc);
                }
            }
        }
        const float sj = acc * a.scale;
        sc[jj] = sj;
        mx = fmaxf(mx, sj);
    }
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = warp_max(lane < 8 ? red[lane] : -INFINITY);
    __syncthreads();
    float sum = 0.0f;
    const int cnt = max(0, j1 - j0), cpad = (cnt + 7) & ~7;
    for (int jj = tid; jj < cpad; jj += 256) {
        const float e = jj < cnt ? expf(sc[jj] - mx) : 0.0f;
        sc[jj] = e;
        sum += e;
    }
    // block sum over 256 threads in the order of the native rms_norm
    sum = warp_sum(sum);
    __syncthreads();
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    sum = warp_sum(lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f);
    __syncthreads();
    const int tpd = 256 / head_dim, d = tid / tpd, part = tid % tpd;
    const uint4* vr = reinterpret_cast<const uint4*>(V + (size_t)d * n_ctx + j0);
    const int nrun = cpad / 8;
    float acc = 0.0f;
    for (int r0 = part; r0 < nrun; r0 += 4 * tpd) {
        uint4 vv[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int r = r0 + u * tpd;
            vv[u] = r < nrun ? __ldcg(vr + r) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int r = r0 + u * tpd;
            if (r < nrun) {
                const __half2* hp = reinterpret_cast<const __half2*>(&vv[u]);
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const float2 f = __half22float2(hp[t]);
                    acc = __fmaf_rn(sc[8 * r + 2 * t], f.x, acc);
                    acc = __fmaf_rn(sc[8 * r + 2 * t + 1], f.y, acc);
                }
            }
        }
    }
    for (int off = tpd / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    float* pp = a.att_part + ((size_t)h * CFI_ATT_MAX_SPLIT + split) * (2 + 128);
    if (part == 0) pp[2 + d] = acc;
    if (tid == 0) {
        pp[0] = mx;
        pp[1] = sum;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) *last = atomicAdd(&a.att_count[h], 1u) == (unsigned)nsplit - 1;
    __syncthreads();
    if (!*last) return;
    __threadfence();
    const float* hp0 = a.att_part + (size_t)h * CFI_ATT_MAX_SPLIT * (2 + 128);
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; sp++) M = fmaxf(M, __ldcg(hp0 + sp * (2 + 128)));
    if (tid < head_dim) {
        float num = 0.0f, den = 0.0f;
        for (int sp = 0; sp < nsplit; sp++) {
            const float* ps = hp0 + sp * (2 + 128);
            const float ms = __ldcg(ps);
            if (ms == -INFINITY) continue;
            const float f = expf(ms - M);
            num = __fmaf_rn(__ldcg(ps + 2 + tid), f, num);
            den = __fmaf_rn(__ldcg(ps + 1), f, den);
        }
        o[tid] = num / den;
    }
    __syncthreads();
    uint8_t* out = static_cast<uint8_t*>(m.aq);
    for (int b = warp; b < head_dim / 32; b += 8)
        q8_1_store_lane(o[32 * b + lane], out + ((size_t)h * (head_dim / 32) + b) * Q8_1_BYTES, lane);
    if (tid == 0) a.att_count[h] = 0;
}

// A norm weight vector -> shared memory by 16-byte cp.async (n % 4 == 0), landing while the
// CTA works on the phase before the norm; ds_wait_staged() before the first read.
CFI_DEV void ds_stage_async(const float* w, float* dst, int n) {
    for (int i = threadIdx.x; i < n / 4; i += DS_THREADS)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(sm100::smem_u32(dst + 4 * i)), "l"(w + 4 * i)
                     : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
}
CFI_DEV void ds_wait_staged() {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
}

// epi_add_rmsnorm_q81 with the norm weight already in shared memory: the same operations in the
// same order (x += y, the 256-thread-strided sum of squares, rsqrtf, scale * x * w, the lane-form
// q8_1 store), so the same bits.
CFI_DEV void ds_add_rmsnorm_q81(float* __restrict__ x, const float* __restrict__ y, const float* __restrict__ wsm,
                                uint8_t* __restrict__ out, int n, float eps, float* hbuf) {
    __shared__ float red[32];
    __shared__ float s_scale;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = blockDim.x;
    for (int c = tid; c < n; c += nt) {
        float v = x[c];
        if (y) {
            v += __ldcg(y + c);
            x[c] = v;
        }
        hbuf[c] = v;
    }
    __syncthreads();
    if (warp < 8) {
        float ss = 0.0f;
        for (int c = tid; c < n; c += 256) ss = __fmaf_rn(hbuf[c], hbuf[c], ss);
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
    }
    __syncthreads();
    if (warp == 0) {
        const float t = warp_sum(lane < 8 ? red[lane] : 0.0f);
        if (lane == 0) s_scale = rsqrtf(t / (float)n + eps);
    }
    __syncthreads();
    const float scale = s_scale;
    for (int c = tid; c < n; c += nt) {
        float v = scale * hbuf[c];
        v = v * wsm[c];
        q8_1_store_lane(v, out + (size_t)(c / 32) * Q8_1_BYTES, lane);
    }
}

// One row's dot (the GEMV's per-row model), the sum in every lane.
CFI_DEV float gemv_one_row(const void* wv, uint32_t row, const uint8_t* xs, uint32_t k) {
    const uint32_t lane = threadIdx.x & 31, nb = k / 32;
    const uint8_t* rp = static_cast<const uint8_t*>(wv) + (size_t)row * nb * Q8_0_BYTES;
    float acc = 0.0f;
    for (uint32_t b = lane; b < nb; b += 32) {
        int wq[8];
        float dw;
        q80_block(rp, b, wq, dw);
        const uint32_t* xb = reinterpret_cast<const uint32_t*>(xs + (size_t)b * Q8_1_BYTES);
        const float d8 = h2f_bits((uint16_t)(xb[0] & 0xffffu));
        acc = __fmaf_rn(__fmul_rn(dw, d8), (float)dot8q(wq, xb + 1), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    return acc;
}

// The QKV GEMV with the bias, rope and cache stores of epi_qkv_rope_store folded in.  Unit u < the
// rotation units takes rotation pairs 4u .. 4u + 3 (warp w < 4: the first row of pair 4u + w,
// w >= 4: the second row of pair 4u + w - 4); a later unit takes 8 consecutive v rows.  Each item
// is then finished exactly as epi_qkv_rope_store finishes it (the same operations on the same
// values), and qkv gets the raw GEMV outputs as the GEMV would leave them.
CFI_DEV void ds_qkv_rope(const DsArgs& a, const CfiDecodeLayer& lay, const uint8_t* xs, float* sres) {
    const CfiDecodeStep& m = a.m;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int head_dim = m.head_dim, half = head_dim / 2;
    const int nq = m.n_head * head_dim, nkv = m.n_kv_head * head_dim;
    const int npairs = (nq + nkv) / 2, rot_units = npairs / 4, units = rot_units + nkv / 8;
    const int p = __ldcg(m.pos);
    const bool in_cache = p >= 0 && p < m.n_ctx;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        int row;
        if (u < rot_units) {
            const int i = 4 * u + (warp & 3), head = i / half, j = i - head * half;
            row = head * head_dim + j + (warp >= 4 ? half : 0);
        } else {
            row = nq + nkv + 8 * (u - rot_units) + warp;
        }
        const float v = gemv_one_row(lay.wqkv, (uint32_t)row, xs, (uint32_t)m.hidden);
        if (lane == 0) {
            m.qkv[row] = v;
            sres[warp] = v;
        }
        __syncthreads();
        if (u < rot_units && tid < 4) {
            const int i = 4 * u + tid, head = i / half, j = i - head * half;
            const int base = head * head_dim;
            const float x0 = sres[tid] + lay.bqkv[base + j];
            const float x1 = sres[tid + 4] + lay.bqkv[base + j + half];
            const float theta = __fmul_rn((float)p, powf(a.theta_scale, (float)(2 * j) / 2.0f));
            float sn, cs;
            sincosf(theta, &sn, &cs);
            const float y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
            if (base < nq) {
                m.qr[base + j] = y0;
                m.qr[base + j + half] = y1;
            } else if (in_cache) {
                const int kh = (base - nq) / head_dim;
                __half* kr = static_cast<__half*>(lay.kc) + ((size_t)kh * m.n_ctx + p) * head_dim;
                kr[j] = __float2half_rn(y0);
                kr[j + half] = __float2half_rn(y1);
            }
        } else if (u >= rot_units && tid < 8 && in_cache) {
            const int e = 8 * (u - rot_units) + tid, kh = e / head_dim, dd = e - kh * head_dim;
            const float vv = sres[tid] + lay.bqkv[nq + nkv + e];
            static_cast<__half*>(lay.vc)[((size_t)kh * head_dim + dd) * m.n_ctx + p] = __float2half_rn(vv);
        }
        __syncthreads();
    }
}

// L2 prefetch of the K rows and V^T columns the CTA's attention units of this layer will read
CFI_DEV void ds_prefetch_kv(const DsArgs& a, const CfiDecodeLayer& lay) {
    const CfiDecodeStep& m = a.m;
    const int npos = min(__ldcg(m.pos) + 1, m.n_ctx);
    for (int u = blockIdx.x; u < m.n_head * a.att_nsplit; u += gridDim.x) {
        const int h = u / a.att_nsplit, split = u % a.att_nsplit, kvh = h / (m.n_head / m.n_kv_head);
        const int j0 = split * a.att_chunk, j1 = min(npos, j0 + a.att_chunk);
        if (j1 <= j0) continue;
        const __half* K = static_cast<const __half*>(lay.kc) + ((size_t)kvh * m.n_ctx + j0) * m.head_dim;
        if (threadIdx.x == 0) l2_prefetch_range(K, (size_t)(j1 - j0) * m.head_dim * 2);
        const __half* V = static_cast<const __half*>(lay.vc) + (size_t)kvh * m.head_dim * m.n_ctx + j0;
        const int cnt16 = ((j1 - j0) * 2 + 15) / 16 * 16;
        for (int d = threadIdx.x; d < m.head_dim; d += DS_THREADS)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(V + (size_t)d * m.n_ctx), "r"(cnt16) : "memory");
    }
}

__global__ void __launch_bounds__(DS_THREADS, 1) cfi_decode_step_kernel(const DsArgs a) {
    const CfiDecodeStep& m = a.m;
    __shared__ __align__(16) float xs[DS_MAX_HIDDEN];     // the residual stream (every CTA's own copy)
    __shared__ __align__(16) float hbuf[DS_MAX_HIDDEN];   // add_rmsnorm's staging
    __shared__ __align__(16) uint8_t qs8[DS_MAX_FFN_BLOCKS * Q8_1_BYTES];  // q8_1 input of a GEMV
    __shared__ float att_sc[DS_ATT_CHUNK * 2], att_red[32];
    __shared__ __align__(16) float att_q[128];
    __shared__ float att_o[128];
    __shared__ int att_last;
    __shared__ __align__(16) float wn_attn[DS_MAX_HIDDEN];  // the next attention norm's weight
    __shared__ __align__(16) float wn_ffn[DS_MAX_HIDDEN];   // the next FFN norm's weight
    __shared__ float sres[DS_WARPS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = m.hidden, nq = m.n_head * m.head_dim, nkv = m.n_kv_head * m.head_dim, F = m.ffn;
    const unsigned int gwarps = gridDim.x * DS_WARPS, gwarp = blockIdx.x * DS_WARPS + warp;
    unsigned int bar = 0;

    // x = row token[0] of the Q8_0 embedding (get_rows_q8_0)
    {
        const int tok = __ldcg(m.token);
        const uint8_t* erow = static_cast<const uint8_t*>(m.embd) + (size_t)tok * (H / 32) * Q8_0_BYTES;
        for (int c = tid; c < H; c += DS_THREADS) {
            const uint8_t* blk = erow + (size_t)(c / 32) * Q8_0_BYTES;
            const float d = h2f_bits((uint16_t)(blk[0] | (blk[1] << 8)));
            xs[c] = d * (float)(int8_t)blk[2 + c % 32];
        }
        __syncthreads();
    }
    prefetch_rows(a.layers[0].wqkv, nq + 2 * nkv, H);
    ds_stage_async(a.layers[0].attn_norm, wn_attn, H);
    for (int l = 0; l < m.n_layers; l++) {
        const CfiDecodeLayer lay = a.layers[l];
        // hq = q8_1(rms_norm(x += dn) * attn_norm)  (layer 0: no residual)
        ds_wait_staged();
        ds_add_rmsnorm_q81(xs, l > 0 ? m.dn : nullptr, wn_attn, qs8, H, m.eps, hbuf);
        __syncthreads();
        ds_stage_async(lay.ffn_norm, wn_ffn, H);
        // QKV GEMV + bias + rope + K/V cache stores
        ds_qkv_rope(a, lay, qs8, sres);
        ds_prefetch_kv(a, lay);
        prefetch_rows(lay.wo, H, nq);
        if (!grid_sync(a, ++bar)) return;
        for (int u = blockIdx.x; u < m.n_head * a.att_nsplit; u += gridDim.x) {
            attention_unit(a, lay, u / a.att_nsplit, u % a.att_nsplit, att_sc, att_red, att_q, att_o, &att_last);
            __syncthreads();
        }
        if (!grid_sync(a, ++bar)) return;
        stage_q81(m.aq, qs8, nq / 32);
        __syncthreads();
        gemv_rows(lay.wo, qs8, m.o, H, nq);
        prefetch_rows(lay.wgu, 2 * F, H);
        if (!grid_sync(a, ++bar)) return;
        ds_wait_staged();
        ds_add_rmsnorm_q81(xs, m.o, wn_ffn, qs8, H, m.eps, hbuf);
        __syncthreads();
        ds_stage_async(l + 1 < m.n_layers ? a.layers[l + 1].attn_norm : m.out_norm, wn_attn, H);
        gemv_rows(lay.wgu, qs8, m.gu, 2 * F, H);
        prefetch_rows(lay.wd, H, F);
        if (!grid_sync(a, ++bar)) return;
        epi_swiglu_q81(m.gu, static_cast<uint8_t*>(m.gq), F, (int)gwarp, (int)gwarps);
        if (!grid_sync(a, ++bar)) return;
        stage_q81(m.gq, qs8, F / 32);
        __syncthreads();
        gemv_rows(lay.wd, qs8, m.dn, H, F);
        if (l + 1 < m.n_layers) prefetch_rows(a.layers[l + 1].wqkv, nq + 2 * nkv, H);
        else prefetch_rows(m.head, m.vocab, H);
        if (!grid_sync(a, ++bar)) return;
    }
    // logits = head . q8_1(rms_norm(x += dn) * out_norm), then the greedy argmax (argmax_next)
    ds_wait_staged();
    ds_add_rmsnorm_q81(xs, m.dn, wn_attn, qs8, H, m.eps, hbuf);
    __syncthreads();
    if (blockIdx.x == 0) {  // the step's final x and hq, as the kernel chain leaves them
        for (int c = tid; c < H; c += DS_THREADS) m.x[c] = xs[c];
        for (int i = tid; i < H / 32 * (Q8_1_BYTES / 4); i += DS_THREADS)
            reinterpret_cast<uint32_t*>(m.hq)[i] = reinterpret_cast<const uint32_t*>(qs8)[i];
    }
    gemv_rows(m.head, qs8, m.logits, m.vocab, H);
    __syncthreads();
    {
        uint32_t r0, r1;
        cta_rows(m.vocab, r0, r1);
        float best = -INFINITY;
        int idx = 0x7fffffff;
        for (uint32_t i = r0 + tid; i < r1; i += DS_THREADS) {
            const float v = __ldcg(m.logits + i);
            if (v > best || (v == best && (int)i < idx)) {
                best = v;
                idx = (int)i;
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (ov > best || (ov == best && oi < idx)) {
                best = ov;
                idx = oi;
            }
        }
        __shared__ float bv[DS_WARPS];
        __shared__ int bi[DS_WARPS];
        if (lane == 0) {
            bv[warp] = best;
            bi[warp] = idx;
        }
        __syncthreads();
        if (warp == 0) {
            best = lane < DS_WARPS ? bv[lane] : -INFINITY;
            idx = lane < DS_WARPS ? bi[lane] : 0x7fffffff;
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, best, o);
                const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
                if (ov > best || (ov == best && oi < idx)) {
                    best = ov;
                    idx = oi;
                }
            }
            int last = 0;
            if (lane == 0) {
                a.amax_val[blockIdx.x] = best;
                a.amax_idx[blockIdx.x] = idx;
                __threadfence();
                last = atomicAdd(a.amax_count, 1u) == gridDim.x - 1;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
                best = -INFINITY;
                idx = 0x7fffffff;
                for (int b = lane; b < (int)gridDim.x; b += 32) {
                    const float v = __ldcg(&a.amax_val[b]);
                    const int i = __ldcg(&a.amax_idx[b]);
                    if (v > best || (v == best && i < idx)) {
                        best = v;
                        idx = i;
                    }
                }
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
                    if (ov > best || (ov == best && oi < idx)) {
                        best = ov;
                        idx = oi;
                    }
                }
                if (lane == 0) {
                    m.token[0] = idx;
                    m.pos[0] += 1;
                    *a.amax_count = 0;
                }
            }
        }
    }
}

}  // namespace

extern "C" int cfi_decode_step_q8_0(const CfiDecodeStep* s, const CfiDecodeLayer* layers_dev, void* stream) {
    if (!s || !layers_dev) return (int)cudaErrorInvalidValue;
    const CfiDecodeStep& m = *s;
    const int nq = m.n_head * m.head_dim, nkv = m.n_kv_head * m.head_dim;
    if (m.hidden <= 0 || m.hidden > DS_MAX_HIDDEN || m.hidden % 64 || ((m.n_head + m.n_kv_head) * m.head_dim / 2) % 4 || m.ffn % 64 || m.ffn / 32 > DS_MAX_FFN_BLOCKS ||
        nq % 64 || nq / 32 > DS_MAX_FFN_BLOCKS || (m.head_dim != 64 && m.head_dim != 128) || m.n_kv_head <= 0 ||
        m.n_head % m.n_kv_head || m.n_head > CFI_ATT_MAX_HEADS || m.n_ctx <= 0 || m.n_ctx % 8 || m.n_ctx > 8192 ||
        m.n_layers <= 0 || m.vocab <= 0 || nkv % 32)
        return (int)cudaErrorInvalidValue;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int dev = 0, sms = 0, coop = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    if (!coop || sms <= 0) return (int)cudaErrorNotSupported;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, cfi_decode_step_kernel, DS_THREADS, 0) != cudaSuccess ||
        per_sm < 1)
        return (int)cudaErrorNotSupported;
    const int grid = sms < CFI_AMAX_CTAS ? sms : CFI_AMAX_CTAS;  // one CTA per SM, every one resident
    CfiGlueSlot sl;
    int rc = cfi_glue_slot(st, &sl);
    if (rc) return rc;
    int e = 0;
    unsigned int* sync = static_cast<unsigned int*>(cfi_stream_buffer(CFI_BUF_DECODE_SYNC, 64, st, &e));
    if (!sync) return e ? e : (int)cudaErrorMemoryAllocation;
    DsArgs a;
    a.m = m;
    a.layers = layers_dev;
    a.sync = sync;
    a.att_part = sl.att_part;
    a.att_count = sl.att_count;
    a.amax_val = sl.amax_val;
    a.amax_idx = sl.amax_idx;
    a.amax_count = sl.amax_count;
    a.att_nsplit = (m.n_ctx + DS_ATT_CHUNK - 1) / DS_ATT_CHUNK;
    a.att_chunk = ((m.n_ctx + a.att_nsplit - 1) / a.att_nsplit + 7) / 8 * 8;
    a.theta_scale = powf(m.theta, -2.0f / (float)m.head_dim);  // as cfi_fused_qkv_rope_store
    a.scale = 1.0f / sqrtf((float)m.head_dim);
    if (a.att_nsplit > CFI_ATT_MAX_SPLIT) return (int)cudaErrorInvalidValue;
    cudaError_t ce = cudaMemsetAsync(sync, 0, 8, st);
    if (ce != cudaSuccess) return (int)ce;
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned)grid, 1, 1);
    c.blockDim = dim3(DS_THREADS, 1, 1);
    c.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    c.attrs = at;
    c.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&c, cfi_decode_step_kernel, a);
}

extern "C" unsigned int cfi_decode_step_error(void) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_ds_error, sizeof v) != cudaSuccess) return 0xffffffffu;
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_ds_error, &z, sizeof z);
    return v;
}
