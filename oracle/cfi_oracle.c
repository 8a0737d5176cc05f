/*
 * cfi_oracle.c -- scalar CPU oracle (TEST INFRASTRUCTURE ONLY; see cfi_oracle.h).
 *
 * A restatement, in C, of the host reference math of cuda-for-intel's kernel-substitution layer.
 * Citations are file:line inside the reference project.  Build with -ffp-contract=off: every
 * fused multiply-add below is an explicit fmaf(), exactly where the reference calls mul_add.
 */
#include "cfi_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- refs.rs:35-45 ---- */
float cfo_f16_to_f32(uint16_t h) {
    uint32_t s = h >> 15, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    float mag;
    if (e == 0)
        mag = (float)m * ldexpf(1.0f, -24);
    else if (e == 0x1f)
        mag = m == 0 ? INFINITY : NAN;
    else
        mag = (1.0f + (float)m / 1024.0f) * ldexpf(1.0f, (int)e - 15);
    return s ? -mag : mag;
}

/* ---- refs.rs:47-80: round to nearest even ---- */
uint16_t cfo_f32_to_f16(float x) {
    uint32_t b;
    memcpy(&b, &x, 4);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000);
    int32_t exp = (int32_t)((b >> 23) & 0xff);
    uint32_t man = b & 0x7fffff;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00 | (man ? 0x200 : 0));
    int32_t e = exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00);
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t mant = man | 0x800000;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t half = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (half & 1))) half += 1;
        return (uint16_t)(sign | half);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h += 1;
    return (uint16_t)(sign | h);
}

/* ---- refs.rs:82-100 ---- */
void cfo_fastdiv_values(uint32_t d, uint32_t out[3]) {
    uint32_t l = 0;
    while (l < 32 && (1ull << l) < (uint64_t)d) l++;
    uint64_t mp = (((1ull << 32) * ((1ull << l) - (uint64_t)d)) / (uint64_t)d) + 1;
    out[0] = (uint32_t)mp;
    out[1] = l;
    out[2] = d;
}
uint32_t cfo_fastdiv(uint32_t n, const uint32_t v[3]) {
    uint32_t hi = (uint32_t)(((uint64_t)n * (uint64_t)v[0]) >> 32);
    return (hi + n) >> v[1];
}
uint32_t cfo_fastmodulo(uint32_t n, const uint32_t v[3]) { return n - cfo_fastdiv(n, v) * v[2]; }

/* ---- refs.rs:102-115 ---- */
static void warp_sum(float lanes[32]) {
    static const int offs[5] = {16, 8, 4, 2, 1};
    for (int o = 0; o < 5; o++) {
        float old[32];
        memcpy(old, lanes, sizeof old);
        for (int l = 0; l < 32; l++) lanes[l] = old[l] + old[l ^ offs[o]];
    }
}
static float fmax_nan(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}
static void wr16(uint8_t *p, uint16_t v) {
    p[0] = (uint8_t)v;
    p[1] = (uint8_t)(v >> 8);
}
static float rdf32(const uint8_t *p) {
    float f;
    uint32_t u = rd32(p);
    memcpy(&f, &u, 4);
    return f;
}
static float h2f(const uint8_t *p) { return cfo_f16_to_f32(rd16(p)); }

/* ---- refs.rs:117-147 ---- */
void cfo_quantize_q8_1(const float *x, size_t n, uint8_t *out) {
    for (size_t ib = 0; ib < n / 32; ib++) {
        const float *c = x + ib * 32;
        float amax[32], sum[32];
        for (int l = 0; l < 32; l++) {
            amax[l] = fabsf(c[l]);
            sum[l] = c[l];
        }
        static const int offs[5] = {16, 8, 4, 2, 1};
        for (int o = 0; o < 5; o++) {
            float old[32];
            memcpy(old, amax, sizeof old);
            for (int l = 0; l < 32; l++) amax[l] = fmax_nan(old[l], old[l ^ offs[o]]);
        }
        warp_sum(sum);
        float a = amax[0];
        float d = a / 127.0f;
        uint8_t *o = out + ib * 36;
        wr16(o, cfo_f32_to_f16(d));
        wr16(o + 2, cfo_f32_to_f16(sum[0]));
        for (int l = 0; l < 32; l++) {
            int8_t q = a == 0.0f ? 0 : (int8_t)(int32_t)roundf(c[l] / d);
            o[4 + l] = (uint8_t)q;
        }
    }
}

/* ---- refs.rs:149-155 ---- */
int32_t cfo_dp4a(uint32_t a, uint32_t b, int32_t c) {
    uint32_t s = (uint32_t)c;
    for (int k = 0; k < 4; k++)
        s += (uint32_t)((int32_t)(int8_t)(a >> (8 * k)) * (int32_t)(int8_t)(b >> (8 * k)));
    return (int32_t)s;
}

/* refs.rs:157-160: little-endian dword `word` of a byte span */
static uint32_t b2(const uint8_t *bytes, size_t word) { return rd32(bytes + word * 4); }

/* ggml get_scale_min_k4 (refs.rs:671-681) */
static void scale_min_k4(size_t j, const uint8_t *s, int32_t *sc, int32_t *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* ---- refs.rs:166-259 ---- */
float cfo_vec_dot(uint32_t ty, const uint8_t *xb, const uint8_t *yb, size_t kqs, float acc) {
#define YQ(blk, word) b2(yb + (blk) * 36 + 4, (word))
#define YD(blk) h2f(yb + (blk) * 36)
#define YS(blk) h2f(yb + (blk) * 36 + 2)
    switch (ty) {
    case CFO_Q8_0: {
        float d0 = h2f(xb);
        int32_t sumi = 0;
        for (size_t i = 0; i < 2; i++) sumi = cfo_dp4a(b2(xb + 2, kqs + i), YQ(0, kqs + i), sumi);
        return fmaf(d0 * YD(0), (float)sumi, acc);
    }
    case CFO_Q4_0: {
        float d4 = h2f(xb);
        int32_t sumi = 0;
        for (size_t i = 0; i < 2; i++) {
            uint32_t v = b2(xb + 2, kqs + i);
            sumi = cfo_dp4a(v & 0x0F0F0F0F, YQ(0, kqs + i), sumi);
            sumi = cfo_dp4a((v >> 4) & 0x0F0F0F0F, YQ(0, kqs + i + 4), sumi);
        }
        float inner = fmaf(YD(0), (float)sumi, YS(0) * -4.0f);
        return fmaf(d4, inner, acc);
    }
    case CFO_Q4_K: {
        float dm0 = h2f(xb), dm1 = h2f(xb + 2);
        const uint8_t *scales = xb + 4, *qs = xb + 16;
        size_t bq8_offset = 2 * ((kqs / 2) / 4);
        size_t q4 = 16 * bq8_offset + 4 * ((kqs / 2) % 4);
        uint32_t v[2] = {b2(qs + q4, 0), b2(qs + q4, 4)};
#define SC16(i) ((uint16_t)(scales[2 * (i)] | (scales[2 * (i) + 1] << 8)))
        size_t j = bq8_offset / 2;
        uint16_t aux[2];
        if (j < 2) {
            aux[0] = SC16(j) & 0x3f3f;
            aux[1] = SC16(j + 2) & 0x3f3f;
        } else {
            aux[0] = (uint16_t)((SC16(j + 2) & 0x0f0f) | ((SC16(j - 2) & 0xc0c0) >> 2));
            aux[1] = (uint16_t)(((SC16(j + 2) >> 4) & 0x0f0f) | ((SC16(j) & 0xc0c0) >> 2));
        }
#undef SC16
        uint8_t sc[2] = {(uint8_t)aux[0], (uint8_t)(aux[0] >> 8)};
        uint8_t m[2] = {(uint8_t)aux[1], (uint8_t)(aux[1] >> 8)};
        float sumf_d = 0.0f, sumf_m = 0.0f;
        for (size_t i = 0; i < 2; i++) {
            size_t blk = bq8_offset + i;
            uint32_t u0 = YQ(blk, (kqs / 2) % 4);
            uint32_t u1 = YQ(blk, (kqs / 2) % 4 + 4);
            uint32_t v0 = (v[0] >> (4 * i)) & 0x0F0F0F0F;
            uint32_t v1 = (v[1] >> (4 * i)) & 0x0F0F0F0F;
            int32_t dot1 = cfo_dp4a(v1, u1, cfo_dp4a(v0, u0, 0));
            int32_t dot2 = cfo_dp4a(0x01010101, u1, cfo_dp4a(0x01010101, u0, 0));
            float d8 = YD(blk);
            sumf_d = fmaf(d8, (float)(int32_t)((uint32_t)dot1 * (uint32_t)sc[i]), sumf_d);
            sumf_m = fmaf(d8, (float)(int32_t)((uint32_t)dot2 * (uint32_t)m[i]), sumf_m);
        }
        return acc + (sumf_d * dm0 - sumf_m * dm1);
    }
    case CFO_Q6_K: {
        const uint8_t *ql = xb, *qh = xb + 128, *scales = xb + 192;
        float d = h2f(xb + 208);
        size_t bq8_offset = 2 * 2 * (kqs / 16) + (kqs % 16) / 8;
        size_t scale_offset = 8 * (kqs / 16) + (kqs % 16) / 4;
        uint32_t vh_shift = (uint32_t)(2 * ((kqs % 16) / 8));
        uint32_t vl = b2(ql, kqs);
        uint32_t vh = b2(qh, 8 * (kqs / 16) + kqs % 8) >> vh_shift;
        float sumf = 0.0f;
        for (size_t i = 0; i < 2; i++) {
            int32_t sc = (int8_t)scales[scale_offset + 4 * i];
            uint32_t vil = (vl >> (4 * i)) & 0x0F0F0F0F;
            uint32_t vih = ((vh >> (4 * i)) << 4) & 0x30303030;
            uint32_t comb = vil | vih, sub = 0;
            for (int k = 0; k < 4; k++) {
                int32_t byte = (int32_t)((comb >> (8 * k)) & 0xff) - 32;
                sub |= ((uint32_t)byte & 0xff) << (8 * k);
            }
            uint32_t u = YQ(bq8_offset + 2 * i, kqs % 8);
            float d8 = YD(bq8_offset + 2 * i);
            sumf = fmaf(d8, (float)(int32_t)((uint32_t)cfo_dp4a(sub, u, 0) * (uint32_t)sc), sumf);
        }
        return fmaf(d, sumf, acc);
    }
    default:
        abort();
    }
#undef YQ
#undef YD
#undef YS
}

typedef struct {
    size_t qk, qi, vdr, block_bytes;
} traits_t;

/* refs.rs:25-33 */
static int traits(uint32_t ty, traits_t *t) {
    switch (ty) {
    case CFO_Q4_0: *t = (traits_t){32, 4, 2, 18}; return 1;
    case CFO_Q8_0: *t = (traits_t){32, 8, 2, 34}; return 1;
    case CFO_Q4_K: *t = (traits_t){256, 32, 2, 144}; return 1;
    case CFO_Q6_K: *t = (traits_t){256, 32, 1, 210}; return 1;
    default: return 0;
    }
}

/* ---- refs.rs:286-299 ---- */
static size_t mmvq_rpb(const cfo_mmvq *p) { return p->ncols_dst == 1 ? 1 : 2; }

/* ---- refs.rs:302-382: thread-by-thread simulation of stock mul_mat_vec_q ---- */
void cfo_mmvq_run(const cfo_mmvq *p, const uint8_t *x, const uint8_t *y, const int32_t *ids, float *dst) {
    traits_t t;
    if (!traits(p->ty, &t)) abort();
    size_t rpb = mmvq_rpb(p), nw = p->nwarps;
    size_t blocks_per_row_x = p->ncols_x / t.qk;
    size_t blocks_per_iter = t.vdr * nw * 32 / t.qi;
    uint32_t chr[3], smr[3], nchy[3];
    cfo_fastdiv_values(p->channel_ratio ? p->channel_ratio : 1, chr);
    cfo_fastdiv_values(p->sample_ratio ? p->sample_ratio : 1, smr);
    cfo_fastdiv_values(p->nchannels_y ? p->nchannels_y : 1, nchy);
    uint32_t gx = (uint32_t)((p->nrows_x + rpb - 1) / rpb), gy = p->nchannels_dst, gz = p->nsamples_dst;
    size_t nd = p->ncols_dst;
    float *tmp = (float *)malloc(sizeof(float) * nw * 32 * nd * rpb);
    for (uint32_t bz = 0; bz < gz; bz++)
        for (uint32_t by = 0; by < gy; by++)
            for (uint32_t bx = 0; bx < gx; bx++) {
                size_t row0 = rpb * bx;
                uint32_t channel_dst = by;
                uint32_t channel_x = (nd == 1 && p->use_ids) ? (uint32_t)ids[channel_dst] : cfo_fastdiv(channel_dst, chr);
                uint32_t channel_y = (nd == 1 && p->use_ids) ? cfo_fastmodulo(channel_dst, nchy) : channel_dst;
                uint32_t sample_dst = bz, sample_x = cfo_fastdiv(sample_dst, smr), sample_y = sample_dst;
                size_t y_base = (size_t)sample_y * p->stride_sample_y + (size_t)channel_y * p->stride_channel_y;
                size_t kbx_offset = (size_t)sample_x * p->stride_sample_x + (size_t)channel_x * p->stride_channel_x +
                                    row0 * p->stride_row_x;
                memset(tmp, 0, sizeof(float) * nw * 32 * nd * rpb);
#define TMP(w, lane, j, i) tmp[(((w) * 32 + (lane)) * nd + (j)) * rpb + (i)]
                for (size_t w = 0; w < nw; w++)
                    for (size_t lane = 0; lane < 32; lane++) {
                        size_t tid = 32 * w + lane;
                        for (size_t kbx = tid / (t.qi / t.vdr); kbx < blocks_per_row_x; kbx += blocks_per_iter) {
                            size_t kby = kbx * (t.qk / 32);
                            size_t kqs = t.vdr * (tid % (t.qi / t.vdr));
                            for (size_t j = 0; j < nd; j++)
                                for (size_t i = 0; i < rpb; i++) {
                                    if (i > 0 && row0 + i >= p->stride_col_dst) continue;
                                    size_t xb_i = kbx_offset + i * p->stride_row_x + kbx;
                                    size_t yb_i = y_base + j * p->stride_col_y + kby;
                                    TMP(w, lane, j, i) = cfo_vec_dot(p->ty, x + xb_i * t.block_bytes, y + yb_i * 36,
                                                                     kqs, TMP(w, lane, j, i));
                                }
                        }
                    }
                size_t dst_base = (size_t)sample_dst * p->stride_sample_dst +
                                  (size_t)channel_dst * p->stride_channel_dst + row0;
                for (size_t j = 0; j < nd; j++) {
                    float lanes[2][32];
                    for (size_t i = 0; i < rpb; i++) {
                        for (size_t lane = 0; lane < 32; lane++) {
                            float v = TMP(0, lane, j, i);
                            for (size_t l = 1; l < nw; l++) v += TMP(l, lane, j, i);
                            lanes[i][lane] = v;
                        }
                        warp_sum(lanes[i]);
                    }
                    for (size_t tx = 0; tx < rpb; tx++)
                        if (rpb == 1 || row0 + tx < p->stride_col_dst)
                            dst[dst_base + j * p->stride_col_dst + tx] = lanes[tx][0];
                }
#undef TMP
            }
    free(tmp);
}

/* ---- refs.rs:384-433 ---- */
float cfo_vec_dot_wide(uint32_t ty, const uint8_t *xb, const uint8_t *yb, size_t g, float acc) {
    float d8 = h2f(yb);
#define U(i) b2(yb + 4, (i))
#define W(o, i) b2(xb + (o), (i))
    switch (ty) {
    case CFO_Q8_0: {
        float dx = h2f(xb);
        int32_t sumi = 0;
        for (size_t i = 0; i < 8; i++) sumi = cfo_dp4a(W(2, i), U(i), sumi);
        return fmaf(dx * d8, (float)sumi, acc);
    }
    case CFO_Q4_K: {
        float dx = h2f(xb), dmin = h2f(xb + 2);
        int32_t sc, m;
        scale_min_k4(g, xb + 4, &sc, &m);
        int32_t sumi = 0, sumy = 0;
        for (size_t i = 0; i < 8; i++) {
            uint32_t v = (W(16 + 32 * (g / 2), i) >> (4 * (g & 1))) & 0x0F0F0F0F;
            sumi = cfo_dp4a(v, U(i), sumi);
            sumy = cfo_dp4a(0x01010101, U(i), sumy);
        }
        float a = d8 * (float)(int32_t)((uint32_t)sumi * (uint32_t)sc);
        float b = d8 * (float)(int32_t)((uint32_t)sumy * (uint32_t)m);
        return acc + (dx * a - dmin * b);
    }
    case CFO_Q6_K: {
        size_t h = g / 4, sub = g % 4;
        float dx = h2f(xb + 208);
        int32_t tot = 0;
        for (size_t half = 0; half < 2; half++) {
            int32_t sumi = 0, sumu = 0;
            for (size_t i = 4 * half; i < 4 * half + 4; i++) {
                uint32_t lo = (W(64 * h + 32 * (sub & 1), i) >> (4 * (sub >> 1))) & 0x0F0F0F0F;
                uint32_t hi = ((W(128 + 32 * h, i) >> (2 * sub)) & 0x03030303) << 4;
                sumi = cfo_dp4a(lo | hi, U(i), sumi);
                sumu = cfo_dp4a(0x01010101, U(i), sumu);
            }
            int32_t sc = (int8_t)xb[192 + 8 * h + 2 * sub + half];
            tot = (int32_t)((uint32_t)tot + ((uint32_t)sumi - ((uint32_t)sumu << 5)) * (uint32_t)sc);
        }
        return fmaf(dx * d8, (float)tot, acc);
    }
    default:
        abort();
    }
#undef U
#undef W
}

/* ---- refs.rs:435-497 ---- */
void cfo_mmvq_fast(const cfo_mmvq *p, const uint8_t *x, const uint8_t *y, const int32_t *ids, float *dst,
                   uint32_t warps, uint32_t unroll, int wide) {
    traits_t t;
    if (!traits(p->ty, &t) || p->ncols_dst != 1 || unroll == 0 || unroll > 8) abort();
    size_t tpb = wide ? t.qk / 32 : t.qi / t.vdr;
    size_t step = warps * 32 / tpb;
    size_t blocks_per_row_x = p->ncols_x / t.qk;
    uint32_t chr[3], smr[3], nchy[3];
    cfo_fastdiv_values(p->channel_ratio ? p->channel_ratio : 1, chr);
    cfo_fastdiv_values(p->sample_ratio ? p->sample_ratio : 1, smr);
    cfo_fastdiv_values(p->nchannels_y ? p->nchannels_y : 1, nchy);
    for (uint32_t bz = 0; bz < p->nsamples_dst; bz++)
        for (uint32_t by = 0; by < p->nchannels_dst; by++) {
            uint32_t channel_x = p->use_ids ? (uint32_t)ids[by] : cfo_fastdiv(by, chr);
            uint32_t channel_y = p->use_ids ? cfo_fastmodulo(by, nchy) : by;
            uint32_t sample_x = cfo_fastdiv(bz, smr);
            size_t y_base = (size_t)bz * p->stride_sample_y + (size_t)channel_y * p->stride_channel_y;
            for (size_t row = 0; row < p->nrows_x; row++) {
                size_t kbx_offset = (size_t)sample_x * p->stride_sample_x + (size_t)channel_x * p->stride_channel_x +
                                    row * p->stride_row_x;
                float total = 0.0f;
                for (size_t w = 0; w < warps; w++) {
                    float lanes[32];
                    for (size_t lane = 0; lane < 32; lane++) {
                        size_t tid = 32 * w + lane;
                        size_t kqs = wide ? tid % tpb : t.vdr * (tid % tpb);
                        float acc[8] = {0};
                        for (size_t k = tid / tpb; k < blocks_per_row_x; k += unroll * step)
                            for (size_t u = 0; u < unroll; u++) {
                                size_t ku = k + u * step;
                                if (ku >= blocks_per_row_x) continue;
                                const uint8_t *xb = x + (kbx_offset + ku) * t.block_bytes;
                                if (wide)
                                    acc[u] = cfo_vec_dot_wide(p->ty, xb, y + (y_base + ku * (t.qk / 32) + kqs) * 36,
                                                              kqs, acc[u]);
                                else
                                    acc[u] = cfo_vec_dot(p->ty, xb, y + (y_base + ku * (t.qk / 32)) * 36, kqs, acc[u]);
                            }
                        float v = acc[0];
                        for (size_t u = 1; u < unroll; u++) v += acc[u];
                        lanes[lane] = v;
                    }
                    warp_sum(lanes);
                    total = w == 0 ? lanes[0] : total + lanes[0];
                }
                dst[(size_t)bz * p->stride_sample_dst + (size_t)by * p->stride_channel_dst + row] = total;
            }
        }
}

/* ---- refs.rs:499-515 ---- */
uint64_t cfo_rng_next(uint64_t *s) {
    *s ^= *s >> 12;
    *s ^= *s << 25;
    *s ^= *s >> 27;
    return *s * 0x2545F4914F6CDD1Dull;
}
uint32_t cfo_rng_u32(uint64_t *s) { return (uint32_t)(cfo_rng_next(s) >> 32); }
float cfo_rng_unit(uint64_t *s) { return (float)(cfo_rng_u32(s) >> 8) / (float)(1u << 24) * 2.0f - 1.0f; }

/* refs.rs:629-639 */
size_t cfo_block_bytes(uint32_t ty) {
    switch (ty) {
    case CFO_Q4_0: return 18;
    case CFO_Q5_0: return 22;
    case CFO_Q8_0: return 34;
    case CFO_Q4_K: return 144;
    case CFO_Q5_K: return 176;
    case CFO_Q6_K: return 210;
    default: return 0;
    }
}

/* ---- refs.rs:517-538 ---- */
void cfo_random_blocks(uint32_t ty, size_t nblocks, uint64_t *rng, uint8_t *out) {
    size_t bytes = cfo_block_bytes(ty);
    for (size_t b = 0; b < nblocks; b++) {
        uint8_t *blk = out + b * bytes;
        for (size_t i = 0; i < bytes; i++) blk[i] = (uint8_t)cfo_rng_u32(rng);
        switch (ty) {
        case CFO_Q4_0:
        case CFO_Q5_0:
        case CFO_Q8_0:
            wr16(blk, cfo_f32_to_f16(cfo_rng_unit(rng) * 0.05f));
            break;
        case CFO_Q4_K:
        case CFO_Q5_K:
            wr16(blk, cfo_f32_to_f16(cfo_rng_unit(rng) * 0.05f));
            wr16(blk + 2, cfo_f32_to_f16(cfo_rng_unit(rng) * 0.05f));
            break;
        case CFO_Q6_K:
            wr16(blk + 208, cfo_f32_to_f16(cfo_rng_unit(rng) * 0.05f));
            break;
        }
    }
}

/* ---- refs.rs:540-547 ---- */
double cfo_nmse(const float *got, const float *want, size_t n) {
    double num = 0, den = 0;
    for (size_t i = 0; i < n; i++) {
        double d = (double)(got[i] - want[i]);
        num += d * d;
        den += (double)want[i] * (double)want[i];
    }
    return den == 0.0 ? num : num / den;
}

/* ---- probe.rs:31-78 ---- */
static void mmvq_case_params(uint32_t ty, uint32_t ncols_dst, uint32_t nrows, uint32_t ncols_x, uint32_t nch,
                             uint32_t ratio, uint32_t nsamples, int use_ids, cfo_mmvq *p, size_t *x_blocks,
                             size_t *acts) {
    traits_t t;
    if (!traits(ty, &t)) abort();
    size_t bpr = ncols_x / t.qk;
    size_t nchannels_x = nch / ratio;
    uint32_t ystride_col = ncols_x / 32;
    uint32_t nch_y = use_ids ? 3 : nch;
    size_t nx_ch = nchannels_x > (use_ids ? 4u : 1u) ? nchannels_x : (use_ids ? 4u : 1u);
    memset(p, 0, sizeof *p);
    p->ty = ty;
    p->ncols_dst = ncols_dst;
    p->nwarps = ncols_dst <= 4 ? 4 : 2; /* refs.rs:290-292 */
    p->nrows_x = nrows;
    p->ncols_x = ncols_x;
    p->nchannels_dst = nch;
    p->nsamples_dst = nsamples;
    p->channel_ratio = ratio;
    p->sample_ratio = 1;
    p->nchannels_y = nch_y;
    p->use_ids = use_ids ? 1 : 0;
    p->stride_row_x = (uint32_t)bpr;
    p->stride_col_y = ystride_col;
    p->stride_col_dst = nrows;
    p->stride_channel_x = (uint32_t)(nrows * bpr);
    p->stride_channel_y = ystride_col * ncols_dst;
    p->stride_channel_dst = nrows * ncols_dst;
    p->stride_sample_x = (uint32_t)(nrows * bpr * nx_ch);
    p->stride_sample_y = ystride_col * ncols_dst * nch_y;
    p->stride_sample_dst = nrows * ncols_dst * nch;
    *x_blocks = (size_t)nrows * bpr * nx_ch * nsamples;
    *acts = (size_t)ncols_x * ncols_dst * nch_y * nsamples;
}

void cfo_mmvq_case_sizes(uint32_t ty, uint32_t ncols_dst, uint32_t nrows, uint32_t ncols_x, uint32_t nch,
                         uint32_t ratio, uint32_t nsamples, int use_ids, size_t *x_bytes, size_t *y_bytes,
                         size_t *nids, size_t *dst_len) {
    cfo_mmvq p;
    size_t xb, acts;
    mmvq_case_params(ty, ncols_dst, nrows, ncols_x, nch, ratio, nsamples, use_ids, &p, &xb, &acts);
    *x_bytes = xb * cfo_block_bytes(ty);
    *y_bytes = acts / 32 * 36;
    *nids = nch;
    *dst_len = (size_t)p.nsamples_dst * p.stride_sample_dst;
}

void cfo_mmvq_case(uint32_t ty, uint32_t ncols_dst, uint32_t nrows, uint32_t ncols_x, uint32_t nch,
                   uint32_t ratio, uint32_t nsamples, int use_ids, uint64_t seed, cfo_mmvq *p, uint8_t *x,
                   uint8_t *y, int32_t *ids) {
    uint64_t rng = seed;
    size_t xb, acts;
    mmvq_case_params(ty, ncols_dst, nrows, ncols_x, nch, ratio, nsamples, use_ids, p, &xb, &acts);
    cfo_random_blocks(ty, xb, &rng, x);
    float *a = (float *)malloc(sizeof(float) * acts);
    for (size_t i = 0; i < acts; i++) a[i] = cfo_rng_unit(&rng) * 3.0f;
    cfo_quantize_q8_1(a, acts, y);
    free(a);
    for (uint32_t i = 0; i < nch; i++) ids[i] = (int32_t)((i * 3 + 1) % 4);
}

/* ---- probe.rs:182-204 ---- */
void cfo_quantize_case_x(size_t ne00, size_t ne1, size_t ne2, size_t ne3, uint64_t seed, float *x) {
    uint64_t rng = seed;
    size_t n = ne00 * ne1 * ne2 * ne3;
    for (size_t i = 0; i < n; i++) x[i] = cfo_rng_unit(&rng) * 5.0f;
    for (size_t i = 0; i < 32 && i < n; i++) x[i] = 0.0f;
    for (size_t i = 32; i < 64 && i < n; i++) x[i] *= 1e-6f;
}

void cfo_quantize_case_reference(const float *x, size_t ne00, size_t ne0, size_t rows, uint8_t *out) {
    float *row = (float *)malloc(sizeof(float) * ne0);
    for (size_t r = 0; r < rows; r++) {
        for (size_t i = 0; i < ne0; i++) row[i] = i < ne00 ? x[r * ne00 + i] : 0.0f;
        cfo_quantize_q8_1(row, ne0, out + r * (ne0 / 32) * 36);
    }
    free(row);
}

/* ---- refs.rs:641-649 ---- */
size_t cfo_mmq_groups(uint32_t ty) { return (ty == CFO_Q4_K || ty == CFO_Q5_K || ty == CFO_Q6_K) ? 8 : 1; }
int cfo_mmq_ds4(uint32_t ty) { return ty == CFO_Q4_0 || ty == CFO_Q4_K || ty == CFO_Q5_K; }

static float round_half(float x) { return cfo_f16_to_f32(cfo_f32_to_f16(x)); }

/* ---- refs.rs:659-740 ---- */
typedef struct {
    int8_t q[32];
    float d, m;
    int32_t sc[2];
} xgroup;

static xgroup decode_group(uint32_t ty, const uint8_t *blk, size_t g) {
    xgroup r;
    memset(&r, 0, sizeof r);
    switch (ty) {
    case CFO_Q8_0:
        r.d = h2f(blk);
        for (int i = 0; i < 32; i++) r.q[i] = (int8_t)blk[2 + i];
        break;
    case CFO_Q4_0:
        r.d = h2f(blk);
        for (int i = 0; i < 32; i++) {
            uint8_t v = blk[2 + i % 16];
            r.q[i] = (int8_t)((i < 16 ? (v & 15) : (v >> 4)) - 8);
        }
        break;
    case CFO_Q5_0: {
        r.d = h2f(blk);
        uint32_t qh = rd32(blk + 2);
        for (int i = 0; i < 32; i++) {
            int j = i % 16;
            uint8_t nib = i < 16 ? (blk[6 + j] & 15) : (blk[6 + j] >> 4);
            r.q[i] = (int8_t)((nib | (((qh >> i) & 1) << 4)) - 16);
        }
        break;
    }
    case CFO_Q4_K:
    case CFO_Q5_K: {
        int32_t sc_, m_;
        scale_min_k4(g, blk + 4, &sc_, &m_);
        r.d = round_half(h2f(blk) * (float)sc_);
        r.m = round_half(-h2f(blk + 2) * (float)m_);
        for (int i = 0; i < 32; i++) {
            uint8_t nib, hi = 0;
            if (ty == CFO_Q4_K) {
                uint8_t v = blk[16 + 32 * (g / 2) + i];
                nib = g % 2 == 0 ? (v & 15) : (v >> 4);
            } else {
                uint8_t v = blk[48 + 32 * (g / 2) + i];
                nib = g % 2 == 0 ? (v & 15) : (v >> 4);
                hi = (blk[16 + i] >> g) & 1;
            }
            r.q[i] = (int8_t)(nib | (hi << 4));
        }
        break;
    }
    case CFO_Q6_K:
        r.d = h2f(blk + 208);
        r.sc[0] = (int8_t)blk[192 + 2 * g];
        r.sc[1] = (int8_t)blk[192 + 2 * g + 1];
        for (int i = 0; i < 32; i++) {
            size_t v = 32 * g + i, half = v / 128, rr = v % 128, quad = rr / 32, l = rr % 32;
            uint8_t lo = blk[64 * half + 32 * (quad & 1) + l];
            lo = (quad >> 1) == 0 ? (lo & 15) : (lo >> 4);
            uint8_t hi = (blk[128 + 32 * half + l] >> (2 * quad)) & 3;
            r.q[i] = (int8_t)((lo | (hi << 4)) - 32);
        }
        break;
    default:
        abort();
    }
    return r;
}

/* ---- refs.rs:742-769 ---- */
void cfo_quantize_mmq(uint32_t ty, const float *x, size_t ne0, size_t ncols, uint8_t *out) {
    int ds4 = cfo_mmq_ds4(ty);
    for (size_t col = 0; col < ncols; col++)
        for (size_t g = 0; g < ne0 / 32; g++) {
            const float *v = x + col * ne0 + g * 32;
            float amax = 0.0f;
            for (int l = 0; l < 32; l++) amax = fmax_nan(amax, fabsf(v[l]));
            float d_inv = 127.0f / amax;
            size_t blk = (g / 4) * ncols + col;
            uint8_t *o = out + blk * 144;
            float d = amax == 0.0f ? 0.0f : 1.0f / d_inv;
            if (ds4) {
                float sum = 0.0f;
                for (int l = 0; l < 32; l++) sum += v[l];
                wr16(o + 4 * (g % 4), cfo_f32_to_f16(d));
                wr16(o + 4 * (g % 4) + 2, cfo_f32_to_f16(sum));
            } else {
                memcpy(o + 4 * (g % 4), &d, 4);
            }
            for (int l = 0; l < 32; l++) {
                int8_t q = amax == 0.0f ? 0 : (int8_t)(int32_t)roundf(v[l] * d_inv);
                o[16 + (g % 4) * 32 + l] = (uint8_t)q;
            }
        }
}

/* ---- refs.rs:771-834 ---- */
void cfo_mmq_ref(uint32_t ty, const cfo_mmq *p, const uint8_t *x, const uint8_t *y, float *dst) {
    size_t nb = p->ncols_x / 32;
    size_t bytes = cfo_block_bytes(ty), groups = cfo_mmq_groups(ty);
    int ds4 = cfo_mmq_ds4(ty);
    for (size_t w = 0; w < p->nsamples_y; w++)
        for (size_t z = 0; z < p->nchannels_y; z++) {
            size_t xo = (w / p->sample_ratio) * p->stride_sample_x + (z / p->channel_ratio) * p->stride_channel_x;
            size_t yo = w * p->stride_sample_y + z * p->stride_channel_y;
            for (size_t col = 0; col < p->ncols_dst; col++)
                for (size_t row = 0; row < p->nrows_x; row++) {
                    float sum = 0.0f, tmp = 0.0f;
                    for (size_t kb = 0; kb < nb; kb++) {
                        size_t bi = xo + row * p->stride_row_x + kb / groups;
                        xgroup xg = decode_group(ty, x + bi * bytes, kb % groups);
                        size_t yb_int = yo + (kb / 4) * p->ncols_y * 36 + col * 36;
                        const uint8_t *yb = y + yb_int * 4;
                        size_t hb = 4 * (kb % 4);
                        float d_b, s_b = 0.0f;
                        if (ds4) {
                            d_b = h2f(yb + hb);
                            s_b = h2f(yb + hb + 2);
                        } else {
                            d_b = rdf32(yb + hb);
                        }
                        const uint8_t *yq = yb + 16 + (kb % 4) * 32;
                        int32_t dots[2] = {0, 0};
                        for (int tt = 0; tt < 8; tt++) {
                            uint32_t xw = (uint32_t)(uint8_t)xg.q[4 * tt] | (uint32_t)(uint8_t)xg.q[4 * tt + 1] << 8 |
                                          (uint32_t)(uint8_t)xg.q[4 * tt + 2] << 16 |
                                          (uint32_t)(uint8_t)xg.q[4 * tt + 3] << 24;
                            dots[tt / 4] = cfo_dp4a(xw, b2(yq, tt), dots[tt / 4]);
                        }
                        int32_t dot = (int32_t)((uint32_t)dots[0] + (uint32_t)dots[1]);
                        /* the reference's dp4a chain over words 0..8 is one running sum; the split
                         * above is an exact integer regrouping (wrapping adds commute). */
                        switch (ty) {
                        case CFO_Q8_0:
                        case CFO_Q4_0:
                        case CFO_Q5_0:
                            sum = fmaf(xg.d * (float)dot, d_b, sum);
                            break;
                        case CFO_Q4_K:
                        case CFO_Q5_K: {
                            float tt = xg.d * d_b;
                            sum = fmaf(tt, (float)dot, sum);
                            sum = fmaf(xg.m, s_b, sum);
                            break;
                        }
                        default: {
                            int32_t v = (int32_t)((uint32_t)dots[0] * (uint32_t)xg.sc[0] +
                                                  (uint32_t)dots[1] * (uint32_t)xg.sc[1]);
                            tmp = fmaf((float)v, d_b, tmp);
                            if (kb % 4 == 3 || kb == nb - 1) {
                                size_t bi0 = xo + row * p->stride_row_x + (kb - kb % 4) / groups;
                                float d0 = decode_group(ty, x + bi0 * bytes, (kb - kb % 4) % groups).d;
                                sum = fmaf(tmp, d0, sum);
                                tmp = 0.0f;
                            }
                        }
                        }
                    }
                    dst[w * p->stride_sample_dst + z * p->stride_channel_dst + col * p->stride_col_dst + row] = sum;
                }
        }
}

/* ---- probe.rs:244-279 ---- */
static void mmq_case_params(uint32_t ty, uint32_t ncols_x, uint32_t nrows, uint32_t ncols, uint32_t nch,
                            uint32_t ratio, uint32_t nsamples, cfo_mmq *p, size_t *x_blocks) {
    uint32_t nb = ncols_x / 32 / (uint32_t)cfo_mmq_groups(ty);
    uint32_t nch_x = nch / ratio;
    uint32_t ychan = ncols_x / 128 * ncols * 36;
    memset(p, 0, sizeof *p);
    p->ncols_x = ncols_x;
    p->nrows_x = nrows;
    p->ncols_dst = ncols;
    p->nchannels_y = nch;
    p->nsamples_y = nsamples;
    p->channel_ratio = ratio;
    p->sample_ratio = 1;
    p->stride_row_x = nb;
    p->ncols_y = ncols;
    p->stride_col_dst = nrows;
    p->stride_channel_x = nrows * nb;
    p->stride_channel_y = ychan;
    p->stride_channel_dst = nrows * ncols;
    p->stride_sample_x = nrows * nb * nch_x;
    p->stride_sample_y = ychan * nch;
    p->stride_sample_dst = nrows * ncols * nch;
    *x_blocks = (size_t)nrows * nb * nch_x * nsamples;
}

void cfo_mmq_case_sizes(uint32_t ty, uint32_t ncols_x, uint32_t nrows, uint32_t ncols, uint32_t nch,
                        uint32_t ratio, uint32_t nsamples, size_t *x_bytes, size_t *y_bytes, size_t *dst_len) {
    cfo_mmq p;
    size_t xb;
    mmq_case_params(ty, ncols_x, nrows, ncols, nch, ratio, nsamples, &p, &xb);
    *x_bytes = xb * cfo_block_bytes(ty);
    *y_bytes = (size_t)nch * nsamples * (ncols_x / 128) * ncols * 144;
    *dst_len = (size_t)p.nsamples_y * p.stride_sample_dst;
}

void cfo_mmq_case(uint32_t ty, uint32_t ncols_x, uint32_t nrows, uint32_t ncols, uint32_t nch, uint32_t ratio,
                  uint32_t nsamples, uint64_t seed, cfo_mmq *p, uint8_t *x, uint8_t *y) {
    uint64_t rng = seed;
    size_t xb;
    mmq_case_params(ty, ncols_x, nrows, ncols, nch, ratio, nsamples, p, &xb);
    cfo_random_blocks(ty, xb, &rng, x);
    size_t per = (size_t)ncols_x * ncols;
    float *acts = (float *)malloc(sizeof(float) * per);
    for (size_t c = 0; c < (size_t)nch * nsamples; c++) {
        for (size_t i = 0; i < per; i++) acts[i] = cfo_rng_unit(&rng) * 2.0f;
        cfo_quantize_mmq(ty, acts, ncols_x, ncols, y + c * (ncols_x / 128) * ncols * 144);
    }
    free(acts);
}

/* ---- src/ptx/ggml_ref.rs:169-446 (f64 second opinion, MMVQ options: half_mul on, min by
 * the q8_1 float sum only for the types that always take it) ---- */
double cfo_dot_ref_f64(uint32_t ty, const uint8_t *row, size_t nblocks, const uint8_t *y, double *abs_sum) {
    double total = 0, ab = 0;
    size_t bb = cfo_block_bytes(ty), per = (ty == CFO_Q4_K || ty == CFO_Q6_K) ? 8 : 1;
    for (size_t bi = 0; bi < nblocks; bi++) {
        const uint8_t *wb = row + bi * bb;
        double s[256], m[256];
        int32_t q[256];
        if (ty == CFO_Q8_0) {
            double d = h2f(wb);
            for (int j = 0; j < 32; j++) s[j] = d, q[j] = (int8_t)wb[2 + j], m[j] = 0;
        } else if (ty == CFO_Q4_K) {
            double d = h2f(wb), dmin = h2f(wb + 2);
            const uint8_t *sc = wb + 4, *ql = wb + 16;
            for (int jj = 0; jj < 4; jj++) {
                int32_t s1, m1, s2, m2;
                scale_min_k4(2 * jj, sc, &s1, &m1);
                scale_min_k4(2 * jj + 1, sc, &s2, &m2);
                for (int l = 0; l < 32; l++) {
                    s[64 * jj + l] = d * s1, q[64 * jj + l] = ql[32 * jj + l] & 0xF, m[64 * jj + l] = dmin * m1;
                    s[64 * jj + 32 + l] = d * s2, q[64 * jj + 32 + l] = ql[32 * jj + l] >> 4,
                                    m[64 * jj + 32 + l] = dmin * m2;
                }
            }
        } else if (ty == CFO_Q6_K) {
            double d = h2f(wb + 208);
            const uint8_t *ql = wb, *qh = wb + 128, *sc = wb + 192;
            for (int n = 0; n < 2; n++)
                for (int l = 0; l < 32; l++) {
                    const uint8_t *L = ql + 64 * n, *H = qh + 32 * n, *S = sc + 8 * n;
                    int is = l / 16, base = 128 * n;
                    q[base + l] = ((L[l] & 0xF) | ((H[l] & 3) << 4)) - 32;
                    q[base + l + 32] = ((L[l + 32] & 0xF) | (((H[l] >> 2) & 3) << 4)) - 32;
                    q[base + l + 64] = ((L[l] >> 4) | (((H[l] >> 4) & 3) << 4)) - 32;
                    q[base + l + 96] = ((L[l + 32] >> 4) | (((H[l] >> 6) & 3) << 4)) - 32;
                    s[base + l] = d * (int8_t)S[is];
                    s[base + l + 32] = d * (int8_t)S[is + 2];
                    s[base + l + 64] = d * (int8_t)S[is + 4];
                    s[base + l + 96] = d * (int8_t)S[is + 6];
                    m[base + l] = m[base + l + 32] = m[base + l + 64] = m[base + l + 96] = 0;
                }
        } else if (ty == CFO_Q4_0) {
            double d = h2f(wb);
            for (int h = 0; h < 2; h++)
                for (int j = 0; j < 16; j++)
                    s[16 * h + j] = d, q[16 * h + j] = h == 0 ? (wb[2 + j] & 0xF) : (wb[2 + j] >> 4),
                               m[16 * h + j] = 8.0 * d;
        } else {
            abort();
        }
        for (size_t g = 0; g < per; g++) {
            const uint8_t *yb = y + (bi * per + g) * 36;
            double d8 = h2f(yb);
            double acc = 0, macc = 0;
            int by_sum = ty == CFO_Q4_0; /* ggml_ref.rs:86-88 */
            for (int i = 0; i < 32; i++) {
                size_t e = 32 * g + i;
                double u = (int8_t)yb[4 + i];
                double term = s[e] * (double)q[e] * u * d8;
                acc += term;
                ab += fabs(term);
                if (!by_sum) {
                    macc += m[e] * u * d8;
                    ab += fabs(m[e] * u * d8);
                }
            }
            total += acc - macc;
            if (by_sum) {
                double s8 = h2f(yb + 2);
                total -= m[32 * g] * s8;
                ab += fabs(m[32 * g] * s8);
            }
        }
    }
    if (abs_sum) *abs_sum = ab;
    return total;
}

/* ---- crates/cublas_shim/src/plan.rs:160-215 ---- */
static int dtype_ok(int t) { return t == 0 || t == 2 || t == 14; }
int cfo_gemm_validate(int transa, int transb, int m, int n, int k, int lda, int ldb, int ldc, int a_type,
                      int b_type, int c_type, int compute_type) {
    if (transa < 0 || transa > 2 || transb < 0 || transb > 2) return 7;
    int ta = transa != 0, tb = transb != 0;
    if (m < 0 || n < 0 || k < 0) return 7;
    int rows_a = ta ? k : m, rows_b = tb ? n : k;
    if (lda < (rows_a > 1 ? rows_a : 1) || ldb < (rows_b > 1 ? rows_b : 1) || ldc < (m > 1 ? m : 1)) return 7;
    if (!dtype_ok(a_type) || !dtype_ok(b_type) || !dtype_ok(c_type)) return 15;
    int scalar; /* 0 f16, 1 f32 */
    switch (compute_type) {
    case 64: case 65: case 2: scalar = 0; break;
    case 68: case 69: case 74: case 75: case 77: case 0: scalar = 1; break;
    default: return 15;
    }
    if (a_type != b_type) return 15;
    int ok = (a_type == 0 && c_type == 0) || (a_type == 2 && (c_type == 2 || c_type == 0)) ||
             (a_type == 14 && (c_type == 14 || c_type == 0));
    if (!ok) return 15;
    if (scalar == 0 && (a_type != 2 || c_type != 2)) return 15;
    return 0;
}

static float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static uint16_t f32_to_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7fffffff) > 0x7f800000) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fff + ((u >> 16) & 1);
    return (uint16_t)(u >> 16);
}
static float dec(int t, const void *p, size_t i) {
    if (t == 0) return ((const float *)p)[i];
    if (t == 2) return cfo_f16_to_f32(((const uint16_t *)p)[i]);
    return bf16_to_f32(((const uint16_t *)p)[i]);
}
static void enc(int t, void *p, size_t i, float v) {
    if (t == 0)
        ((float *)p)[i] = v;
    else if (t == 2)
        ((uint16_t *)p)[i] = cfo_f32_to_f16(v);
    else
        ((uint16_t *)p)[i] = f32_to_bf16(v);
}

/* ---- plan.rs:344-362 ---- */
void cfo_reference_gemm(int transa, int transb, int m, int n, int k, float alpha, const void *a, int a_type,
                        int lda, const void *b, int ldb, float beta, void *c, int c_type, int ldc) {
    int ta = transa != 0, tb = transb != 0;
    for (int j = 0; j < n; j++)
        for (int i = 0; i < m; i++) {
            float acc = 0.0f;
            for (int l = 0; l < k; l++) {
                size_t ai = ta ? (size_t)l + (size_t)i * lda : (size_t)i + (size_t)l * lda;
                size_t bi = tb ? (size_t)j + (size_t)l * ldb : (size_t)l + (size_t)j * ldb;
                acc += dec(a_type, a, ai) * dec(a_type, b, bi);
            }
            size_t ci = (size_t)i + (size_t)j * ldc;
            float prior = beta == 0.0f ? 0.0f : beta * dec(c_type, c, ci);
            enc(c_type, c, ci, alpha * acc + prior);
        }
}

/* ---- tests/gpu/ggml_rms_norm.rs:43-55 (sequential f32 sum, sqrt then reciprocal), with the
 * fused weight multiply of examples/rmsnorm.cu:25-29 when w is given ---- */
void cfo_rms_norm(const float *x, const float *w, float *dst, size_t rows, size_t ncols, float eps) {
    for (size_t r = 0; r < rows; r++) {
        const float *s = x + r * ncols;
        float acc = 0.0f;
        for (size_t i = 0; i < ncols; i++) acc += s[i] * s[i];
        float mean_sq = acc / (float)ncols;
        float inv = 1.0f / sqrtf(mean_sq + eps);
        for (size_t i = 0; i < ncols; i++) dst[r * ncols + i] = w ? (s[i] * inv) * w[i] : s[i] * inv;
    }
}

/* ---- NeoX rope: the rotate-half pairing (i, i + n_dims/2) with the angle schedule of
 * tests/gpu/ggml_rope.rs:38-53 (theta = pos * theta_scale^i, theta_scale = base^(-2/n_dims)) and
 * the yarn scaling with ext_factor 0: cos/sin multiplied by attn_factor, theta by freq_scale,
 * theta divided by the optional frequency factor of pair i ---- */
void cfo_rope_neox(const float *x, float *dst, size_t ne0, size_t ne1, size_t nch, size_t n_dims,
                   const int32_t *pos, float freq_base, float freq_scale, float attn_factor, const float *ff) {
    float theta_scale = powf(freq_base, -2.0f / (float)n_dims);
    for (size_t c = 0; c < nch; c++)
        for (size_t h = 0; h < ne1; h++) {
            const float *s = x + (c * ne1 + h) * ne0;
            float *o = dst + (c * ne1 + h) * ne0;
            for (size_t i = 0; i < n_dims / 2; i++) {
                float theta = (float)pos[c] * powf(theta_scale, (float)i);
                if (ff) theta = theta / ff[i];
                theta = freq_scale * theta;
                float cs = cosf(theta) * attn_factor, sn = sinf(theta) * attn_factor;
                float x0 = s[i], x1 = s[i + n_dims / 2];
                o[i] = x0 * cs - x1 * sn;
                o[i + n_dims / 2] = x0 * sn + x1 * cs;
            }
            for (size_t i = n_dims; i < ne0; i++) o[i] = s[i];
        }
}

/* ---- tests/gpu/soft_max_generic.rs:73-92, plus the ALiBi slope (max_bias > 0) and the
 * attention-sink logit of ggml's soft_max params ---- */
void cfo_soft_max(const float *x, const float *mask, const float *sinks, float *dst, size_t ncols, size_t ne01,
                  size_t nheads, size_t rows, float scale, float max_bias) {
    uint32_t n_head_log2 = 1;
    while (n_head_log2 * 2 <= nheads) n_head_log2 *= 2;
    float m0 = powf(2.0f, -max_bias / (float)n_head_log2);
    float m1 = powf(2.0f, -(max_bias / 2.0f) / (float)n_head_log2);
    float *v = (float *)malloc(sizeof(float) * ncols);
    for (size_t r = 0; r < rows; r++) {
        size_t h = (r / ne01) % nheads;
        float slope = 1.0f;
        if (max_bias > 0.0f)
            slope = h < n_head_log2 ? powf(m0, (float)(h + 1)) : powf(m1, (float)(2 * (h - n_head_log2) + 1));
        const float *s = x + r * ncols;
        const float *mk = mask ? mask + (r % ne01) * ncols : NULL;
        float maxv = -INFINITY;
        for (size_t i = 0; i < ncols; i++) {
            v[i] = s[i] * scale + (mk ? slope * mk[i] : 0.0f);
            maxv = fmax_nan(maxv, v[i]);
        }
        if (sinks) maxv = fmax_nan(maxv, sinks[h]);
        float sum = 0.0f;
        for (size_t i = 0; i < ncols; i++) {
            dst[r * ncols + i] = expf(v[i] - maxv);
            sum += dst[r * ncols + i];
        }
        if (sinks) sum += expf(sinks[h] - maxv);
        for (size_t i = 0; i < ncols; i++) dst[r * ncols + i] /= sum;
    }
    free(v);
}

/* ---- src/subst/probe.rs:421-489: FlashAttention case (xorshift64* draws in the reference's
 * order: Q, K, V, then the mask biases) and the exact f64 softmax attention ---- */
void cfo_fattn_case(uint32_t d, uint32_t nq, uint32_t nh, uint32_t nh_kv, uint32_t nkv, uint32_t ns, int causal,
                    uint64_t seed, float *q, uint16_t *k, uint16_t *v, uint16_t *mask) {
    uint64_t rng = seed;
    for (size_t i = 0; i < (size_t)d * nq * nh * ns; i++) q[i] = cfo_rng_unit(&rng);
    for (size_t i = 0; i < (size_t)d * nkv * nh_kv * ns; i++) k[i] = cfo_f32_to_f16(cfo_rng_unit(&rng));
    for (size_t i = 0; i < (size_t)d * nkv * nh_kv * ns; i++) v[i] = cfo_f32_to_f16(cfo_rng_unit(&rng));
    if (!causal || !mask) return;
    size_t nq_pad = (nq + 15) / 16 * 16;
    for (size_t s = 0; s < ns; s++)
        for (size_t i = 0; i < nq_pad; i++)
            for (size_t j = 0; j < nkv; j++) {
                /* the last third of the keys is padding; query i sees keys up to nvis - nq + i */
                size_t nvis = nkv - nkv / 3;
                int visible = j < nvis && j + nq <= nvis + i;
                mask[(s * nq_pad + i) * nkv + j] = visible ? cfo_f32_to_f16(cfo_rng_unit(&rng) * 0.5f) : 0xfc00;
            }
}

void cfo_fattn_reference(uint32_t d, uint32_t nq, uint32_t nh, uint32_t nh_kv, uint32_t nkv, uint32_t ns,
                         const float *q, const uint16_t *k, const uint16_t *v, const uint16_t *mask, float scale,
                         float *dst) {
    size_t gqa = nh / nh_kv, nq_pad = (nq + 15) / 16 * 16;
    double *sc = (double *)malloc(sizeof(double) * nkv);
    for (size_t s = 0; s < ns; s++)
        for (size_t h = 0; h < nh; h++) {
            size_t kh = h / gqa;
            for (size_t i = 0; i < nq; i++) {
                const float *qrow = q + ((s * nh + h) * nq + i) * d;
                double mx = -INFINITY;
                for (size_t j = 0; j < nkv; j++) {
                    const uint16_t *krow = k + ((s * nh_kv + kh) * nkv + j) * d;
                    double acc = 0;
                    for (size_t t = 0; t < d; t++) acc += (double)(qrow[t] * scale) * (double)cfo_f16_to_f32(krow[t]);
                    if (mask) acc += (double)cfo_f16_to_f32(mask[(s * nq_pad + i) * nkv + j]);
                    sc[j] = acc;
                    if (acc > mx) mx = acc;
                }
                double l = 0;
                for (size_t j = 0; j < nkv; j++) {
                    sc[j] = exp(sc[j] - mx);
                    l += sc[j];
                }
                for (size_t t = 0; t < d; t++) {
                    double o = 0;
                    for (size_t j = 0; j < nkv; j++) o += sc[j] * (double)cfo_f16_to_f32(v[((s * nh_kv + kh) * nkv + j) * d + t]);
                    dst[((s * nq + i) * nh + h) * d + t] = (float)(o / l);
                }
            }
        }
    free(sc);
}
