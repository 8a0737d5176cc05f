/*
 * cpu_baseline.c -- the CPU evaluation of the decode GEMV that bench.py times beside the GPU
 * (TEST/BENCH INFRASTRUCTURE ONLY).
 *
 * It is the reference's decode-fast host model (src/subst/refs.rs:435-497 with one warp, one
 * accumulator and whole-group lanes, the default shape of src/subst/mod.rs:353-356 narrowed to
 * one row) run row-parallel over POSIX host threads, plus quantize_q8_1 of the activation
 * columns (refs.rs:117-147).  Row results are bitwise those of cfo_mmvq_fast(warps=1, unroll=1,
 * wide=1) for each column.
 */
#include "cfi_oracle.h"

#include <pthread.h>
#include <unistd.h>
#include <stdlib.h>
#include <string.h>

/* Per row r and column c: 32 lanes, lane g takes groups g, g+32/tpb*..., one accumulator,
 * butterfly, lane 0.  W rows are contiguous (stride ncols_x/qk blocks); y columns are
 * ncols_x/32 q8_1 blocks apart; dst is column-major with stride rows. */
static float row_dot(uint32_t ty, const uint8_t *wrow, size_t nblk, size_t qk, size_t bb, const uint8_t *ycol) {
    size_t tpb = qk / 32, step = 32 / tpb;
    float lanes[32];
    for (size_t lane = 0; lane < 32; lane++) {
        size_t kqs = lane % tpb;
        float acc = 0.0f;
        for (size_t k = lane / tpb; k < nblk; k += step)
            acc = cfo_vec_dot_wide(ty, wrow + k * bb, ycol + (k * tpb + kqs) * 36, kqs, acc);
        lanes[lane] = acc;
    }
    static const int offs[5] = {16, 8, 4, 2, 1};
    for (int o = 0; o < 5; o++) {
        float old[32];
        memcpy(old, lanes, sizeof old);
        for (int l = 0; l < 32; l++) lanes[l] = old[l] + old[l ^ offs[o]];
    }
    return lanes[0];
}

typedef struct {
    uint32_t ty;
    const uint8_t *w;
    size_t rows, ncols_x, ncols_dst, qk, bb, nblk, yb, r0, r1;
    const uint8_t *yq;
    float *dst;
} job_t;

static void *rows_job(void *arg) {
    job_t *j = (job_t *)arg;
    for (size_t r = j->r0; r < j->r1; r++)
        for (size_t c = 0; c < j->ncols_dst; c++)
            j->dst[c * j->rows + r] = row_dot(j->ty, j->w + r * j->nblk * j->bb, j->nblk, j->qk, j->bb, j->yq + c * j->yb);
    return NULL;
}

/* One decode step on the host: quantize ncols_dst activation columns (ncols_x floats each) into
 * yq (caller buffer of ncols_dst*ncols_x/32*36 bytes), then y = W * x for rows [0, rows), split
 * into `threads` contiguous row ranges (threads <= 0: every online core).  Returns the number of
 * threads used. */
int cfo_cpu_decode_step(uint32_t ty, const uint8_t *w, size_t rows, size_t ncols_x, const float *x,
                        size_t ncols_dst, uint8_t *yq, float *dst, int threads) {
    size_t qk = ty == CFO_Q8_0 ? 32 : 256, bb = cfo_block_bytes(ty), nblk = ncols_x / qk;
    size_t yb = ncols_x / 32 * 36;
    if (threads <= 0) threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (threads < 1) threads = 1;
    if ((size_t)threads > rows) threads = (int)rows;
    for (size_t c = 0; c < ncols_dst; c++) cfo_quantize_q8_1(x + c * ncols_x, ncols_x, yq + c * yb);
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    job_t *jobs = (job_t *)malloc(sizeof(job_t) * (size_t)threads);
    for (int t = 0; t < threads; t++) {
        jobs[t] = (job_t){ty, w, rows, ncols_x, ncols_dst, qk, bb, nblk, yb,
                          rows * (size_t)t / (size_t)threads, rows * (size_t)(t + 1) / (size_t)threads, yq, dst};
        if (t > 0) pthread_create(&tid[t], NULL, rows_job, &jobs[t]);
    }
    rows_job(&jobs[0]);
    for (int t = 1; t < threads; t++) pthread_join(tid[t], NULL);
    free(tid);
    free(jobs);
    return threads;
}
