// tc_epilogue.cuh -- drains a 128-row fp32 accumulator tile from tensor memory to a column-major
// matrix with 16-byte stores (shared by the tcgen05 GEMM kernels).
//
// tcgen05.ld 32x32b gives thread l of a warp row l of its 32-lane TMEM quadrant and one register
// per column, which as direct global stores is one 4-byte store per value.  Instead each warp
// writes a 32 x 32 chunk into shared memory column by column (conflict-free: lanes write
// consecutive words) and reads it back as float4 runs of 4 rows (8 lanes cover one column's 32
// rows), so a warp stores a chunk with 8 coalesced 16-byte stores per lane instead of 32.
//
// tmem_tile_tma_store: the same chunks handed to the TMA engine (cp.async.bulk.tensor store from
// shared memory, double-buffered per warp), so the warps never wait on global stores; the tensor
// map clips rows and columns outside the matrix.
#pragma once
#include <cuda.h>

#include "cfi_common.cuh"
#include "sm100_ptx.cuh"

namespace sm100 {

CFI_DEV void tma_store_4d(const CUtensorMap* map, const void* src, int x, int y, int z, int w) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
}
CFI_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N> CFI_DEV void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
template <int N> CFI_DEV void bulk_wait() { asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory"); }

// Warp `warp` of `nwarps` (4 or 8) epilogue warps: TMEM lane quadrant warp & 3 (tile rows
// 32 (warp & 3) .. + 31); with 8 warps the two warps of a quadrant take alternate 32-column chunks.
// `buf`: this warp's 32 x 32 fp32 staging area (4 KB, 16-byte aligned) in shared memory.
// store(col, row, float4 v): tile-relative column and first of 4 consecutive rows.
template <class Store>
CFI_DEV void tmem_tile_store(uint32_t tmem, int warp, int lane, int nwarps, uint32_t bn, float* buf, Store&& store) {
    const uint32_t q = (uint32_t)warp & 3u;
    const uint32_t first = nwarps == 8 ? ((uint32_t)warp >> 2) : 0u, step = nwarps == 8 ? 2u : 1u;
    for (uint32_t ci = first; ci * 32 < bn; ci += step) {
        const uint32_t cb = ci * 32;
        uint32_t v[32];
        tmem_ld32(tmem + ((q * 32u) << 16) + cb, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i++) buf[i * 32 + lane] = __uint_as_float(v[i]);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t cl = 4u * j + ((uint32_t)lane >> 3), rl = 4u * ((uint32_t)lane & 7u);
            const float4 f = *reinterpret_cast<const float4*>(buf + cl * 32 + rl);
            if (cb + cl < bn) store(cb + cl, q * 32 + rl, f);
        }
        __syncwarp();
    }
}

// As tmem_tile_store, for an fp32 matrix described by `map` (4-D: rows, columns, z, w; box 32 x 32
// x 1 x 1, no swizzle): chunk (cb) of warp quadrant q goes to (row0 + 32 q, col0 + cb, z, w).
// `buf`: this warp's 2 x 32 x 32 fp32 (8 KB, 128-byte aligned); `scale` maps each accumulator.
template <class Scale>
CFI_DEV void tmem_tile_tma_store(uint32_t tmem, int warp, int lane, int nwarps, uint32_t bn, float* buf,
                                 const CUtensorMap* map, int row0, int col0, int z, int w, Scale&& scale) {
    const uint32_t q = (uint32_t)warp & 3u;
    const uint32_t first = nwarps == 8 ? ((uint32_t)warp >> 2) : 0u, step = nwarps == 8 ? 2u : 1u;
    uint32_t k = 0;
    for (uint32_t ci = first; ci * 32 < bn; ci += step, k++) {
        const uint32_t cb = ci * 32;
        float* b = buf + (k & 1u) * 1024;
        if (k >= 2) {  // the store issued from this buffer two chunks ago has read it
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
        }
        uint32_t v[32];
        tmem_ld32(tmem + ((q * 32u) << 16) + cb, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i++) b[i * 32 + lane] = scale(__uint_as_float(v[i]));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_4d(map, b, row0 + (int)(q * 32u), col0 + (int)cb, z, w);
            bulk_commit();
        }
    }
    // the staging buffers must not be reused or released before the engine has read them; the
    // global writes themselves complete before the grid does
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
}

}  // namespace sm100
