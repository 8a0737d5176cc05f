// tc_epilogue.cuh -- drains a 128-row fp32 accumulator tile from tensor memory to a column-major
// matrix with 16-byte stores (shared by the tcgen05 GEMM kernels).
//
// tcgen05.ld 32x32b gives thread l of a warp row l of its 32-lane TMEM quadrant and one register
// per column, which as direct global stores is one 4-byte store per value.  Instead each warp
// writes a 32 x 32 chunk into shared memory column by column (conflict-free: lanes write
// consecutive words) and reads it back as float4 runs of 4 rows (8 lanes cover one column's 32
// rows), so a warp stores a chunk with 8 coalesced 16-byte stores per lane instead of 32.
#pragma once
#include "cfi_common.cuh"
#include "sm100_ptx.cuh"

namespace sm100 {

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

}  // namespace sm100
