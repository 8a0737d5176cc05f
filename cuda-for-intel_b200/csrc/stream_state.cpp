// stream_state.cpp -- scratch memory of the library's kernels, one set per (device, stream).
//
// Kernels that combine per-CTA partials (the split attention and multi-CTA argmax of the decode
// glue, the GEMVs that run a fused decode step in their last CTA), the split-K partial tiles of the
// tensor-core GEMMs and the fp16 activation copy of mul_mat_q need device memory beyond their
// inputs and outputs.  Calls on different streams may run at the same time, so each (device,
// stream) gets its own:
//   * glue slots (cfi_glue_slot): fixed-size partial buffers and counters, taken from a per-device
//     pool.  The first call on a device outside stream capture fills the pool with
//     CFI_GLUE_SLOTS_INITIAL slots, so a stream first seen while it is being captured (as a
//     capture side stream is) still gets a slot of its own; the pool grows outside capture only.
//   * buffers (cfi_stream_buffer): grown on demand outside capture, kept (not freed) when replaced,
//     since graphs captured earlier may still name them.
// A graph keeps the slot and buffers of the stream it was captured on.
#include "cfi_kernels.h"

#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <tuple>
#include <vector>

namespace {

constexpr int CFI_GLUE_SLOTS_INITIAL = 4;

std::mutex g_mu;

bool capturing(cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &st) != cudaSuccess) {
        cudaGetLastError();
        return true;  // unknown (e.g. the legacy stream during another stream's capture): do not allocate
    }
    return st != cudaStreamCaptureStatusNone;
}

// ---- glue slots ----
struct SlotPool {
    std::vector<CfiGlueSlot> slots;
    std::vector<bool> used;
    std::map<cudaStream_t, int> owner;
};
std::map<int, SlotPool> g_pools;

bool alloc_slot(CfiGlueSlot* out) {
    // counters first (zeroed once; every kernel leaves them at zero), then the partials
    const size_t counters = 4u * (1u + CFI_ATT_MAX_HEADS + 4u);
    const size_t amax = (size_t)CFI_AMAX_CTAS * 8u;
    const size_t att = (size_t)CFI_ATT_MAX_HEADS * CFI_ATT_MAX_SPLIT * (2 + 128) * 4u;
    const size_t off_amax = (counters + 255) & ~(size_t)255, off_att = (off_amax + amax + 255) & ~(size_t)255;
    uint8_t* p = nullptr;
    if (cudaMalloc(reinterpret_cast<void**>(&p), off_att + att) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (cudaMemset(p, 0, counters) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return false;
    }
    unsigned int* c = reinterpret_cast<unsigned int*>(p);
    out->amax_count = c;
    out->att_count = c + 1;
    out->epi_count = c + 1 + CFI_ATT_MAX_HEADS;
    out->amax_val = reinterpret_cast<float*>(p + off_amax);
    out->amax_idx = reinterpret_cast<int*>(p + off_amax + (size_t)CFI_AMAX_CTAS * 4u);
    out->att_part = reinterpret_cast<float*>(p + off_att);
    return true;
}

// ---- buffers ----
struct Buf {
    void* p = nullptr;
    size_t cap = 0;
};
std::map<std::tuple<int, cudaStream_t, int>, Buf> g_bufs;
std::vector<void*> g_retired;

}  // namespace

int cfi_glue_slot(cudaStream_t stream, CfiGlueSlot* out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return (int)cudaErrorNoDevice;
    }
    std::lock_guard<std::mutex> g(g_mu);
    SlotPool& pool = g_pools[dev];
    auto it = pool.owner.find(stream);
    if (it != pool.owner.end()) {
        *out = pool.slots[it->second];
        return 0;
    }
    const bool cap = capturing(stream);
    if (pool.slots.empty() && !cap) {
        for (int i = 0; i < CFI_GLUE_SLOTS_INITIAL; i++) {
            CfiGlueSlot sl;
            if (!alloc_slot(&sl)) return (int)cudaErrorMemoryAllocation;
            pool.slots.push_back(sl);
            pool.used.push_back(false);
        }
    }
    int idx = -1;
    for (size_t i = 0; i < pool.slots.size() && idx < 0; i++)
        if (!pool.used[i]) idx = (int)i;
    if (idx < 0) {
        if (cap) return (int)cudaErrorStreamCaptureUnsupported;  // no free slot, and no allocation under capture
        CfiGlueSlot sl;
        if (!alloc_slot(&sl)) return (int)cudaErrorMemoryAllocation;
        pool.slots.push_back(sl);
        pool.used.push_back(false);
        idx = (int)pool.slots.size() - 1;
    }
    pool.used[idx] = true;
    pool.owner[stream] = idx;
    *out = pool.slots[idx];
    return 0;
}

void* cfi_stream_buffer(int kind, size_t bytes, cudaStream_t stream, int* err) {
    int dev = 0;
    *err = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        *err = (int)cudaErrorNoDevice;
        return nullptr;
    }
    std::lock_guard<std::mutex> g(g_mu);
    Buf& b = g_bufs[std::make_tuple(dev, stream, kind)];
    if (b.cap < bytes) {
        if (capturing(stream)) {
            *err = (int)cudaErrorStreamCaptureUnsupported;
            return nullptr;
        }
        if (b.p) g_retired.push_back(b.p);
        b.p = nullptr;
        b.cap = 0;
        const size_t want = bytes + bytes / 4;
        if (cudaMalloc(&b.p, want) != cudaSuccess) {
            cudaGetLastError();
            *err = (int)cudaErrorMemoryAllocation;
            return nullptr;
        }
        if (kind == CFI_BUF_COUNTERS && cudaMemset(b.p, 0, want) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(b.p);
            b.p = nullptr;
            *err = (int)cudaErrorMemoryAllocation;
            return nullptr;
        }
        b.cap = want;
    }
    return b.p;
}
