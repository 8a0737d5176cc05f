// k_peer.cu -- peer buffers over NVLink (CUDA IPC), the check of a rank's peer set, and the
// group barrier: the host side of the all-gather that the skinny mul_mat_q performs with plain
// stores into every rank's mapped output (cfi_mmq_skinny_group_peers).
//
// Protocol, per product launch of every rank: the launch stores each output value into its own
// and every peer's copy of the output; every CTA then makes its stores visible at system scope
// and adds its share of the launch's signal (CFI_PEER_UNIT in all) to this rank's slot in each
// peer's buffer, and CTA 0 waits until each peer's slot here has grown by one unit per launch
// so far before the launch ends, so the work after it sees every rank's rows (peer_sync.cuh).
// cfi_peer_barrier is the same signal and wait alone.  No counterpart in cuda-for-intel (single
// GPU).
#include <string.h>

#include <algorithm>

#include "../../include/cfi_peer.h"
#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "peer_sync.cuh"
#include "sm100_ptx.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == CFI_PEER_HANDLE_BYTES, "IPC handle size");

namespace {
using namespace sm100;

// Ranks can reach a step seconds apart (a peer still building its state, a first-use probe), so
// the wait for a peer is bounded more loosely than the in-kernel pipeline waits (CFI_PEER_WAIT_MS
// sets another bound).
constexpr uint64_t PEER_WAIT_LIMIT_NS = 10000000000ull;  // 10 s

// One thread, after the kernels queued before it (with programmatic launch the kernels after
// this one can be resident before it ends; the wait counts are read after the previous
// launch's update).
__global__ void __launch_bounds__(32, 1) cfi_peer_barrier_kernel(const __grid_constant__ CfiPeerDev p, unsigned int* err) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) {
        peer_signal_cta(p, 1, true);
        peer_wait_all(p, err);
    }
}

// All-gather of one slice per rank: grid-stride 16-byte copies of this rank's slice into its
// place in every rank's buffer (ranks in turn from this one), then the per-CTA signal and CTA 0's
// wait (peer_sync.cuh).  dst: this rank's buffer at the gathered range; delta[r] maps it to rank r's.
__global__ void __launch_bounds__(256) cfi_peer_all_gather_kernel(const uint4* __restrict__ src, uint4* dst, uint32_t n16,
                                                                   const __grid_constant__ CfiPeerDev p, unsigned int* err) {
    pdl_launch_dependents();
    pdl_wait();
    uint4* mine = dst + (size_t)p.rank * n16;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += gridDim.x * blockDim.x) {
        const uint4 v = src[i];
        for (int k = 0; k < p.world; k++) {
            const int r = p.rank + k < p.world ? p.rank + k : p.rank + k - p.world;
            reinterpret_cast<uint4*>(reinterpret_cast<char*>(mine + i) + p.delta[r])[0] = v;
        }
    }
    if (p.world > 1) {
        __syncthreads();
        if (threadIdx.x == 0) {
            const bool first = blockIdx.x == 0;
            peer_signal_cta(p, gridDim.x, first);
            if (first) peer_wait_all(p, err);
        }
    }
}

}  // namespace

int cfi_peer_dev(const CfiPeerSet* in, CfiPeerDev* out) {
    static_assert(CFI_MAX_RANKS == CFI_PEER_MAX_RANKS, "ranks of a group");
    if (!in || !out || in->world < 1 || in->world > CFI_PEER_MAX_RANKS || in->rank < 0 || in->rank >= in->world)
        return (int)cudaErrorInvalidValue;
    *out = CfiPeerDev{};
    out->rank = in->rank;
    out->world = in->world;
    for (int r = 0; r < in->world; r++) {
        if (r != in->rank && !in->sig_remote[r]) return (int)cudaErrorInvalidValue;
        out->delta[r] = r == in->rank ? 0 : in->delta[r];
        out->sig_remote[r] = in->sig_remote[r];
    }
    if (in->world > 1 && (!in->sig_local || !in->expect)) return (int)cudaErrorInvalidValue;
    out->sig_local = in->sig_local;
    out->expect = in->expect;
    const char* el = getenv("CFI_PEER_WAIT_MS");
    out->limit_ns = el && atoll(el) > 0 ? (unsigned long long)atoll(el) * 1000000ull : PEER_WAIT_LIMIT_NS;
    return 0;
}

extern "C" int cfi_peer_alloc(size_t bytes, void** ptr, void* handle) {
    if (!ptr || !handle || bytes == 0) return (int)cudaErrorInvalidValue;
    *ptr = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return (int)e;
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return (int)e;
    }
    memcpy(handle, &h, sizeof h);
    *ptr = p;
    return 0;
}

extern "C" int cfi_peer_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return (int)cudaErrorInvalidValue;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    *ptr = nullptr;
    return (int)cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

extern "C" int cfi_peer_close(void* ptr) { return ptr ? (int)cudaIpcCloseMemHandle(ptr) : (int)cudaErrorInvalidValue; }

extern "C" int cfi_peer_free(void* ptr) { return ptr ? (int)cudaFree(ptr) : (int)cudaErrorInvalidValue; }

extern "C" int cfi_peer_barrier(const CfiPeerSet* peers, void* stream) {
    CfiPeerDev p;
    const int rc = cfi_peer_dev(peers, &p);
    if (rc) return rc;
    const char* ep = getenv("CFI_PDL");
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3(1, 1, 1);
    c.blockDim = dim3(32, 1, 1);
    c.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = at;
    c.numAttrs = ep && strcmp(ep, "0") == 0 ? 0 : 1;
    unsigned int* err = cfi_device_error_word();
    return (int)cudaLaunchKernelEx(&c, cfi_peer_barrier_kernel, p, err);
}

extern "C" int cfi_peer_all_gather(const void* src, size_t bytes, void* dst, const CfiPeerSet* peers, void* stream) {
    CfiPeerDev p;
    const int rc = cfi_peer_dev(peers, &p);
    if (rc) return rc;
    if (!src || !dst || (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15) || bytes % 16 ||
        bytes / 16 > 0xffffffffull)
        return (int)cudaErrorInvalidValue;
    if (bytes == 0) return 0;
    const uint32_t n16 = (uint32_t)(bytes / 16);
    const char* ep = getenv("CFI_PDL");
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3(std::min<uint32_t>(16u, std::max<uint32_t>(1u, (n16 + 4095) / 4096)), 1, 1);
    c.blockDim = dim3(256, 1, 1);
    c.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = at;
    c.numAttrs = ep && strcmp(ep, "0") == 0 ? 0 : 1;
    unsigned int* err = cfi_device_error_word();
    return (int)cudaLaunchKernelEx(&c, cfi_peer_all_gather_kernel, static_cast<const uint4*>(src), static_cast<uint4*>(dst),
                                   n16, p, err);
}
