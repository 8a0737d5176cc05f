// cfi_common.cuh -- device helpers shared by the sm_100a kernels of the substitution path.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <utility>

#define CFI_DEV __device__ __forceinline__

// ---- host side: state that belongs to one device ----
// Kernel attributes (cudaFuncSetAttribute) and the addresses of __device__ symbols
// (cudaGetSymbolAddress) are per device, so one process driving several GPUs sets and looks them
// up once for each device, keyed by the current device's index.
constexpr int CFI_MAX_DEVICES = 64;

// Index of the current device, or -1 when it cannot be queried or is past CFI_MAX_DEVICES (the
// callers then redo the per-device work on every call instead of caching it).
inline int cfi_device_index() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return d >= 0 && d < CFI_MAX_DEVICES ? d : -1;
}

struct CfiPerDeviceOnce {
    std::once_flag f[CFI_MAX_DEVICES];
};

// Runs fn() once for each device it is called with current.
template <class F> void cfi_once_per_device(CfiPerDeviceOnce& o, F&& fn) {
    const int d = cfi_device_index();
    if (d < 0)
        fn();
    else
        std::call_once(o.f[d], std::forward<F>(fn));
}

// Device address of the __device__ symbol `sym` on the current device (nullptr if the lookup
// fails), looked up once per device.
template <class T> struct CfiSymbolPtr {
    T* ptr[CFI_MAX_DEVICES] = {};
    CfiPerDeviceOnce once;
    T* get(const T& sym) {
        const int d = cfi_device_index();
        T* p = nullptr;
        auto look = [&p, &sym] {
            if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), sym) != cudaSuccess) {
                cudaGetLastError();
                p = nullptr;
            }
        };
        if (d < 0) {
            look();
            return p;
        }
        std::call_once(once.f[d], [&] {
            look();
            ptr[d] = p;
        });
        return ptr[d];
    }
};

// ggml block sizes (ggml-common.h layouts; see the block structs below).
constexpr int QK8_0 = 32, QK8_1 = 32, QK4_0 = 32, QK_K = 256;
constexpr int Q8_0_BYTES = 34, Q8_1_BYTES = 36, Q4_0_BYTES = 18, Q5_0_BYTES = 22, Q4_K_BYTES = 144, Q5_K_BYTES = 176,
              Q6_K_BYTES = 210;
constexpr int MMQ_BLOCK_BYTES = 144;  // block_q8_1_mmq: 4 scales (16 B) + 128 int8

// ggml type ids.
constexpr uint32_t T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14;

// ggml's fastdiv triple {mp, L, d}: n / d == (umulhi(n, mp) + n) >> L.
CFI_DEV uint32_t fastdiv(uint32_t n, uint3 v) { return (__umulhi(n, v.x) + n) >> v.y; }
CFI_DEV uint32_t fastmodulo(uint32_t n, uint3 v) { return n - fastdiv(n, v) * v.z; }

CFI_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
CFI_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

CFI_DEV float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }
CFI_DEV uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

CFI_DEV int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Bounded waits that give up record a code in a device error word instead of hanging; the
// host reads it back after a synchronize (first code wins).
CFI_DEV void cfi_set_error(unsigned int *err, unsigned int code) {
    if (err) atomicCAS(err, 0u, code);
}
