// subst_host.hpp -- C++ model of the substitution API (internal to libcfi_b200.so).
//
// Mirrors cuda-for-intel's src/subst/mod.rs (Switch, demangle, the kernel table, layouts,
// Plan geometry) and src/cuda/subst_hook.rs (native registry, router, fallback, fixup skipping),
// re-designed for the real CUDA driver on B200: the "translated" kernel of the reference is the
// caller's own stock CUfunction, and the native kernels are precompiled sm_100a code.
#pragma once
#include <stdint.h>

#include <map>
#include <mutex>
#include <optional>
#include <string>
#include <vector>

#include "../../include/cfi_subst.h"

namespace cfi {

// ---- environment switch (mod.rs:57-113) ----
struct Switch {
    bool all = false, aut = false;
    std::vector<std::string> items, denied;
    static Switch parse(const std::string& text);
    static Switch from_env();
    bool allows(const std::string& family, const char* ty) const;
    bool denies(const std::string& family, const char* ty) const;
    bool is_none() const { return !all && !aut && items.empty(); }
};

// ---- Itanium names (mod.rs:115-171) ----
struct TArg {
    enum Kind { Int = 0, Enum = 1, Type = 2 } kind;
    int64_t value;
    std::string name;  // enum or type name
};
struct Mangled {
    std::string base;
    std::vector<TArg> targs;
};
std::optional<Mangled> demangle(const std::string& name);

// ---- parameter layouts ----
using Layout = std::vector<cfi_param>;
uint64_t layout_hash(const cfi_param* p, int n);
size_t param_bytes(const cfi_param& p);
std::string layout_debug(const cfi_param* p, int n);

const char* type_name(uint32_t ty);
Layout layout_for(int kernel, uint32_t aux);
int nparams_for(int kernel, uint32_t aux);

// ---- plan helpers (mod.rs:323-387, 468-565) ----
std::optional<cfi_fast> mmvq_fast_from(const char* text, uint32_t ty);
bool mmvq_fast_is_opt_out(const std::string& t);
cfi_fast mmvq_fast_default(uint32_t ty);
std::string mmvq_key(uint32_t ty, uint32_t ncols, const cfi_fast* fast, uint32_t nwarps);
uint32_t ggml_mmvq_nwarps(uint32_t ncols);

int decide(const std::string& name, const cfi_param* params, int nparams, const Switch& sw, cfi_plan* out,
           std::string* why);

// Native geometry and trailing words of a launch.  `args` are the caller's kernelParams (may be
// null when only `vals` are known, e.g. for the pure-host C API).  Returns false when the launch
// is not one the native kernel serves.
struct NativeLaunch {
    const void* fn = nullptr;
    uint32_t grid[3] = {1, 1, 1}, block[3] = {1, 1, 1};
    size_t smem = 0;
    std::vector<uint32_t> extra;  // trailing u32 words after the stock parameters
    int nparams = 0;              // stock parameters forwarded
    bool own_launch = false;      // tcgen05 GEMM: launched by its own code (see gemm_launch)
    bool pdl = false;             // launch with programmatic stream serialization
};
bool map_launch(const cfi_plan& plan, const uint32_t grid[3], const uint32_t block[3], const uint64_t* vals, int nvals,
                void** args, NativeLaunch* out);

// Reads one u64 per parameter (first min(size, 8) bytes), as subst_hook.rs:199-209 does.
std::vector<uint64_t> arg_values(const cfi_plan& plan, void** args);

// Native kernel handle for a plan, or an error (the plan then falls back to the stock kernel).
const void* native_kernel(const cfi_plan& plan, std::string* why);

// probe.cpp: first-use validation on the device (probe.rs:350-403).
int probe_validate(const cfi_plan& plan, void* stream, std::string* why);

// Launch of the native mmq (k_mmq_sm100.cu), with its own grid and launch attributes.
int mmq_launch(const cfi_plan& plan, void** args, void* stream);

// Native FlashAttention (k_fattn_sm100.cu): the launch words it serves (plan.aux = head size) and
// its own launch.
bool fattn_geometry_ok(uint32_t d, const uint64_t* vals, int n);
int fattn_launch(const cfi_plan& plan, void** args, void* stream);
int fattn_threads();
int fattn_tile();

}  // namespace cfi
