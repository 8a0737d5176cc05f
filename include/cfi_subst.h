/*
 * cfi_subst.h -- C ABI of the B200-native kernel-substitution layer (libcfi_b200.so).
 *
 * A ggml-cuda kernel launch (cuLaunchKernel: function, grid, block, shared bytes, stream,
 * kernelParams) is matched by its Itanium-mangled name and parameter layout, and replaced by a
 * hand-written sm_100a kernel that takes the same kernelParams.  Every entry point returns an
 * error code; nothing aborts the caller.  Each declaration names the interface of cuda-for-intel
 * it replaces (paths inside that project).
 */
#ifndef CFI_SUBST_H
#define CFI_SUBST_H
#include <stddef.h>
#include <stdint.h>

#ifndef CFI_API
#define CFI_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- parameter layouts (replaces ptx::Param, src/ptx.rs:66-78) ---- */
enum cfi_param_kind {
    CFI_P_U8 = 0,
    CFI_P_U16 = 1,
    CFI_P_U32 = 2,
    CFI_P_F32 = 3,
    CFI_P_U64 = 4,
    CFI_P_PTR = 5,   /* GlobalPtr */
    CFI_P_WORDS = 6, /* by-value aggregate: a = words, b = align, c = trim (uint3 = {3, 4, 0}) */
    CFI_P_STAGED = 7 /* large aggregate passed through memory: a = bytes, b = align */
};
typedef struct cfi_param {
    int32_t kind;
    uint16_t a, b;
    uint8_t c;
} cfi_param;

/* ---- kernels the table knows (replaces subst::Kernel, src/subst/mod.rs:175-187) ---- */
enum cfi_kernel {
    CFI_K_MMVQ = 1,         /* mul_mat_vec_q<ty, ncols> */
    CFI_K_QUANTIZE_Q8_1 = 2,
    CFI_K_MMQ = 3,          /* mul_mat_q<ty, mmq_x, need_check>, non-MoE */
    CFI_K_MMQ_FIXUP = 4,    /* mul_mat_q_stream_k_fixup<ty, ...>: skipped after a native mmq */
    CFI_K_QUANTIZE_MMQ = 5, /* quantize_mmq_q8_1<layout> */
    CFI_K_RMS_NORM = 6,     /* rms_norm_f32<block, do_multiply, do_add> */
    CFI_K_RMS_NORM_PLAIN = 7, /* rms_norm_f32<block> (older iiilllf parameter list) */
    CFI_K_ROPE_NEOX = 8,    /* rope_neox<forward, has_ff, float> */
    CFI_K_SOFT_MAX = 9,     /* soft_max_f32<use_shared, ncols, block, T> */
    CFI_K_FATTN = 10,       /* flash_attn_ext_f16<D, D, ncols1, ncols2, nwarps, ntiles, false, false> */
    CFI_K_FATTN_FIXUP = 11  /* flash_attn_stream_k_fixup<D, ncols1, ncols2>: skipped after a native one */
};

/* Decode-fast shape of mmvq (replaces mmvq::Fast, src/subst/mmvq.rs:727-735). */
typedef struct cfi_fast {
    uint32_t rows, warps, unroll, wide;
} cfi_fast;

/* A substitution decision (replaces subst::Plan, src/subst/mod.rs:309-321). */
typedef struct cfi_plan {
    int32_t kernel;   /* enum cfi_kernel */
    uint32_t ty;      /* ggml type (mmvq, mmq, quantize_mmq layout) */
    uint32_t ncols;   /* mmvq ncols_dst */
    uint32_t nwarps;  /* CFI_SUBST_NWARPS override, 0 = none */
    uint32_t aux;     /* mmq_x of mul_mat_q; template flags of the row kernels */
    uint32_t has_fast;
    cfi_fast fast;
    uint64_t layout_hash;
    char key[64];     /* native module key (mod.rs:358-366) */
} cfi_plan;

enum { CFI_SUBSTITUTE = 0, CFI_MISMATCH = 1, CFI_NOT_APPLICABLE = 2 };

/* decide(name, params, switch) -> Decision (src/subst/mod.rs:397-466).  `switch_text` NULL reads
 * CFI_SUBST from the environment (unset = "auto").  On CFI_MISMATCH, `why` receives the reason. */
CFI_API int cfi_subst_decide(const char *mangled, const cfi_param *params, int nparams, const char *switch_text,
                     cfi_plan *out, char *why, size_t why_len);

/* Switch (src/subst/mod.rs:57-113): 1/0 answers for a switch text. */
CFI_API int cfi_switch_allows(const char *switch_text, const char *family, const char *ty);
CFI_API int cfi_switch_denies(const char *switch_text, const char *family, const char *ty);
CFI_API int cfi_switch_is_none(const char *switch_text);

/* demangle (src/subst/mod.rs:129-171): base name and template arguments.  kinds[i]: 0 int,
 * 1 enum literal (enum name in the '\n'-separated `names`), 2 type.  Returns the number of
 * template arguments, or -1 when the name has a form the parser does not handle. */
CFI_API int cfi_demangle(const char *mangled, char *base, size_t base_len, int64_t *values, int *kinds, char *names,
                 size_t names_len, int max_args);

/* FNV-1a layout hash over the debug rendering of the layout (src/subst/mod.rs:249-257). */
CFI_API uint64_t cfi_layout_hash(const cfi_param *params, int nparams);

/* CFI_MMVQ_FAST grammar (src/subst/mod.rs:323-387): 1 = shape written, 0 = stock order. */
CFI_API int cfi_mmvq_fast_from(const char *text, uint32_t ty, cfi_fast *out);
CFI_API int cfi_mmvq_fast_is_opt_out(const char *text);
CFI_API void cfi_mmvq_fast_default(uint32_t ty, cfi_fast *out);
/* Module key of an mmvq plan (src/subst/mod.rs:358-366); fast may be NULL. */
CFI_API void cfi_mmvq_key(uint32_t ty, uint32_t ncols, const cfi_fast *fast, uint32_t nwarps, char *out, size_t len);
/* Entry name of the native kernel (src/subst/mod.rs:474-487). */
CFI_API void cfi_plan_entry_name(const cfi_plan *plan, char *out, size_t len);

/* Plan::map_geometry / map_launch / extra_word (src/subst/mod.rs:509-565).  map_* return 1 and
 * the native geometry when the launch has the shape the native kernel serves, else 0 (the stock
 * kernel then runs).  `vals` holds one little-endian u64 per kernel parameter. */
CFI_API int cfi_plan_map_geometry(const cfi_plan *plan, const uint32_t grid[3], const uint32_t block[3], uint32_t grid_out[3],
                          uint32_t block_out[3]);
CFI_API int cfi_plan_map_launch(const cfi_plan *plan, const uint32_t grid[3], const uint32_t block[3], const uint64_t *vals,
                        int nvals, uint32_t grid_out[3], uint32_t block_out[3]);
CFI_API int cfi_plan_extra_word(const cfi_plan *plan, const uint32_t grid[3], uint32_t *word);

/* ---- per-context native registry and launch router (replaces cuda/subst_hook.rs) ---- */
typedef struct cfi_ctx cfi_ctx;
/* CFI_CTX_FAKE: host-only backend, launches are recorded, never executed.
 * CFI_CTX_DEFER_Q8_1: a native quantize_q8_1 (up to 8 columns, one plane) is held back until the
 * next launch on the context; when that launch is the native streaming mul_mat_vec_q reading
 * exactly its output on the same stream, one kernel does both (the GEMV quantizes the activations
 * in its prologue with the quantizer's arithmetic and stores the q8_1 buffer too, so memory ends
 * up byte-identical), saving one dependent launch per GEMV.  Any other launch, cfi_ctx_flush and
 * cfi_ctx_destroy launch the held-back quantize first.  No counterpart in the reference, whose
 * hook sees every driver call: a caller of this ABI must call cfi_ctx_flush before any operation
 * that is not a launch through this context (memcpy, event record, stream sync, end of capture)
 * whenever the last launch may have been a quantize_q8_1. */
/* CFI_CTX_CONST_WEIGHTS: the caller promises that no kernel writes a weight matrix (the `x`
 * operand of mul_mat_vec_q) while launches through the context may read it -- true for inference
 * on loaded weights, false for example for a quantized KV cache multiplied by mul_mat_vec_q.  The
 * native GEMV then copies its first weight rows into shared memory before waiting on the previous
 * kernel of its stream (programmatic dependent launch), so that copy overlaps the previous
 * kernel instead of following it; activations are still read only after the wait. */
enum { CFI_CTX_FAKE = 1, CFI_CTX_DEFER_Q8_1 = 2, CFI_CTX_CONST_WEIGHTS = 4 };

/* Natives::default (subst_hook.rs:14-24) for `device`; NULL on failure. */
CFI_API cfi_ctx *cfi_ctx_create(int device, int flags);
/* Natives::destroy (subst_hook.rs:32-38); launches a held-back quantize_q8_1 first. */
CFI_API void cfi_ctx_destroy(cfi_ctx *ctx);
/* Launches a held-back quantize_q8_1 (CFI_CTX_DEFER_Q8_1), if any.  Returns 0 or a CUDA error. */
CFI_API int cfi_ctx_flush(cfi_ctx *ctx);

/* launch / launch_to (subst_hook.rs:99-197): runs the native kernel when `plan` is non-NULL, the
 * launch has the expected shape and the native kernel passed its first-use probe; otherwise (and
 * on any native failure, which marks the plan failed) launches `stock_fn` (a CUfunction) with the
 * caller's arguments through cuLaunchKernel.  A mul_mat_q_stream_k_fixup launch whose (dst, tmp)
 * match the last native mmq is skipped.  Returns 0 or a CUDA error code. */
CFI_API int cfi_subst_launch(cfi_ctx *ctx, const cfi_plan *plan, void *stock_fn, const uint32_t grid[3],
                     const uint32_t block[3], uint32_t shared_bytes, void *stream, void **kernel_params);

/* First-use validation probe::validate (src/subst/probe.rs:350-403) on `stream`: 0 = the native
 * kernel matches the host reference on the reference's probe case, else an error code. */
CFI_API int cfi_subst_probe(cfi_ctx *ctx, const cfi_plan *plan, void *stream, char *why, size_t why_len);

/* Native state of a module key: 0 not built, 1 ready, 2 failed (subst_hook.rs:9-12). */
CFI_API int cfi_ctx_native_state(cfi_ctx *ctx, const char *key);

/* fused_q8_1: GEMV launches that absorbed a held-back quantize_q8_1 (each also counts as two
 * native launches, the quantize's and the GEMV's). */
typedef struct cfi_stats {
    uint64_t native_launches, stock_launches, fixups_skipped, probes_run, probes_failed, native_failures;
    uint64_t fused_q8_1;
} cfi_stats;
CFI_API void cfi_ctx_stats(cfi_ctx *ctx, cfi_stats *out);

/* Host-side fault injection (replaces level_zero/fault.rs:25-40): the `nth` (1-based) call of
 * `site` returns `code` instead of running.  Sites below.  code 0 clears. */
enum { CFI_SITE_NATIVE_LAUNCH = 1, CFI_SITE_PROBE = 2, CFI_SITE_STOCK_LAUNCH = 3, CFI_SITE_BUILD = 4 };
CFI_API void cfi_ctx_inject(cfi_ctx *ctx, int site, int nth, int code);

/* ---- prefill GEMM without device allocation ----
 * No counterpart in the reference: cuda-for-intel has no equivalent entry point.
 *
 * cfi_mmq_static_scratch runs the native tensor-core mul_mat_q (Q8_0 or Q4_K weights, non-MoE)
 * exactly as cfi_subst_launch does, for callers that are not allowed to allocate device memory:
 * a launch hook sitting inside the host application's cuLaunchKernel (allocating there would
 * re-enter the driver's allocator and change the application's own memory accounting), a
 * serving process whose memory pool reserved all free HBM up front (cudaMalloc would fail at run
 * time), or a code path that cannot afford cudaMalloc's implicit device synchronisation.  The
 * GEMM's one piece of scratch -- an fp16 copy of the activations, planes x ncols_dst x Kt x 2
 * bytes, where planes = nchannels_y x nsamples_y and Kt = ncols_x (Q8_0) or ncols_x +
 * ceil(ncols_x / 2048) x 64 (Q4_K: the min-correction columns) -- then lives in a fixed array of
 * CFI_MMQ_STATIC_SCRATCH_BYTES compiled into the library; every GPU on which the library's
 * kernels are loaded holds that array until the process exits.  Larger problems are rejected
 * with cudaErrorInvalidValue and a message in `why` before anything is launched.
 *
 * kernel_params are the 23 parameters of ggml-cuda's mul_mat_q<type, mmq_x, need_check> (x, y,
 * ids_dst, expert_bounds, dst, tmp_fixup, then 17 ints); inputs and outputs stay the caller's.
 * The array's device address is looked up (cudaGetSymbolAddress) on the first call on each
 * device, which must be the current device; make that first call before any stream capture.
 * Every call uses the same array and leaves its contents behind (nothing in it has to start at
 * zero), so two calls whose work overlaps on the GPU -- on different streams without ordering
 * between them -- race on it.  The entry point itself calls no cudaMalloc, cudaFree or other
 * allocating routine; in particular it never splits K (a split-K launch needs a device
 * workspace), so its results match cfi_subst_launch's whenever that one does not split K and
 * agree within fp32 summation order otherwise.  Returns 0 or a CUDA error code. */
#define CFI_MMQ_STATIC_SCRATCH_BYTES (8u * 1024u * 1024u)
CFI_API int cfi_mmq_static_scratch(uint32_t ggml_type, void **kernel_params, void *stream, char *why, size_t why_len);

/* Reads and clears the device error word of the bounded waits in the tcgen05 kernels. */
CFI_API unsigned int cfi_device_error(void);

/* Library version string. */
CFI_API const char *cfi_version(void);

#ifdef __cplusplus
}
#endif
#endif
