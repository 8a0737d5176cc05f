"""Python binding of libcfi_b200.so (ctypes) and a ggml-style caller of its C ABI.

The product is the C ABI in include/cfi_subst.h: a ggml-cuda kernel launch is decided by
mangled name + parameter layout and launched through cfi_subst_launch with the caller's
kernelParams.  This module packs kernelParams exactly as ggml-cuda does for each kernel
(`GgmlCaller`), so tests and the benchmark drive the library the way the driver hook would.
It also holds the host-side weight quantizers (Q8_0 and a seeded Q4_K) used to make synthetic
weights.  There is no CPU compute path: without the shared library or a GPU every launch raises.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libcfi_b200.so")

# ---- ggml types ----
Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K = 2, 6, 8, 12, 13, 14
BLOCK_BYTES = {Q4_0: 18, Q5_0: 22, Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210}
QK = {Q4_0: 32, Q5_0: 32, Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}

# ---- cfi_param kinds (include/cfi_subst.h) ----
P_U8, P_U16, P_U32, P_F32, P_U64, P_PTR, P_WORDS, P_STAGED = range(8)
SUBSTITUTE, MISMATCH, NOT_APPLICABLE = 0, 1, 2
K_MMVQ, K_QUANTIZE_Q8_1, K_MMQ, K_MMQ_FIXUP, K_QUANTIZE_MMQ, K_RMS_NORM, K_RMS_NORM_PLAIN, K_ROPE_NEOX, K_SOFT_MAX = range(1, 10)
CTX_FAKE, CTX_DEFER_Q8_1, CTX_CONST_WEIGHTS = 1, 2, 4
SITE_NATIVE_LAUNCH, SITE_PROBE, SITE_STOCK_LAUNCH, SITE_BUILD = 1, 2, 3, 4


class Param(C.Structure):
    _fields_ = [("kind", C.c_int32), ("a", C.c_uint16), ("b", C.c_uint16), ("c", C.c_uint8)]


class Fast(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("warps", C.c_uint32), ("unroll", C.c_uint32), ("wide", C.c_uint32)]

    def tup(self):
        return (self.rows, self.warps, self.unroll, bool(self.wide))


class Plan(C.Structure):
    _fields_ = [("kernel", C.c_int32), ("ty", C.c_uint32), ("ncols", C.c_uint32), ("nwarps", C.c_uint32),
                ("aux", C.c_uint32), ("has_fast", C.c_uint32), ("fast", Fast), ("layout_hash", C.c_uint64),
                ("key", C.c_char * 64)]


class Stats(C.Structure):
    _fields_ = [("native_launches", C.c_uint64), ("stock_launches", C.c_uint64), ("fixups_skipped", C.c_uint64),
                ("probes_run", C.c_uint64), ("probes_failed", C.c_uint64), ("native_failures", C.c_uint64),
                ("fused_q8_1", C.c_uint64)]


_lib = None


def lib():
    """Loads libcfi_b200.so (raises when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError("libcfi_b200.so is not built (run cuda-for-intel_b200/build.py): %s" % LIB_PATH)
    L = C.CDLL(LIB_PATH)
    u32p = C.POINTER(C.c_uint32)
    L.cfi_subst_decide.argtypes = [C.c_char_p, C.POINTER(Param), C.c_int, C.c_char_p, C.POINTER(Plan), C.c_char_p, C.c_size_t]
    L.cfi_switch_allows.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p]
    L.cfi_switch_denies.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p]
    L.cfi_switch_is_none.argtypes = [C.c_char_p]
    L.cfi_demangle.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_int64), C.POINTER(C.c_int), C.c_char_p,
                               C.c_size_t, C.c_int]
    L.cfi_layout_hash.argtypes = [C.POINTER(Param), C.c_int]
    L.cfi_layout_hash.restype = C.c_uint64
    L.cfi_mmvq_fast_from.argtypes = [C.c_char_p, C.c_uint32, C.POINTER(Fast)]
    L.cfi_mmvq_fast_is_opt_out.argtypes = [C.c_char_p]
    L.cfi_mmvq_fast_default.argtypes = [C.c_uint32, C.POINTER(Fast)]
    L.cfi_mmvq_fast_default.restype = None
    L.cfi_mmvq_key.argtypes = [C.c_uint32, C.c_uint32, C.POINTER(Fast), C.c_uint32, C.c_char_p, C.c_size_t]
    L.cfi_mmvq_key.restype = None
    L.cfi_plan_entry_name.argtypes = [C.POINTER(Plan), C.c_char_p, C.c_size_t]
    L.cfi_plan_entry_name.restype = None
    L.cfi_plan_map_geometry.argtypes = [C.POINTER(Plan), u32p, u32p, u32p, u32p]
    L.cfi_plan_map_launch.argtypes = [C.POINTER(Plan), u32p, u32p, C.POINTER(C.c_uint64), C.c_int, u32p, u32p]
    L.cfi_plan_extra_word.argtypes = [C.POINTER(Plan), u32p, u32p]
    L.cfi_ctx_create.argtypes = [C.c_int, C.c_int]
    L.cfi_ctx_create.restype = C.c_void_p
    L.cfi_ctx_destroy.argtypes = [C.c_void_p]
    L.cfi_ctx_destroy.restype = None
    L.cfi_ctx_flush.argtypes = [C.c_void_p]
    L.cfi_subst_launch.argtypes = [C.c_void_p, C.POINTER(Plan), C.c_void_p, u32p, u32p, C.c_uint32, C.c_void_p,
                                   C.POINTER(C.c_void_p)]
    L.cfi_subst_probe.argtypes = [C.c_void_p, C.POINTER(Plan), C.c_void_p, C.c_char_p, C.c_size_t]
    L.cfi_ctx_native_state.argtypes = [C.c_void_p, C.c_char_p]
    L.cfi_ctx_stats.argtypes = [C.c_void_p, C.POINTER(Stats)]
    L.cfi_ctx_stats.restype = None
    L.cfi_ctx_inject.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
    L.cfi_ctx_inject.restype = None
    L.cfi_mmq_static_scratch.argtypes = [C.c_uint32, C.POINTER(C.c_void_p), C.c_void_p, C.c_char_p, C.c_size_t]
    vp, i, ll = C.c_void_p, C.c_int, C.c_longlong
    L.cfi_blas_create.argtypes = [C.POINTER(vp)]
    L.cfi_blas_destroy.argtypes = [vp]
    L.cfi_blas_set_stream.argtypes = [vp, vp]
    L.cfi_blas_get_stream.argtypes = [vp, C.POINTER(vp)]
    L.cfi_blas_set_pointer_mode.argtypes = [vp, i]
    L.cfi_blas_last_path.argtypes = [vp]
    L.cfi_blas_validate.argtypes = [i] * 12
    L.cfi_blas_gemm_ex.argtypes = [vp, i, i, i, i, i, vp, vp, i, i, vp, i, i, vp, vp, i, i, i, i]
    L.cfi_blas_gemm_strided_batched_ex.argtypes = [vp, i, i, i, i, i, vp, vp, i, i, ll, vp, i, i, ll, vp, vp, i, i, ll, i,
                                                   i, i]
    L.cfi_blas_gemm_batched_ex.argtypes = [vp, i, i, i, i, i, vp, vp, i, i, vp, i, i, vp, vp, i, i, i, i, i]
    L.cfi_blas_sgemm.argtypes = [vp, i, i, i, i, i, vp, vp, i, vp, i, vp, vp, i]
    L.cfi_device_error.restype = C.c_uint
    L.cfi_version.restype = C.c_char_p
    f = C.c_float
    L.cfi_glue_get_rows_q8_0.argtypes = [vp, vp, vp, i, vp]
    L.cfi_glue_qkv_bias.argtypes = [vp, vp, vp, vp, vp, vp, i, i, vp]
    L.cfi_glue_kv_store.argtypes = [vp, vp, vp, vp, vp, vp, vp, i, i, i, i, vp]
    L.cfi_glue_causal_mask.argtypes = [vp, vp, i, vp]
    L.cfi_glue_to_f16.argtypes = [vp, vp, i, vp]
    L.cfi_glue_add.argtypes = [vp, vp, i, vp]
    L.cfi_glue_swiglu.argtypes = [vp, vp, vp, i, vp]
    L.cfi_glue_argmax_next.argtypes = [vp, i, vp, vp, vp]
    L.cfi_glue_gather_row_shards.argtypes = [vp, vp, i, i, i, ll, vp]
    L.cfi_decode_step_q8_0.argtypes = [vp, vp, vp]
    L.cfi_decode_step_error.restype = C.c_uint
    L.cfi_mmq_skinny_group.argtypes = [C.c_uint32, i, vp, vp, vp, vp, vp, vp, C.c_uint32, C.c_uint32, C.c_uint32, vp]
    L.cfi_mmq_skinny_group_peers.argtypes = [C.c_uint32, i, vp, vp, vp, vp, vp, vp, C.c_uint32, C.c_uint32, C.c_uint32,
                                             C.POINTER(PeerSet), vp]
    L.cfi_peer_alloc.argtypes = [C.c_size_t, C.POINTER(C.c_void_p), vp]
    L.cfi_peer_open.argtypes = [vp, C.POINTER(C.c_void_p)]
    L.cfi_peer_close.argtypes = [vp]
    L.cfi_peer_free.argtypes = [vp]
    L.cfi_peer_barrier.argtypes = [C.POINTER(PeerSet), vp]
    L.cfi_peer_all_gather.argtypes = [vp, C.c_size_t, vp, C.POINTER(PeerSet), vp]
    L.cfi_fused_add_rmsnorm_q8_1.argtypes = [vp, vp, vp, vp, i, f, vp]
    L.cfi_fused_qkv_rope_store.argtypes = [vp, vp, vp, vp, vp, vp, i, i, i, i, f, vp]
    L.cfi_fused_attention_q8_1.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, f, vp]
    L.cfi_fused_swiglu_q8_1.argtypes = [vp, vp, i, vp]
    L.cfi_fused_mmvq_add_rmsnorm_q8_1.argtypes = [vp, vp, vp, i, i, vp, vp, vp, f, vp]
    L.cfi_fused_mmvq_swiglu_q8_1.argtypes = [vp, vp, vp, i, i, vp, vp]
    L.cfi_fused_mmvq_qkv_rope_store.argtypes = [vp, vp, vp, i, vp, vp, vp, vp, vp, i, i, i, i, f, vp]
    _lib = L
    return L


def exported_symbols():
    """Names every include/*.h of the product declares (the C ABI)."""
    import re
    names = set()
    inc = os.path.join(HERE, "..", "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            txt = open(os.path.join(inc, f)).read()
            names.update(re.findall(r"^CFI_API[^;(]*?\b(\w+)\s*\(", txt, re.M))
    return sorted(names)


# ---------------------------------------------------------------------------------------------
# layouts of the ggml kernels (what a PTX reader reports for each parameter)
# ---------------------------------------------------------------------------------------------
def _p(kind, a=0, b=0, c=0):
    return (kind, a, b, c)


PTR, U32, U64, F32, U3 = _p(P_PTR), _p(P_U32), _p(P_U64), _p(P_F32), _p(P_WORDS, 3, 4, 0)
LAYOUTS = {
    "mmvq": [PTR, PTR, PTR, PTR, U32, U3, U32, U32, U32, U3, U32, U32, U32, U3, U32, U32, U32],
    "quantize_q8_1": [PTR, PTR, U64, U64, U64, U64, U64, U32, U3],
    "mmq": [PTR] * 6 + [U32] * 17,
    "mmq_fixup": [PTR] * 4 + [U32] * 9,
    "quantize_mmq": [PTR, PTR, PTR, U64, U64, U64, U64, U64, U32, U32],
    "rms_norm": [PTR, PTR, U32, U64, U64, U64, F32, PTR, U64, U64, U64, U3, U3, U3, U3, PTR, U64, U64, U64, U3, U3, U3, U3],
    "rms_norm_plain": [PTR, PTR, U32, U32, U32, U64, U64, U64, F32],
    "rope_neox": [PTR, PTR, U32, U32, U32, U32, U32, PTR, F32, F32, F32, _p(P_WORDS, 2, 4, 0), F32, PTR],
    "soft_max": [PTR, PTR, PTR, PTR, _p(P_WORDS, 32, 8, 0)],
    "fattn": [PTR] * 8 + [F32, F32, F32, F32, U32, F32] + [U32] * 13 + [U64, U32, U32, U64, U32, U32, U32, U32, U32, U64],
    "fattn_fixup": [PTR, PTR, U32, U32, U32, U32],
}

NAMES = {
    "mmvq": "_Z13mul_mat_vec_qIL9ggml_type{ty}ELi{ncols}EEvPKvS2_PKiPfj5uint3jjjS6_jjjS6_jjj",
    "quantize_q8_1": "_Z13quantize_q8_1PKfPvxxxxxj5uint3",
    "mmq": "_Z9mul_mat_qIL9ggml_type{ty}ELi{mmq_x}ELb{check}EEvPKcPKiS4_S4_PfS5_iiiiiiiiiiiiiiiii",
    "mmq_fixup": "_Z24mul_mat_q_stream_k_fixupIL9ggml_type{ty}ELi{mmq_x}ELb{check}EEvPKiS2_PfPKfiiiiiiiii",
    "quantize_mmq": "_Z17quantize_mmq_q8_1IL18mmq_q8_1_ds_layout{layout}EEvPKfPKiPvxxxxxii",
    "rms_norm": "_Z12rms_norm_f32ILi256ELb{mul}ELb{add}EEvPKfPfixxxfS1_xxx5uint3S3_S3_S3_S1_xxxS3_S3_S3_S3_",
    "rms_norm_plain": "_Z12rms_norm_f32ILi32EEvPKfPfiiilllf",
    "rope_neox": "_Z9rope_neoxILb{fwd}ELb{ff}EfEvPKT1_PS0_iiiiiPKifff14rope_corr_dimsfPKf",
    "soft_max": "_Z12soft_max_f32ILb1ELi0ELi0E{t}EvPKfPKT2_S1_Pf15soft_max_params",
    "fattn": "_Z18flash_attn_ext_f16ILi{d}ELi{d}ELi32ELi1ELi4ELi2ELb0ELb0EEvPKcS1_S1_S1_S1_PKiPfP6float2ffffjfiiiiiiiiiiiiiliiliiiiil",
    "fattn_fixup": "_Z25flash_attn_stream_k_fixupILi{d}ELi32ELi1EEvPfPK6float2iiii",
}


def layout(name):
    ps = LAYOUTS[name]
    arr = (Param * len(ps))()
    for i, (k, a, b, c) in enumerate(ps):
        arr[i].kind, arr[i].a, arr[i].b, arr[i].c = k, a, b, c
    return arr


def decide(name, params, switch=None):
    """decide(name, params, switch) -> (code, Plan, why)."""
    if isinstance(params, str):
        params = layout(params)
    plan = Plan()
    why = C.create_string_buffer(512)
    sw = None if switch is None else switch.encode()
    n = len(params)
    code = lib().cfi_subst_decide(name.encode(), params if n else None, n, sw, C.byref(plan), why, 512)
    return code, plan, why.value.decode()


def demangle(name):
    base = C.create_string_buffer(256)
    vals = (C.c_int64 * 16)()
    kinds = (C.c_int * 16)()
    names = C.create_string_buffer(512)
    n = lib().cfi_demangle(name.encode(), base, 256, vals, kinds, names, 512, 16)
    if n < 0:
        return None
    nm = names.value.decode().split("\n") if n else []
    targs = []
    for i in range(n):
        k = kinds[i]
        targs.append(("int", vals[i]) if k == 0 else ("enum", nm[i], vals[i]) if k == 1 else ("type", nm[i]))
    return base.value.decode(), targs


def _u3(*v):
    return (C.c_uint32 * 3)(*v)


def map_geometry(plan, grid, block):
    go, bo = _u3(), _u3()
    ok = lib().cfi_plan_map_geometry(C.byref(plan), _u3(*grid), _u3(*block), go, bo)
    return (tuple(go), tuple(bo)) if ok else None


def map_launch(plan, grid, block, vals):
    go, bo = _u3(), _u3()
    arr = (C.c_uint64 * len(vals))(*vals)
    ok = lib().cfi_plan_map_launch(C.byref(plan), _u3(*grid), _u3(*block), arr, len(vals), go, bo)
    return (tuple(go), tuple(bo)) if ok else None


def entry_name(plan):
    b = C.create_string_buffer(128)
    lib().cfi_plan_entry_name(C.byref(plan), b, 128)
    return b.value.decode()


def fastdiv_values(d):
    """ggml init_fastdiv_values: (mp, L, d)."""
    l = 0
    while l < 32 and (1 << l) < d:
        l += 1
    mp = ((1 << 32) * ((1 << l) - d)) // d + 1
    return (mp & 0xFFFFFFFF, l, d)


# ---------------------------------------------------------------------------------------------
# kernelParams packing
# ---------------------------------------------------------------------------------------------
class KernelArgs:
    """A cuLaunchKernel-style kernelParams array: one pointer per parameter, each to its value."""

    def __init__(self, values):
        self._keep = []
        self.ptrs = (C.c_void_p * len(values))()
        for i, (kind, v) in enumerate(values):
            if kind == "ptr" or kind == "u64":
                o = C.c_uint64(int(v) & 0xFFFFFFFFFFFFFFFF)
            elif kind == "i64":
                o = C.c_int64(int(v))
            elif kind == "u32":
                o = C.c_uint32(int(v) & 0xFFFFFFFF)
            elif kind == "i32":
                o = C.c_int32(int(v))
            elif kind == "f32":
                o = C.c_float(float(v))
            elif kind == "u3":
                o = (C.c_uint32 * 3)(*[int(x) & 0xFFFFFFFF for x in v])
            elif kind == "f2":
                o = (C.c_float * 2)(*v)
            elif kind == "bytes":
                o = C.create_string_buffer(bytes(v), len(v))
            else:
                raise ValueError(kind)
            self._keep.append(o)
            self.ptrs[i] = C.cast(C.pointer(o), C.c_void_p)

    def vals(self):
        out = []
        for o in self._keep:
            raw = C.string_at(C.addressof(o), min(8, C.sizeof(o)))
            out.append(int.from_bytes(raw.ljust(8, b"\0"), "little"))
        return out


class DecodeLayer(C.Structure):
    """CfiDecodeLayer (include/cfi_glue.h)."""
    _fields_ = [(n, C.c_void_p) for n in ("wqkv", "bqkv", "wo", "wgu", "wd", "attn_norm", "ffn_norm", "kc", "vc")]


class DecodeStep(C.Structure):
    """CfiDecodeStep (include/cfi_glue.h)."""
    _fields_ = ([(n, C.c_int) for n in ("hidden", "n_head", "n_kv_head", "head_dim", "ffn", "vocab", "n_ctx", "n_layers")] +
                [("eps", C.c_float), ("theta", C.c_float)] +
                [(n, C.c_void_p) for n in ("embd", "head", "out_norm", "x", "qkv", "qr", "o", "gu", "dn", "logits", "hq", "aq",
                                           "gq", "token", "pos")])


class Ctx:
    """A cfi_ctx: per-device native registry, router and statistics."""

    def __init__(self, device=0, fake=False, defer_q8_1=False, const_weights=False):
        """defer_q8_1: hold each quantize_q8_1 back for the GEMV that reads it (one fused kernel);
        call flush() before reading its output by anything but a launch through this context.
        const_weights: no kernel writes the GEMVs' weight matrices, so each GEMV copies its
        weights before waiting on the previous kernel."""
        flags = (CTX_FAKE if fake else 0) | (CTX_DEFER_Q8_1 if defer_q8_1 else 0)
        self.h = lib().cfi_ctx_create(device, flags | (CTX_CONST_WEIGHTS if const_weights else 0))
        if not self.h:
            raise RuntimeError("cfi_ctx_create failed")

    def close(self):
        if self.h:
            lib().cfi_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def launch(self, plan, grid, block, args, stream=0, stock_fn=None, shared=0):
        return lib().cfi_subst_launch(self.h, C.byref(plan) if plan is not None else None, stock_fn, _u3(*grid),
                                      _u3(*block), shared, C.c_void_p(stream), args.ptrs)

    def flush(self):
        check(lib().cfi_ctx_flush(self.h), "cfi_ctx_flush")

    def probe(self, plan, stream=0):
        why = C.create_string_buffer(512)
        rc = lib().cfi_subst_probe(self.h, C.byref(plan), C.c_void_p(stream), why, 512)
        return rc, why.value.decode()

    def state(self, key):
        return lib().cfi_ctx_native_state(self.h, key.encode() if isinstance(key, str) else key)

    def stats(self):
        s = Stats()
        lib().cfi_ctx_stats(self.h, C.byref(s))
        return {f: getattr(s, f) for f, _ in Stats._fields_}

    def inject(self, site, nth, code):
        lib().cfi_ctx_inject(self.h, site, nth, code)


class Blas:
    """A cfi_blas handle (the cuBLAS-compatible GEMM entry points of include/cfi_cublas.h)."""

    OP_N, OP_T = 0, 1
    R_32F, R_16F, R_16BF = 0, 2, 14
    COMPUTE_16F, COMPUTE_32F = 64, 68

    def __init__(self, stream=0):
        h = C.c_void_p()
        st = lib().cfi_blas_create(C.byref(h))
        if st:
            raise RuntimeError("cfi_blas_create: %d" % st)
        self.h = h
        lib().cfi_blas_set_stream(self.h, C.c_void_p(stream))

    def close(self):
        if self.h:
            lib().cfi_blas_destroy(self.h)
            self.h = None

    def set_stream(self, stream):
        return lib().cfi_blas_set_stream(self.h, C.c_void_p(stream))

    def set_pointer_mode(self, mode):
        return lib().cfi_blas_set_pointer_mode(self.h, mode)

    def last_path(self):
        return lib().cfi_blas_last_path(self.h)

    @staticmethod
    def _scalar(v, f16):
        return C.byref(C.c_uint16(int(np.float16(v).view(np.uint16))) if f16 else C.c_float(v))

    def gemm_ex(self, ta, tb, m, n, k, alpha, A, at, lda, B, bt, ldb, beta, Cp, ct, ldc, compute=68, dev_scalars=None):
        f16 = compute == self.COMPUTE_16F
        al, be = (dev_scalars if dev_scalars else (self._scalar(alpha, f16), self._scalar(beta, f16)))
        return lib().cfi_blas_gemm_ex(self.h, ta, tb, m, n, k, al, C.c_void_p(A), at, lda, C.c_void_p(B), bt, ldb, be,
                                      C.c_void_p(Cp), ct, ldc, compute, -1)

    def gemm_strided_batched_ex(self, ta, tb, m, n, k, alpha, A, at, lda, sa, B, bt, ldb, sb, beta, Cp, ct, ldc, sc,
                                batch, compute=68):
        f16 = compute == self.COMPUTE_16F
        return lib().cfi_blas_gemm_strided_batched_ex(self.h, ta, tb, m, n, k, self._scalar(alpha, f16), C.c_void_p(A),
                                                      at, lda, sa, C.c_void_p(B), bt, ldb, sb, self._scalar(beta, f16),
                                                      C.c_void_p(Cp), ct, ldc, sc, batch, compute, -1)

    def gemm_batched_ex(self, ta, tb, m, n, k, alpha, Aarr, at, lda, Barr, bt, ldb, beta, Carr, ct, ldc, batch,
                        compute=68):
        f16 = compute == self.COMPUTE_16F
        return lib().cfi_blas_gemm_batched_ex(self.h, ta, tb, m, n, k, self._scalar(alpha, f16), C.c_void_p(Aarr), at,
                                              lda, C.c_void_p(Barr), bt, ldb, self._scalar(beta, f16), C.c_void_p(Carr),
                                              ct, ldc, batch, compute, -1)

    def sgemm(self, ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, Cp, ldc):
        return lib().cfi_blas_sgemm(self.h, ta, tb, m, n, k, C.byref(C.c_float(alpha)), C.c_void_p(A), lda,
                                    C.c_void_p(B), ldb, C.byref(C.c_float(beta)), C.c_void_p(Cp), ldc)


def check(rc, what):
    if rc != 0:
        raise RuntimeError("%s failed with CUDA error %d" % (what, rc))


class GgmlCaller:
    """Launches ggml-cuda kernels the way ggml does (stock grid, block and kernelParams), through
    the substitution C ABI.  Pointers are device addresses (ints); `stream` a cudaStream_t."""

    def __init__(self, ctx, switch="all"):
        self.ctx = ctx
        self.switch = switch
        self._plans = {}

    def plan(self, key, name, lay):
        p = self._plans.get(key)
        if p is None:
            code, p, why = decide(name, lay, self.switch)
            if code != SUBSTITUTE:
                raise RuntimeError("no substitution for %s (%d %s)" % (name, code, why))
            self._plans[key] = p
        return p

    def _go(self, plan, grid, block, vals, stream, what):
        args = KernelArgs(vals)
        check(self.ctx.launch(plan, grid, block, args, stream), what)
        return args

    def quantize_q8_1(self, x, vy, ne00, ne0, ne1, ne2=1, ne3=1, s01=None, s02=None, s03=None, stream=0):
        s01 = ne00 if s01 is None else s01
        s02 = s01 * ne1 if s02 is None else s02
        s03 = s02 * ne2 if s03 is None else s03
        p = self.plan("q81", NAMES["quantize_q8_1"], "quantize_q8_1")
        vals = [("ptr", x), ("ptr", vy), ("i64", ne00), ("i64", s01), ("i64", s02), ("i64", s03), ("i64", ne0),
                ("u32", ne1), ("u3", fastdiv_values(ne2))]
        return self._go(p, ((ne0 + 255) // 256, ne1, ne2 * ne3), (256, 1, 1), vals, stream, "quantize_q8_1")

    def mmvq(self, ty, ncols, vx, vy, dst, ncols_x, nrows, stride_row_x=None, stride_col_y=None, stride_col_dst=None,
             nchannels=1, channel_ratio=1, nsamples=1, sample_ratio=1, ids=0, nchannels_y=1, strides=None, stream=0):
        """mul_mat_vec_q<ty, ncols>: y[c][r] = sum_k W[r][k] x[c][k]; x given as q8_1 blocks."""
        bpr = ncols_x // QK[ty]
        stride_row_x = bpr if stride_row_x is None else stride_row_x
        stride_col_y = ncols_x // 32 if stride_col_y is None else stride_col_y
        stride_col_dst = nrows if stride_col_dst is None else stride_col_dst
        st = strides or {}
        scx = st.get("channel_x", nrows * stride_row_x)
        scy = st.get("channel_y", stride_col_y * ncols)
        scd = st.get("channel_dst", stride_col_dst * ncols)
        ssx = st.get("sample_x", scx * max(1, nchannels // channel_ratio))
        ssy = st.get("sample_y", scy * nchannels)
        ssd = st.get("sample_dst", scd * nchannels)
        p = self.plan(("mmvq", ty, ncols), NAMES["mmvq"].format(ty=ty, ncols=ncols), "mmvq")
        nchy = fastdiv_values(nchannels_y) if ids else (0, 0, 0)
        chr_ = (0, 0, 0) if ids else fastdiv_values(channel_ratio)
        vals = [("ptr", vx), ("ptr", vy), ("ptr", ids), ("ptr", dst), ("u32", ncols_x), ("u3", nchy),
                ("u32", stride_row_x), ("u32", stride_col_y), ("u32", stride_col_dst), ("u3", chr_), ("u32", scx),
                ("u32", scy), ("u32", scd), ("u3", fastdiv_values(sample_ratio)), ("u32", ssx), ("u32", ssy),
                ("u32", ssd)]
        rpb = 1 if ncols == 1 else 2
        nw = 4 if ncols <= 4 else 2
        return self._go(p, ((nrows + rpb - 1) // rpb, nchannels, nsamples), (32, nw, 1), vals, stream, "mmvq")

    def quantize_mmq(self, layout_ds4, x, vy, ne00, ne0, ne1, ne2=1, ne3=1, s01=None, s02=None, s03=None, ids=0,
                     stream=0):
        s01 = ne00 if s01 is None else s01
        s02 = s01 * ne1 if s02 is None else s02
        s03 = s02 * ne2 if s03 is None else s03
        p = self.plan(("qmmq", layout_ds4), NAMES["quantize_mmq"].format(layout=int(layout_ds4)), "quantize_mmq")
        vals = [("ptr", x), ("ptr", ids), ("ptr", vy), ("i64", ne00), ("i64", s01), ("i64", s02), ("i64", s03),
                ("i64", ne0), ("i32", ne1), ("i32", ne2)]
        return self._go(p, (ne1, (ne0 + 511) // 512, ne2 * ne3), (128, 1, 1), vals, stream, "quantize_mmq_q8_1")

    def mmq(self, ty, vx, vy, dst, ncols_x, nrows, ncols_dst, mmq_x=128, stream=0, tmp_fixup=0, stride_col_dst=None):
        """mul_mat_q<ty> non-MoE, one channel and sample: dst[col][row] (column stride nrows unless
        given)."""
        groups = 8 if ty in (Q4_K, Q5_K, Q6_K) else 1
        nb = ncols_x // 32 // groups
        ychan = ncols_x // 128 * ncols_dst * 36
        scd = nrows if stride_col_dst is None else stride_col_dst
        p = self.plan(("mmq", ty, mmq_x), NAMES["mmq"].format(ty=ty, mmq_x=mmq_x, check=0), "mmq")
        w = [ncols_x, nrows, ncols_dst, nb, ncols_dst, scd, 1, 1, nrows * nb, ychan, scd * ncols_dst, 1, 1,
             nrows * nb, ychan, scd * ncols_dst, ncols_dst]
        vals = [("ptr", vx), ("ptr", vy), ("ptr", 0), ("ptr", 0), ("ptr", dst), ("ptr", tmp_fixup)] + [("u32", v) for v in w]
        return self._go(p, (148, 1, 1), (32, 8, 1), vals, stream, "mul_mat_q")

    def mmq_words(self, ty, vx, vy, dst, words, mmq_x=128, stream=0, tmp_fixup=0):
        """mul_mat_q<ty> with the 17 integer words given explicitly (ncols_x, nrows_x, ncols_dst,
        stride_row_x, ncols_y, stride_col_dst, channel_ratio, nchannels_y, stride_channel_x/y/dst,
        sample_ratio, nsamples_y, stride_sample_x/y/dst, ncols_max; probe.rs:293-321)."""
        p = self.plan(("mmq", ty, mmq_x), NAMES["mmq"].format(ty=ty, mmq_x=mmq_x, check=0), "mmq")
        vals = [("ptr", vx), ("ptr", vy), ("ptr", 0), ("ptr", 0), ("ptr", dst), ("ptr", tmp_fixup)] + [("u32", v) for v in words]
        return self._go(p, (148, 1, 1), (32, 8, 1), vals, stream, "mul_mat_q")

    def fattn(self, d, q, k, v, mask, dst, nq, nh, nh_kv, nkv, ns, scale, nq_pad=None, dst_meta=0, q_strides=None,
              kv_strides=None, stream=0):
        """flash_attn_ext_f16<d, d, ...> on ggml's contiguous layouts (probe.rs:490-528): Q f32
        [ns][nh][nq][d], K/V f16 [ns][nh_kv][nkv][d], mask f16 [ns][nq_pad][nkv] (0: none), dst f32
        [ns][nq][nh][d]."""
        nq_pad = (nq + 15) // 16 * 16 if nq_pad is None else nq_pad
        p = self.plan(("fattn", d), NAMES["fattn"].format(d=d), "fattn")
        nb01, nb02, nb03 = q_strides or (d * 4, d * 4 * nq, d * 4 * nq * nh)
        nb11, nb12, nb13 = kv_strides or (d * 2, d * 2 * nkv, d * 2 * nkv * nh_kv)
        vals = [("ptr", q), ("ptr", k), ("ptr", v), ("ptr", mask), ("ptr", 0), ("ptr", 0), ("ptr", dst),
                ("ptr", dst_meta), ("f32", scale), ("f32", 0.0), ("f32", 1.0), ("f32", 1.0), ("u32", 0), ("f32", 0.0),
                ("u32", d), ("u32", nq), ("u32", nh), ("u32", ns), ("u32", nb01), ("u32", nb02), ("u32", nb03),
                ("u32", d), ("u32", nkv), ("u32", nh_kv), ("u32", ns), ("u32", nb11), ("u32", nb12), ("u64", nb13),
                ("u32", nb11), ("u32", nb12), ("u64", nb13), ("u32", nkv), ("u32", nq_pad), ("u32", ns if mask else 0),
                ("u32", nkv * 2), ("u32", nkv * 2 * nq_pad), ("u64", nkv * 2 * nq_pad)]
        return self._go(p, ((nq + 31) // 32, nh, ns), (32, 4, 1), vals, stream, "flash_attn_ext_f16")

    def fattn_fixup(self, d, dst, dst_meta, nq, nh, ns, nkv, stream=0):
        p = self.plan(("fattn_fixup", d), NAMES["fattn_fixup"].format(d=d), "fattn_fixup")
        vals = [("ptr", dst), ("ptr", dst_meta), ("i32", nq), ("i32", nh), ("i32", ns), ("i32", nkv)]
        return self._go(p, (nq, nh, ns), (d, 1, 1), vals, stream, "flash_attn_stream_k_fixup")

    def rms_norm(self, x, dst, ncols, nrows, mul=0, add=0, eps=1e-6, nchannels=1, nsamples=1, stream=0):
        m, a = int(bool(mul)), int(bool(add))
        p = self.plan(("rms", m, a), NAMES["rms_norm"].format(mul=m, add=a), "rms_norm")
        fc, f1 = fastdiv_values(ncols), fastdiv_values(1)
        vals = [("ptr", x), ("ptr", dst), ("i32", ncols), ("i64", ncols), ("i64", ncols * nrows),
                ("i64", ncols * nrows * nchannels), ("f32", eps), ("ptr", mul), ("i64", 0), ("i64", 0), ("i64", 0),
                ("u3", fc), ("u3", f1), ("u3", f1), ("u3", f1), ("ptr", add), ("i64", 0), ("i64", 0), ("i64", 0),
                ("u3", fc), ("u3", f1), ("u3", f1), ("u3", f1)]
        return self._go(p, (nrows, nchannels, nsamples), (256, 1, 1), vals, stream, "rms_norm_f32")

    def rms_norm_plain(self, x, dst, ncols, nrows, eps=1e-5, stream=0):
        p = self.plan("rms_plain", NAMES["rms_norm_plain"], "rms_norm_plain")
        vals = [("ptr", x), ("ptr", dst), ("i32", ncols), ("i32", 1), ("i32", 1), ("i64", ncols),
                ("i64", ncols * nrows), ("i64", ncols * nrows), ("f32", eps)]
        return self._go(p, (nrows, 1, 1), (32, 1, 1), vals, stream, "rms_norm_f32<32>")

    def rope_neox(self, x, dst, ne0, ne1, ntok, n_dims, pos, freq_base=1e6, freq_scale=1.0, ext_factor=0.0,
                  attn_factor=1.0, freq_factors=0, forward=True, stream=0):
        ff = int(bool(freq_factors))
        p = self.plan(("rope", forward, ff), NAMES["rope_neox"].format(fwd=int(forward), ff=ff), "rope_neox")
        theta_scale = float(np.float32(freq_base) ** np.float32(-2.0 / n_dims))
        vals = [("ptr", x), ("ptr", dst), ("i32", ne0), ("i32", ne1), ("i32", ne0), ("i32", ne0 * ne1),
                ("i32", n_dims), ("ptr", pos), ("f32", freq_scale), ("f32", ext_factor), ("f32", attn_factor),
                ("f2", (0.0, 0.0)), ("f32", theta_scale), ("ptr", freq_factors)]
        return self._go(p, (ne1 * ntok, (ne0 + 511) // 512, 1), (1, 256, 1), vals, stream, "rope_neox")

    def soft_max(self, x, mask, dst, ncols, ne01, nheads, scale, max_bias=0.0, mask_f16=False, sinks=0, stream=0):
        t = "6__half" if mask_f16 else "f"
        p = self.plan(("sm", mask_f16), NAMES["soft_max"].format(t=t), "soft_max")
        n_head_log2 = 1 << int(np.floor(np.log2(nheads)))
        m0 = 2.0 ** (-max_bias / n_head_log2)
        m1 = 2.0 ** (-(max_bias / 2.0) / n_head_log2)
        esz = 2 if mask_f16 else 4
        params = np.zeros(1, dtype=[("nheads", "<i8"), ("n_head_log2", "<u4"), ("pad", "<u4"), ("ncols", "<i8"),
                                    ("nrows_x", "<i8"), ("nrows_y", "<i8"), ("ne00", "<i8"), ("ne01", "<i8"),
                                    ("ne02", "<i8"), ("ne03", "<i8"), ("nb11", "<i8"), ("nb12", "<i8"), ("nb13", "<i8"),
                                    ("ne12", "<i8"), ("ne13", "<i8"), ("scale", "<f4"), ("max_bias", "<f4"),
                                    ("m0", "<f4"), ("m1", "<f4")])
        params[0] = (nheads, n_head_log2, 0, ncols, ne01 * nheads, ne01, ncols, ne01, nheads, 1, ncols * esz,
                     ncols * ne01 * esz, ncols * ne01 * esz, 1, 1, scale, max_bias, m0, m1)
        vals = [("ptr", x), ("ptr", mask), ("ptr", sinks), ("ptr", dst), ("bytes", params.tobytes())]
        return self._go(p, (ne01, nheads, 1), (32, 1, 1), vals, stream, "soft_max_f32")


# ---------------------------------------------------------------------------------------------
# host-side weight quantizers (synthetic weights for tests and the benchmark)
# ---------------------------------------------------------------------------------------------
def mmq_skinny_group(ty, xs, y, dsts, nrows, k, ncols, ncols_y=None, stride_row_x=None, stride_col_dst=None,
                     stream=0):
    """cfi_mmq_skinny_group: products i (device pointers xs[i] -> dsts[i], nrows[i] rows each) over one
    q8_1_mmq activation buffer y in one launch; row strides default to k / block values, output
    column strides to nrows[i]."""
    n = len(xs)
    qk = 256 if ty == Q4_K else 32
    srx = stride_row_x or [k // qk] * n
    scd = stride_col_dst or list(nrows)
    P = C.c_void_p * n
    U = C.c_uint32 * n
    rc = lib().cfi_mmq_skinny_group(ty, n, P(*xs), C.c_void_p(y), P(*dsts), U(*nrows), U(*srx), U(*scd), k, ncols,
                                    ncols_y or ncols, C.c_void_p(stream))
    check(rc, "cfi_mmq_skinny_group")


PEER_HANDLE_BYTES = 64
PEER_MAX_RANKS = 8


class PeerSet(C.Structure):
    """cfi_peer.h's CfiPeerSet: a rank's view of its group."""
    _fields_ = [("rank", C.c_int), ("world", C.c_int), ("delta", C.c_longlong * PEER_MAX_RANKS),
                ("sig_remote", C.c_void_p * PEER_MAX_RANKS), ("sig_local", C.c_void_p), ("expect", C.c_void_p)]


class PeerGroup:
    """One peer buffer per rank of one node, each mapped into every rank's process (CUDA IPC over
    NVLink; cfi_peer.h): `nbytes` bytes of outputs at offset 0, then the ranks' signal slots and
    this rank's wait counts.  `exchange(obj)` returns every rank's obj in rank
    order (torch.distributed.all_gather_object, or any channel between the ranks).  A product
    launched with `peers` stores its outputs into every rank's copy at the same offset and ends
    once every rank's rows are here; barrier() is the group's signal and wait alone."""

    def __init__(self, rank, world, nbytes, exchange):
        if not 1 <= world <= PEER_MAX_RANKS or not 0 <= rank < world:
            raise ValueError("bad rank %d of %d" % (rank, world))
        self.rank, self.world = rank, world
        self.data_bytes = (nbytes + 255) // 256 * 256
        sig_off = self.data_bytes
        expect_off = sig_off + 4 * world
        L = lib()
        self.base = C.c_void_p()
        handle = C.create_string_buffer(PEER_HANDLE_BYTES)
        check(L.cfi_peer_alloc(expect_off + 4 * world + 256, C.byref(self.base), C.cast(handle, C.c_void_p)),
              "cfi_peer_alloc")
        self.ptrs, self._opened = [], []
        try:
            handles = exchange(handle.raw)
            for r, h in enumerate(handles):
                if r == rank:
                    self.ptrs.append(self.base.value)
                    continue
                p = C.c_void_p()
                check(L.cfi_peer_open(h, C.byref(p)), "cfi_peer_open")
                self._opened.append(p.value)
                self.ptrs.append(p.value)
        except Exception:
            self.close()
            raise
        ps = PeerSet()
        ps.rank, ps.world = rank, world
        for r in range(world):
            ps.delta[r] = self.ptrs[r] - self.base.value
            ps.sig_remote[r] = self.ptrs[r] + sig_off + 4 * rank
        ps.sig_local = self.base.value + sig_off
        ps.expect = self.base.value + expect_off
        self.peers = ps

    @property
    def data(self):
        """Device address of this rank's outputs."""
        return self.base.value

    def barrier(self, stream=0):
        check(lib().cfi_peer_barrier(C.byref(self.peers), C.c_void_p(stream)), "cfi_peer_barrier")

    def all_gather(self, src, nbytes, dst_off, stream=0):
        """Every rank's nbytes at device address src into [dst_off + r * nbytes) of every rank's
        data, ranks in order; returns once (on the stream) this rank's data holds them all."""
        check(lib().cfi_peer_all_gather(C.c_void_p(src), nbytes, C.c_void_p(self.data + dst_off), C.byref(self.peers),
                                        C.c_void_p(stream)), "cfi_peer_all_gather")

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (every rank synchronised first)."""
        L = lib()
        for p in self._opened:
            L.cfi_peer_close(C.c_void_p(p))
        self._opened = []
        if self.base.value:
            L.cfi_peer_free(self.base)
            self.base = C.c_void_p()


def mmq_skinny_group_peers(ty, xs, y, dsts, nrows, k, ncols, group, ncols_y=None, stride_row_x=None,
                           stride_col_dst=None, stream=0):
    """cfi_mmq_skinny_group_peers: mmq_skinny_group whose outputs (inside `group`'s data) are also
    stored into every other rank's copy; it ends once every rank's rows are here."""
    n = len(xs)
    qk = 256 if ty == Q4_K else 32
    srx = stride_row_x or [k // qk] * n
    scd = stride_col_dst or list(nrows)
    P = C.c_void_p * n
    U = C.c_uint32 * n
    rc = lib().cfi_mmq_skinny_group_peers(ty, n, P(*xs), C.c_void_p(y), P(*dsts), U(*nrows), U(*srx), U(*scd), k, ncols,
                                          ncols_y or ncols, C.byref(group.peers), C.c_void_p(stream))
    check(rc, "cfi_mmq_skinny_group_peers")


def quantize_q8_0(w):
    """ggml quantize_row_q8_0 over rows of `w` (float32, K % 32 == 0): d = amax/127 (fp16),
    q = round(x / d).  Returns uint8 [rows, K/32*34]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    b = w.reshape(rows, k // 32, 32)
    amax = np.abs(b).max(axis=2)
    d = amax / np.float32(127.0)
    inv = np.where(d != 0, np.float32(1.0) / np.where(d != 0, d, 1), 0).astype(np.float32)
    q = np.clip(np.round(b * inv[..., None]), -128, 127).astype(np.int8)
    out = np.empty((rows, k // 32, 34), dtype=np.uint8)
    out[..., 0:2] = d.astype(np.float16).view(np.uint8).reshape(rows, k // 32, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(rows, -1)


def quantize_q4_k(w):
    """Seeded-data Q4_K quantizer (256-value superblocks; 8 sub-blocks of 32 with 6-bit scale and
    min): x ~ d*sc*q - dmin*m, q in 0..15.  Returns uint8 [rows, K/256*144]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    nsb = k // 256
    x = w.reshape(rows, nsb, 8, 32)
    mn = np.minimum(x.min(axis=3), 0.0)
    mx = x.max(axis=3)
    scale = (mx - mn) / 15.0
    mins = -mn
    d = (scale.max(axis=2) / 63.0).astype(np.float16).astype(np.float32)
    dmin = (mins.max(axis=2) / 63.0).astype(np.float16).astype(np.float32)
    sc = np.where(d[..., None] > 0, np.round(scale / np.where(d[..., None] > 0, d[..., None], 1)), 0)
    sc = np.clip(sc, 0, 63).astype(np.uint8)
    m = np.where(dmin[..., None] > 0, np.round(mins / np.where(dmin[..., None] > 0, dmin[..., None], 1)), 0)
    m = np.clip(m, 0, 63).astype(np.uint8)
    eff_d = d[..., None] * sc
    eff_m = dmin[..., None] * m
    q = np.where(eff_d[..., None] > 0, np.round((x + eff_m[..., None]) / np.where(eff_d[..., None] > 0, eff_d[..., None], 1)), 0)
    q = np.clip(q, 0, 15).astype(np.uint8)
    out = np.zeros((rows, nsb, 144), dtype=np.uint8)
    out[..., 0:2] = d.astype(np.float16).view(np.uint8).reshape(rows, nsb, 2)
    out[..., 2:4] = dmin.astype(np.float16).view(np.uint8).reshape(rows, nsb, 2)
    s = np.zeros((rows, nsb, 12), dtype=np.uint8)
    for j in range(4):
        s[..., j] = (sc[..., j] & 63) | ((sc[..., j + 4] >> 4) << 6)
        s[..., j + 4] = (m[..., j] & 63) | ((m[..., j + 4] >> 4) << 6)
        s[..., j + 8] = (sc[..., j + 4] & 0xF) | ((m[..., j + 4] & 0xF) << 4)
    out[..., 4:16] = s
    for c in range(4):
        out[..., 16 + 32 * c:16 + 32 * (c + 1)] = q[..., 2 * c, :] | (q[..., 2 * c + 1, :] << 4)
    return out.reshape(rows, -1)


def synthetic_weights(ty, rows, k, seed, std=0.02):
    """Seeded N(0, std) float32 weights quantized to `ty` (Q8_0 or Q4_K)."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, std, size=(rows, k)).astype(np.float32)
    return quantize_q8_0(w) if ty == Q8_0 else quantize_q4_k(w)
