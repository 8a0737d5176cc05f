"""ctypes wrapper of the CPU oracle (oracle/liboracle.so) -- test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this module.
"""
import ctypes as C
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
LIB = os.path.join(ORACLE_DIR, "liboracle.so")


class Mmvq(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "ty", "ncols_dst", "nwarps", "nrows_x", "ncols_x", "nchannels_dst", "nsamples_dst", "channel_ratio",
        "sample_ratio", "nchannels_y", "use_ids", "stride_row_x", "stride_col_y", "stride_col_dst",
        "stride_channel_x", "stride_channel_y", "stride_channel_dst", "stride_sample_x", "stride_sample_y",
        "stride_sample_dst")]


class Mmq(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "ncols_x", "nrows_x", "ncols_dst", "nchannels_y", "nsamples_y", "channel_ratio", "sample_ratio",
        "stride_row_x", "ncols_y", "stride_col_dst", "stride_channel_x", "stride_channel_y", "stride_channel_dst",
        "stride_sample_x", "stride_sample_y", "stride_sample_dst")]


_o = None


def build():
    subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)


def use_native_build():
    """Rebuilds the oracle at -O3 -march=native for the host this runs on (`make native`, always
    rebuilt so a copy made on another machine is never used) and makes lib() load that copy.
    Only bench.py's CPU-baseline legs call this, before any other use of lib()."""
    global LIB
    if _o is not None:
        raise RuntimeError("the oracle is already loaded")
    subprocess.run(["make", "-s", "-B", "-C", ORACLE_DIR, "native"], check=True)
    LIB = os.path.join(ORACLE_DIR, "_native", "liboracle.so")


def lib():
    global _o
    if _o is None:
        srcs = [os.path.join(ORACLE_DIR, f) for f in ("cfi_oracle.c", "cfi_oracle.h", "cpu_baseline.c")]
        if os.path.dirname(LIB) == ORACLE_DIR and (
                not os.path.exists(LIB) or any(os.path.getmtime(s) > os.path.getmtime(LIB) for s in srcs)):
            build()
        _o = C.CDLL(LIB)
        u8p, f32p = C.POINTER(C.c_uint8), C.POINTER(C.c_float)
        _o.cfo_f16_to_f32.restype = C.c_float
        _o.cfo_f16_to_f32.argtypes = [C.c_uint16]
        _o.cfo_f32_to_f16.restype = C.c_uint16
        _o.cfo_f32_to_f16.argtypes = [C.c_float]
        _o.cfo_nmse.restype = C.c_double
        _o.cfo_vec_dot.restype = C.c_float
        _o.cfo_vec_dot.argtypes = [C.c_uint32, u8p, u8p, C.c_size_t, C.c_float]
        _o.cfo_vec_dot_wide.restype = C.c_float
        _o.cfo_vec_dot_wide.argtypes = [C.c_uint32, u8p, u8p, C.c_size_t, C.c_float]
        _o.cfo_dot_ref_f64.restype = C.c_double
        _o.cfo_dot_ref_f64.argtypes = [C.c_uint32, u8p, C.c_size_t, u8p, C.POINTER(C.c_double)]
        _o.cfo_rng_unit.restype = C.c_float
        _o.cfo_rng_u32.restype = C.c_uint32
        _o.cfo_rng_next.restype = C.c_uint64
        _o.cfo_dp4a.restype = C.c_int32
        _o.cfo_dp4a.argtypes = [C.c_uint32, C.c_uint32, C.c_int32]
        u32 = C.c_uint32
        _o.cfo_fattn_case.argtypes = [u32, u32, u32, u32, u32, u32, C.c_int, C.c_uint64, f32p, C.c_void_p, C.c_void_p,
                                      C.c_void_p]
        _o.cfo_fattn_case.restype = None
        _o.cfo_fattn_reference.argtypes = [u32, u32, u32, u32, u32, u32, f32p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_float, f32p]
        _o.cfo_fattn_reference.restype = None
        _o.cfo_fastdiv.restype = C.c_uint32
        _o.cfo_fastmodulo.restype = C.c_uint32
        _o.cfo_gemm_validate.restype = C.c_int
        _o.cfo_cpu_decode_step.restype = C.c_int
        _o.cfo_cpu_decode_step.argtypes = [C.c_uint32, u8p, C.c_size_t, C.c_size_t, f32p, C.c_size_t, u8p, f32p, C.c_int]
        _o.cfo_reference_gemm.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_void_p, C.c_int,
                                          C.c_int, C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_int, C.c_int]
        _o.cfo_rope_neox.argtypes = [f32p, f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.POINTER(C.c_int32),
                                     C.c_float, C.c_float, C.c_float, f32p]
        _o.cfo_soft_max.argtypes = [f32p, f32p, f32p, f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float,
                                    C.c_float]
        _o.cfo_rms_norm.argtypes = [f32p, f32p, f32p, C.c_size_t, C.c_size_t, C.c_float]
    return _o


def u8(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint8))


def f32(a):
    return a.ctypes.data_as(C.POINTER(C.c_float)) if a is not None else None


def i32(a):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def nmse(got, want):
    got = np.ascontiguousarray(got, dtype=np.float32)
    want = np.ascontiguousarray(want, dtype=np.float32)
    return lib().cfo_nmse(f32(got), f32(want), C.c_size_t(want.size))


def rel_l2(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    den = np.sqrt((want * want).sum())
    return float(np.sqrt(((got - want) ** 2).sum()) / den) if den > 0 else float(np.sqrt(((got - want) ** 2).sum()))


def quantize_q8_1(x):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(x.size // 32 * 36, dtype=np.uint8)
    lib().cfo_quantize_q8_1(f32(x), C.c_size_t(x.size), u8(out))
    return out


def quantize_mmq(ty, x, ne0, ncols):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(ne0 // 128 * ncols * 144, dtype=np.uint8)
    lib().cfo_quantize_mmq(C.c_uint32(ty), f32(x), C.c_size_t(ne0), C.c_size_t(ncols), u8(out))
    return out


def mmvq_case(ty, ncols_dst, nrows, ncols_x, nch, ratio, nsamples, use_ids, seed):
    """probe.rs:33-78 -> (params, x bytes, y bytes, ids, dst_len)."""
    L = lib()
    xb, yb, ni, dl = C.c_size_t(), C.c_size_t(), C.c_size_t(), C.c_size_t()
    L.cfo_mmvq_case_sizes(C.c_uint32(ty), C.c_uint32(ncols_dst), C.c_uint32(nrows), C.c_uint32(ncols_x),
                          C.c_uint32(nch), C.c_uint32(ratio), C.c_uint32(nsamples), C.c_int(int(use_ids)),
                          C.byref(xb), C.byref(yb), C.byref(ni), C.byref(dl))
    p = Mmvq()
    x = np.zeros(xb.value, dtype=np.uint8)
    y = np.zeros(yb.value, dtype=np.uint8)
    ids = np.zeros(max(1, ni.value), dtype=np.int32)
    L.cfo_mmvq_case(C.c_uint32(ty), C.c_uint32(ncols_dst), C.c_uint32(nrows), C.c_uint32(ncols_x), C.c_uint32(nch),
                    C.c_uint32(ratio), C.c_uint32(nsamples), C.c_int(int(use_ids)), C.c_uint64(seed), C.byref(p),
                    u8(x), u8(y), i32(ids))
    return p, x, y, ids, dl.value


def mmvq_ref(p, x, y, ids, dst_len, nwarps=None):
    q = Mmvq.from_buffer_copy(p)
    if nwarps is not None:
        q.nwarps = nwarps
    dst = np.zeros(dst_len, dtype=np.float32)
    lib().cfo_mmvq_run(C.byref(q), u8(x), u8(y), i32(ids), f32(dst))
    return dst


def mmvq_fast_ref(p, x, y, ids, dst_len, warps=1, unroll=1, wide=True):
    dst = np.zeros(dst_len, dtype=np.float32)
    lib().cfo_mmvq_fast(C.byref(p), u8(x), u8(y), i32(ids), f32(dst), C.c_uint32(warps), C.c_uint32(unroll),
                        C.c_int(int(wide)))
    return dst


def mmq_case(ty, ncols_x, nrows, ncols, nch, ratio, nsamples, seed):
    L = lib()
    xb, yb, dl = C.c_size_t(), C.c_size_t(), C.c_size_t()
    L.cfo_mmq_case_sizes(C.c_uint32(ty), C.c_uint32(ncols_x), C.c_uint32(nrows), C.c_uint32(ncols), C.c_uint32(nch),
                         C.c_uint32(ratio), C.c_uint32(nsamples), C.byref(xb), C.byref(yb), C.byref(dl))
    p = Mmq()
    x = np.zeros(xb.value, dtype=np.uint8)
    y = np.zeros(yb.value, dtype=np.uint8)
    L.cfo_mmq_case(C.c_uint32(ty), C.c_uint32(ncols_x), C.c_uint32(nrows), C.c_uint32(ncols), C.c_uint32(nch),
                   C.c_uint32(ratio), C.c_uint32(nsamples), C.c_uint64(seed), C.byref(p), u8(x), u8(y))
    return p, x, y, dl.value


def mmq_ref(ty, p, x, y, dst_len):
    dst = np.zeros(dst_len, dtype=np.float32)
    lib().cfo_mmq_ref(C.c_uint32(ty), C.byref(p), u8(x), u8(y), f32(dst))
    return dst


def quantize_case(ne00, ne0, ne1, ne2, ne3, seed):
    L = lib()
    x = np.zeros(ne00 * ne1 * ne2 * ne3, dtype=np.float32)
    L.cfo_quantize_case_x(C.c_size_t(ne00), C.c_size_t(ne1), C.c_size_t(ne2), C.c_size_t(ne3), C.c_uint64(seed), f32(x))
    rows = ne1 * ne2 * ne3
    ref = np.zeros(rows * ne0 // 32 * 36, dtype=np.uint8)
    L.cfo_quantize_case_reference(f32(x), C.c_size_t(ne00), C.c_size_t(ne0), C.c_size_t(rows), u8(ref))
    return x, ref


def dot_ref_f64(ty, row, nblocks, y):
    a = C.c_double()
    t = lib().cfo_dot_ref_f64(C.c_uint32(ty), u8(row), C.c_size_t(nblocks), u8(y), C.byref(a))
    return t, a.value


def rms_norm(x, w, rows, ncols, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(rows * ncols, dtype=np.float32)
    wv = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
    lib().cfo_rms_norm(f32(x), f32(wv), f32(out), C.c_size_t(rows), C.c_size_t(ncols), C.c_float(eps))
    return out


def rope_neox(x, ne0, ne1, nch, n_dims, pos, freq_base, freq_scale=1.0, attn_factor=1.0, ff=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    out = np.zeros_like(x)
    ffv = None if ff is None else np.ascontiguousarray(ff, dtype=np.float32)
    lib().cfo_rope_neox(f32(x), f32(out), ne0, ne1, nch, n_dims, i32(pos), C.c_float(freq_base),
                        C.c_float(freq_scale), C.c_float(attn_factor), f32(ffv))
    return out


def soft_max(x, mask, sinks, ncols, ne01, nheads, rows, scale, max_bias=0.0):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros_like(x)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    s = None if sinks is None else np.ascontiguousarray(sinks, dtype=np.float32)
    lib().cfo_soft_max(f32(x), f32(m), f32(s), f32(out), ncols, ne01, nheads, rows, C.c_float(scale),
                       C.c_float(max_bias))
    return out


def cpu_decode_step(ty, w, rows, ncols_x, x, ncols_dst, threads=0):
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    yq = np.zeros(ncols_dst * ncols_x // 32 * 36, dtype=np.uint8)
    dst = np.zeros(ncols_dst * rows, dtype=np.float32)
    used = lib().cfo_cpu_decode_step(C.c_uint32(ty), u8(w), rows, ncols_x, f32(x), ncols_dst, u8(yq), f32(dst), threads)
    return dst, yq, used


def fattn_case(d, nq, nh, nh_kv, nkv, ns, causal, seed):
    """src/subst/probe.rs:421-446: Q f32 [ns][nh][nq][d], K/V f16 bits [ns][nh_kv][nkv][d], mask f16
    bits [ns][nq_pad][nkv] (None without a mask)."""
    q = np.zeros(d * nq * nh * ns, dtype=np.float32)
    k = np.zeros(d * nkv * nh_kv * ns, dtype=np.uint16)
    v = np.zeros_like(k)
    nq_pad = (nq + 15) // 16 * 16
    m = np.zeros(nkv * nq_pad * ns, dtype=np.uint16) if causal else None
    lib().cfo_fattn_case(d, nq, nh, nh_kv, nkv, ns, int(causal), C.c_uint64(seed), f32(q),
                         k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p),
                         m.ctypes.data_as(C.c_void_p) if m is not None else None)
    return q, k, v, m


def fattn_reference(d, nq, nh, nh_kv, nkv, ns, q, k, v, m, scale):
    """Exact softmax attention in f64 (probe.rs:451-487); dst [ns][nq][nh][d] f32."""
    out = np.zeros(d * nh * nq * ns, dtype=np.float32)
    lib().cfo_fattn_reference(d, nq, nh, nh_kv, nkv, ns, f32(q), k.ctypes.data_as(C.c_void_p),
                              v.ctypes.data_as(C.c_void_p), m.ctypes.data_as(C.c_void_p) if m is not None else None,
                              C.c_float(scale), f32(out))
    return out
