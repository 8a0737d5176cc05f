"""Generate tests/golden/golden.npz: frozen inputs and oracle outputs for the GPU parity tests.

The reference project ships no stored expected outputs; its known-answer tests are generator
based (xorshift64* Rng and random_blocks, src/subst/refs.rs:501-538; probe seeds
src/subst/probe.rs:356-393).  The cases below use those generators through the CPU oracle and
freeze both the inputs and the outputs, so a change of the oracle or of a kernel shows up as a
mismatch against committed bytes.  Run from the repository root:

    python tests/golden/make_golden.py
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import oracle_py as O  # noqa: E402

Q8_0, Q4_K = 8, 12

# (ty, ncols_dst, nrows, ncols_x, seed): probe-style shapes (probe.rs:33-78) and a ragged row count
MMVQ = [(Q8_0, 1, 11, 896, 0x5eed + Q8_0), (Q8_0, 3, 7, 512, 0x5eed + Q8_0 + 3), (Q8_0, 8, 5, 1024, 0xDEC0 + 8 + 5),
        (Q4_K, 1, 11, 512, 0x5eed + Q4_K), (Q4_K, 2, 9, 1024, 0x5eed + Q4_K + 2), (Q4_K, 8, 5, 768, 0xDEC0 + 12 + 5)]
# (ty, ncols_x, nrows, ncols, seed)
MMQ = [(Q8_0, 256, 70, 9, 0xfa77), (Q4_K, 512, 33, 5, 0xfa77 + 1)]


def mmvq_fields(p):
    return np.array([getattr(p, n) for n, _ in O.Mmvq._fields_], dtype=np.uint32)


def mmq_fields(p):
    return np.array([getattr(p, n) for n, _ in O.Mmq._fields_], dtype=np.uint32)


def main():
    out = {}
    # quantize_q8_1 (probe.rs:392-401, seed 0x3171): 3 rows of 640 values padded to 768
    x, ref = O.quantize_case(640, 768, 3, 1, 1, 0x3171)
    out["q81_x"], out["q81_y"], out["q81_shape"] = x, ref, np.array([640, 768, 3], dtype=np.int64)
    for i, (ty, nc, nr, nx, seed) in enumerate(MMVQ):
        p, xw, y, ids, n = O.mmvq_case(ty, nc, nr, nx, 1, 1, 1, False, seed)
        out["mmvq%d_p" % i] = mmvq_fields(p)
        out["mmvq%d_x" % i], out["mmvq%d_y" % i] = xw, y
        out["mmvq%d_fast" % i] = O.mmvq_fast_ref(p, xw, y, ids, n, 1, 1, True) if nc == 1 else per_column(p, xw, y, ids, n)
        out["mmvq%d_stock" % i] = O.mmvq_ref(p, xw, y, ids, n)
    rng = np.random.default_rng(0x71)
    xa = rng.normal(0, 1, size=(7, 512)).astype(np.float32)
    out["qmmq_x"] = xa
    out["qmmq_d4"] = O.quantize_mmq(Q8_0, xa, 512, 7)
    out["qmmq_ds4"] = O.quantize_mmq(Q4_K, xa, 512, 7)
    for i, (ty, nx, nr, nc, seed) in enumerate(MMQ):
        p, xw, y, n = O.mmq_case(ty, nx, nr, nc, 1, 1, 1, seed)
        out["mmq%d_p" % i] = mmq_fields(p)
        out["mmq%d_ty" % i] = np.array([ty], dtype=np.uint32)
        out["mmq%d_x" % i], out["mmq%d_y" % i] = xw, y
        out["mmq%d_dst" % i] = O.mmq_ref(ty, p, xw, y, n)
    xr = rng.normal(0, 1, size=(4, 896)).astype(np.float32)
    wr = rng.normal(1, 0.1, size=896).astype(np.float32)
    out["rms_x"], out["rms_w"] = xr, wr
    out["rms_y"] = O.rms_norm(xr, wr, 4, 896, 1e-6)
    xs = rng.normal(0, 3, size=(2 * 14, 631)).astype(np.float32)
    ms = rng.normal(0, 1, size=(2, 631)).astype(np.float32)
    out["sm_x"], out["sm_mask"] = xs, ms
    out["sm_y"] = O.soft_max(xs, ms, None, 631, 2, 14, 2 * 14, 0.125)
    xq = rng.normal(0, 1, size=(3, 16, 64)).astype(np.float32)   # 3 tokens x 16 heads x dim 64
    pos = np.array([0, 7, 630], dtype=np.int32)
    out["rope_x"], out["rope_pos"] = xq, pos
    out["rope_y"] = O.rope_neox(xq, 64, 16, 3, 64, pos, 1e6)
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", os.path.join(HERE, "golden.npz"), sum(v.nbytes for v in out.values()), "bytes raw")


def per_column(p, xw, y, ids, n):
    """Each output column through the one-warp whole-group model (refs.rs:435-497)."""
    res = np.zeros(n, dtype=np.float32)
    for c in range(p.ncols_dst):
        q = O.Mmvq.from_buffer_copy(p)
        q.ncols_dst = 1
        ysub = np.ascontiguousarray(y[c * p.stride_col_y * 36:])
        col = np.zeros(n, dtype=np.float32)
        O.lib().cfo_mmvq_fast(C.byref(q), O.u8(xw), O.u8(ysub), O.i32(ids), O.f32(col), 1, 1, 1)
        res[c * p.stride_col_dst:c * p.stride_col_dst + p.nrows_x] = col[:p.nrows_x]
    return res


if __name__ == "__main__":
    main()
