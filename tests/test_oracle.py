"""Checks of the CPU oracle itself (no GPU).

The reference ships no golden output vectors for this path, so the oracle is pinned by
(a) independent restatements of the primitive steps (Python integer xorshift, numpy float16,
integer division), (b) the invariants the reference's own tests assert (stock-order vs
decode-fast mmvq nmse < 1e-10, src/subst/tests.rs:543-597), and (c) the reference's second
opinion: the f64 dequantised dot of src/ptx/ggml_ref.rs.
"""
import ctypes as C

import numpy as np
import pytest

import oracle_py as O

Q4_0, Q8_0, Q4_K, Q6_K = 2, 8, 12, 14


def test_f16_conversions_match_numpy_round_to_nearest_even():
    L = O.lib()
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.normal(0, 1, 4000), rng.normal(0, 1e-5, 2000), rng.normal(0, 3e4, 1000),
                           [0.0, -0.0, 65504.0, 65520.0, 1e-8, 5.96e-8, 2.98e-8, np.inf, -np.inf]]).astype(np.float32)
    for v in vals:
        assert L.cfo_f32_to_f16(C.c_float(v)) == int(np.float16(v).view(np.uint16)), v
    for h in range(0, 65536, 7):
        f = L.cfo_f16_to_f32(C.c_uint16(h))
        want = np.uint16(h).view(np.float16).astype(np.float32)
        assert (np.isnan(f) and np.isnan(want)) or f == want


def test_fastdiv_matches_integer_division():
    L = O.lib()
    rng = np.random.default_rng(2)
    for d in [1, 2, 3, 5, 7, 14, 28, 100, 151936, 65535, 1 << 20]:
        v = (C.c_uint32 * 3)()
        L.cfo_fastdiv_values(C.c_uint32(d), v)
        for n in list(rng.integers(0, 1 << 31, 200)) + [0, d - 1, d, d + 1]:
            n = int(n)
            assert L.cfo_fastdiv(C.c_uint32(n), v) == n // d
            assert L.cfo_fastmodulo(C.c_uint32(n), v) == n % d


def test_dp4a_matches_signed_byte_dot():
    L = O.lib()
    rng = np.random.default_rng(3)
    for _ in range(500):
        a, b = (int(x) for x in rng.integers(0, 1 << 32, 2))
        c = int(rng.integers(-(1 << 20), 1 << 20))
        av = np.frombuffer(a.to_bytes(4, "little"), dtype=np.int8).astype(np.int64)
        bv = np.frombuffer(b.to_bytes(4, "little"), dtype=np.int8).astype(np.int64)
        assert L.cfo_dp4a(a, b, c) == int((av * bv).sum()) + c


def test_rng_is_xorshift64_star():
    L = O.lib()
    s = C.c_uint64(0x5eed + 8)
    x = 0x5eed + 8
    for _ in range(100):
        x ^= x >> 12
        x ^= (x << 25) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 27
        want = (x * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF
        assert L.cfo_rng_next(C.byref(s)) == want


def _quantize_q8_1_numpy(x):
    """Independent restatement of refs.rs:117-147 in numpy."""
    out = np.zeros(x.size // 32 * 36, dtype=np.uint8)
    for ib in range(x.size // 32):
        c = x[ib * 32:(ib + 1) * 32].astype(np.float32)
        s = c.copy()
        for off in (16, 8, 4, 2, 1):
            s = (s + s[np.arange(32) ^ off]).astype(np.float32)
        amax = np.float32(np.abs(c).max())
        d = np.float32(amax / np.float32(127.0))
        out[ib * 36:ib * 36 + 2] = np.frombuffer(np.float16(d).tobytes(), np.uint8)
        out[ib * 36 + 2:ib * 36 + 4] = np.frombuffer(np.float16(s[0]).tobytes(), np.uint8)
        if amax != 0:
            t = (c / d).astype(np.float32)
            q = (np.sign(t) * np.floor(np.abs(t) + np.float32(0.5))).astype(np.int32).astype(np.int8)
            out[ib * 36 + 4:ib * 36 + 36] = q.view(np.uint8)
    return out


def test_quantize_q8_1_matches_an_independent_numpy_restatement():
    x, ref = O.quantize_case(96, 128, 3, 2, 1, 0x71)
    rows = []
    for r in range(6):
        row = np.zeros(128, dtype=np.float32)
        row[:96] = x[r * 96:(r + 1) * 96]
        rows.append(row)
    want = np.concatenate([_quantize_q8_1_numpy(r) for r in rows])
    assert np.array_equal(ref, want)
    # the all-zero and x1e-6 blocks of the probe case (probe.rs:185-191)
    assert ref[0:36].tolist() == [0] * 36
    assert np.frombuffer(ref[36:38].tobytes(), np.float16)[0] != 0


@pytest.mark.parametrize("ty", [Q8_0, Q4_0, Q4_K, Q6_K])
def test_stock_order_and_decode_fast_orders_agree(ty):
    """tests.rs:566-582: the decode-fast model is bitwise its own reference and within 1e-10 nmse of
    the stock order, at 11 rows and partial unroll steps."""
    fasts = [(1, 2, 1024), (2, 1, 2304), (1, 3, 2304), (4, 4, 512), (2, 8, 2304)]
    for warps, unroll, ncols_x in fasts:
        p, x, y, ids, n = O.mmvq_case(ty, 1, 11, ncols_x, 1, 1, 1, False, 31 + ty)
        stock = O.mmvq_ref(p, x, y, ids, n, nwarps=4)
        for wide in ([False, True] if ty != Q4_0 else [False]):
            got = O.mmvq_fast_ref(p, x, y, ids, n, warps, unroll, wide)
            assert O.nmse(got, stock) < 1e-10
            assert np.all(got != 0)


@pytest.mark.parametrize("ty", [Q8_0, Q4_K])
def test_multi_column_channels_samples_and_ids(ty):
    for ncols in (2, 5, 8):
        p, x, y, ids, n = O.mmvq_case(ty, ncols, 5, 512, 1, 1, 1, False, 11 + ty + ncols)
        want = O.mmvq_ref(p, x, y, ids, n)
        assert np.any(want != 0)
        # each column equals a one-column problem over that column's q8_1 blocks
        for c in range(ncols):
            col = O.mmvq_ref(p, x, y, ids, n, nwarps=8)[c * 5:(c + 1) * 5]
            assert O.nmse(col, want[c * 5:(c + 1) * 5]) < 1e-10
    p, x, y, ids, n = O.mmvq_case(ty, 1, 3, 512, 4, 2, 2, False, 99)
    a = O.mmvq_ref(p, x, y, ids, n)
    b = O.mmvq_fast_ref(p, x, y, ids, n, 1, 1, True)
    assert O.nmse(b, a) < 1e-10
    p, x, y, ids, n = O.mmvq_case(ty, 1, 3, 512, 5, 1, 1, True, 100)
    a = O.mmvq_ref(p, x, y, ids, n)
    b = O.mmvq_fast_ref(p, x, y, ids, n, 1, 1, True)
    assert O.nmse(b, a) < 1e-10 and np.any(a != 0)


@pytest.mark.parametrize("ty", [Q8_0, Q4_0, Q4_K, Q6_K])
def test_vec_dot_agrees_with_the_f64_second_opinion(ty):
    """src/ptx/ggml_ref.rs:384-446: f64 dequantised dot of a row against q8_1 blocks."""
    qk = 32 if ty in (Q8_0, Q4_0) else 256
    for seed in range(4):
        p, x, y, ids, n = O.mmvq_case(ty, 1, 3, 2048, 1, 1, 1, False, 1000 + seed)
        got = O.mmvq_ref(p, x, y, ids, n)
        bb = {Q8_0: 34, Q4_0: 18, Q4_K: 144, Q6_K: 210}[ty]
        nb = 2048 // qk
        for r in range(3):
            row = np.ascontiguousarray(x[r * nb * bb:(r + 1) * nb * bb])
            t, a = O.dot_ref_f64(ty, row, nb, y)
            assert abs(got[r] - t) <= 2e-6 * a + 1e-30, (ty, r, got[r], t, a)


def test_mmq_reference_agrees_with_f64_dequantised_dot():
    for ty in (Q8_0, Q4_K):
        ncols_x = 512
        p, x, y, n = O.mmq_case(ty, ncols_x, 70, 9, 1, 1, 1, 5 + ty)
        got = O.mmq_ref(ty, p, x, y, n).reshape(9, 70)
        groups = 8 if ty == Q4_K else 1
        bb = 144 if ty == Q4_K else 34
        nb = ncols_x // 32 // groups
        yb = y.reshape(ncols_x // 128, 9, 144)
        for col in (0, 4, 8):
            # rebuild the column's activations as dequantised values from block_q8_1_mmq
            acts = np.zeros(ncols_x)
            sums = np.zeros(ncols_x // 32)
            for kb in range(ncols_x // 32):
                blk = yb[kb // 4, col]
                if ty == Q4_K:
                    d = np.frombuffer(blk[4 * (kb % 4):4 * (kb % 4) + 2].tobytes(), np.float16)[0]
                    sums[kb] = np.frombuffer(blk[4 * (kb % 4) + 2:4 * (kb % 4) + 4].tobytes(), np.float16)[0]
                else:
                    d = np.frombuffer(blk[4 * (kb % 4):4 * (kb % 4) + 4].tobytes(), np.float32)[0]
                q = blk[16 + 32 * (kb % 4):16 + 32 * (kb % 4 + 1)].view(np.int8).astype(np.float64)
                acts[kb * 32:(kb + 1) * 32] = q * float(d)
            for row in (0, 33, 69):
                blocks = x[row * nb * bb:(row + 1) * nb * bb].reshape(nb, bb)
                w = np.zeros(ncols_x)
                wmin = np.zeros(ncols_x // 32)
                for b in range(nb):
                    if ty == Q8_0:
                        d = float(np.frombuffer(blocks[b, :2].tobytes(), np.float16)[0])
                        w[b * 32:(b + 1) * 32] = blocks[b, 2:].view(np.int8) * d
                    else:
                        d = float(np.frombuffer(blocks[b, 0:2].tobytes(), np.float16)[0])
                        dmin = float(np.frombuffer(blocks[b, 2:4].tobytes(), np.float16)[0])
                        s = blocks[b, 4:16]
                        for g in range(8):
                            if g < 4:
                                sc, m = s[g] & 63, s[g + 4] & 63
                            else:
                                sc = (s[g + 4] & 0xF) | ((s[g - 4] >> 6) << 4)
                                m = (s[g + 4] >> 4) | ((s[g] >> 6) << 4)
                            qs = blocks[b, 16 + 32 * (g // 2):16 + 32 * (g // 2 + 1)]
                            q = (qs & 15) if g % 2 == 0 else (qs >> 4)
                            w[(b * 8 + g) * 32:(b * 8 + g + 1) * 32] = float(np.float16(d * sc)) * q
                            wmin[b * 8 + g] = float(np.float16(-dmin * m))
                want = float((w * acts).sum() + (wmin * sums).sum())
                scale = float(np.abs(w * acts).sum() + np.abs(wmin * sums).sum())
                assert abs(got[col, row] - want) <= 1e-5 * scale


def test_gemm_validation_follows_cublas():
    """crates/cublas_shim/src/plan.rs:160-215."""
    V = O.lib().cfo_gemm_validate
    T, N = 1, 0
    R32F, R16F, R16BF = 0, 2, 14
    assert V(T, N, 4864, 631, 896, 896, 896, 4864, R16F, R16F, R32F, 68) == 0
    assert V(T, N, -1, 1, 1, 1, 1, 1, R16F, R16F, R32F, 68) == 7
    assert V(3, N, 1, 1, 1, 1, 1, 1, R16F, R16F, R32F, 68) == 7
    assert V(T, N, 4, 4, 8, 4, 8, 4, R16F, R16F, R32F, 68) == 7  # lda < k for op(A)=T
    assert V(N, N, 4, 4, 8, 4, 8, 3, R16F, R16F, R32F, 68) == 7  # ldc < m
    assert V(N, N, 4, 4, 8, 4, 8, 4, R16F, R16BF, R32F, 68) == 15
    assert V(N, N, 4, 4, 8, 4, 8, 4, R32F, R32F, R16F, 68) == 15
    assert V(N, N, 4, 4, 8, 4, 8, 4, R16F, R16F, R32F, 64) == 15  # 16F compute needs f16 out
    assert V(N, N, 4, 4, 8, 4, 8, 4, R16F, R16F, R16F, 64) == 0
    assert V(N, N, 4, 4, 8, 4, 8, 4, R16BF, R16BF, R32F, 2) == 15
    assert V(N, N, 0, 0, 0, 1, 1, 1, R32F, R32F, R32F, 0) == 0


def test_reference_gemm_matches_numpy():
    rng = np.random.default_rng(5)
    m, n, k = 13, 7, 33
    a = rng.normal(size=(m, k)).astype(np.float16)  # op(A) = A^T stored k x m column-major
    b = rng.normal(size=(k, n)).astype(np.float16)
    a_store = np.ascontiguousarray(a)  # row i contiguous along k == column-major k x m
    b_store = np.ascontiguousarray(b.T)  # column j contiguous along k
    c = np.zeros((n, m), dtype=np.float32)
    O.lib().cfo_reference_gemm(1, 0, m, n, k, C.c_float(1.0), a_store.ctypes.data, 2, k, b_store.ctypes.data, k,
                               C.c_float(0.0), c.ctypes.data, 0, m)
    want = a.astype(np.float32) @ b.astype(np.float32)
    assert np.allclose(c.T, want, rtol=1e-4, atol=1e-4)


def test_row_op_references():
    rng = np.random.default_rng(6)
    x = rng.normal(size=(4, 32)).astype(np.float32)
    got = O.rms_norm(x, None, 4, 32, 1e-5).reshape(4, 32)
    want = x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + 1e-5)
    assert np.allclose(got, want, rtol=2e-6, atol=1e-6)
    # rope: position 0 is the identity; rotation preserves each pair's norm
    xs = rng.normal(size=(3, 2, 64)).astype(np.float32)
    out = O.rope_neox(xs, 64, 2, 3, 64, np.array([0, 3, 631]), 1e6).reshape(3, 2, 64)
    assert np.allclose(out[0], xs[0])
    n_in = xs[..., :32] ** 2 + xs[..., 32:] ** 2
    n_out = out[..., :32] ** 2 + out[..., 32:] ** 2
    assert np.allclose(n_in, n_out, rtol=1e-5)
    # softmax rows sum to one; the masked column gets zero weight
    s = 0.03 * (np.arange(24) % 23) - 0.2
    mask = np.zeros(12, dtype=np.float32)
    mask[11] = -np.inf
    sm = O.soft_max(s.astype(np.float32), mask, None, 12, 1, 2, 2, 0.125).reshape(2, 12)
    assert np.allclose(sm.sum(axis=1), 1.0, atol=1e-6) and np.all(sm[:, 11] == 0)


def test_cpu_decode_step_equals_the_decode_fast_model():
    for ty in (Q8_0, Q4_K):
        p, x, y, ids, n = O.mmvq_case(ty, 1, 37, 1024, 1, 1, 1, False, 77)
        rng = np.random.default_rng(7)
        acts = rng.normal(size=1024).astype(np.float32)
        dst, yq, used = O.cpu_decode_step(ty, x, 37, 1024, acts, 1, threads=3)
        assert used == 3
        want = O.mmvq_fast_ref(p, x, yq, ids, n, 1, 1, True)
        assert np.array_equal(dst, want)
