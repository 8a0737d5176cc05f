"""Host-side tests of the cuBLAS-compatible GEMM API (no GPU): validation follows cuBLAS exactly
as the reference's shim does (crates/cublas_shim/src/plan.rs:160-215), handle state."""
import ctypes as C
import itertools

import cfi_b200 as cfi
import oracle_py as O


def test_validation_matches_the_reference_semantics_everywhere():
    L, V = cfi.lib(), O.lib().cfo_gemm_validate
    types = [0, 2, 14, 3]
    computes = [64, 65, 68, 69, 74, 75, 77, 0, 2, 70]
    dims = [(4, 4, 8), (0, 0, 0), (-1, 2, 2), (5, 7, 3)]
    lds = [1, 4, 8]
    n = 0
    for (ta, tb) in itertools.product([0, 1, 2, 3], [0, 1]):
        for (m, nn, k) in dims:
            for lda, ldb, ldc in itertools.product(lds, lds, lds):
                for at, ct in itertools.product(types, types):
                    for comp in computes[:: 3 if (lda, ldb, ldc) != (8, 8, 8) else 1]:
                        args = (ta, tb, m, nn, k, lda, ldb, ldc, at, at, ct, comp)
                        assert L.cfi_blas_validate(*args) == V(*args), args
                        n += 1
    assert n > 1000
    assert L.cfi_blas_validate(1, 0, 4864, 631, 896, 896, 896, 4864, 2, 2, 0, 68) == 0


def test_handle_state_and_errors():
    L = cfi.lib()
    h = C.c_void_p()
    assert L.cfi_blas_create(C.byref(h)) == 0
    assert L.cfi_blas_set_stream(h, C.c_void_p(1234)) == 0
    s = C.c_void_p()
    assert L.cfi_blas_get_stream(h, C.byref(s)) == 0 and s.value == 1234
    assert L.cfi_blas_set_pointer_mode(h, 2) == 7 and L.cfi_blas_set_pointer_mode(h, 1) == 0
    # invalid arguments are refused before anything touches the device
    one = C.byref(C.c_float(1.0))
    assert L.cfi_blas_gemm_ex(h, 1, 0, -1, 1, 1, one, None, 2, 1, None, 2, 1, one, None, 0, 1, 68, -1) == 7
    assert L.cfi_blas_gemm_ex(h, 1, 0, 4, 4, 4, one, None, 2, 4, None, 14, 4, one, None, 0, 4, 68, -1) == 15
    assert L.cfi_blas_gemm_strided_batched_ex(h, 1, 0, 4, 4, 4, one, None, 2, 4, 0, None, 2, 4, 0, one, None, 0, 4, 0,
                                              -1, 68, -1) == 7
    # empty problems succeed without launching anything
    assert L.cfi_blas_gemm_ex(h, 1, 0, 0, 4, 4, one, None, 2, 4, None, 2, 4, one, None, 0, 1, 68, -1) == 0
    assert L.cfi_blas_last_path(h) == 0
    assert L.cfi_blas_destroy(h) == 0
    assert L.cfi_blas_gemm_ex(None, 1, 0, 4, 4, 4, one, None, 2, 4, None, 2, 4, one, None, 0, 4, 68, -1) == 1
