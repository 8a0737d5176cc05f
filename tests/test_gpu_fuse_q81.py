"""GPU tests of the router's context modes.  CFI_CTX_CONST_WEIGHTS (weights copied before the
programmatic-dependent-launch wait) must not change a bit of any GEMV result.  The deferred
quantize_q8_1 (CFI_CTX_DEFER_Q8_1): the streaming mul_mat_vec_q that
absorbs the quantize must leave memory exactly as the two separate native launches do -- the
same q8_1 bytes in the quantizer's output buffer (byte-exact to the oracle, src/subst/refs.rs:
117-147) and the same GEMV outputs bit for bit -- for every GEMV type and column count, padded
rows (ne00 < ne0), unaligned activation rows, inside a CUDA graph, and when the held-back
quantize is launched on its own (flush, or a GEMV that reads something else)."""
import numpy as np
import pytest

import cfi_b200 as cfi
import oracle_py as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TYPES = [cfi.Q8_0, cfi.Q4_K, cfi.Q6_K, cfi.Q4_0]


@pytest.fixture(scope="module")
def ctxs():
    assert torch.cuda.is_available()
    plain = cfi.Ctx(0)
    fused = cfi.Ctx(0, defer_q8_1=True)
    yield cfi.GgmlCaller(plain, "all"), cfi.GgmlCaller(fused, "all"), fused
    fused.close()
    plain.close()


@pytest.mark.parametrize("ty", TYPES)
@pytest.mark.parametrize("direct", ["0", "1"])
def test_const_weights_gemv_equals_plain(ctxs, monkeypatch, ty, direct):
    """Weights fetched before the wait, in a chain of dependent GEMVs (each reads the previous
    one's output as its activations after a quantize), on both fill paths."""
    monkeypatch.setenv("CFI_MMVQ_DIRECT", direct)
    gp = ctxs[0]
    cw = cfi.Ctx(0, const_weights=True)
    gc = cfi.GgmlCaller(cw, "all")
    for ncols in (1, 2, 5, 8):
        w, x, ne00, ne0, s01 = case(ty, ncols, 1024, 1024, 0, 3 + ty + ncols)
        outs = []
        for g in (gp, gc):
            s = torch.cuda.current_stream().cuda_stream
            dw, dx = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
            dq = torch.zeros(ncols * ne0 // 32 * 36, dtype=torch.uint8, device="cuda")
            dd = torch.zeros(ncols * 1024, device="cuda")
            for _ in range(3):  # out = W q8_1(x); x = out, three times
                g.quantize_q8_1(dx.data_ptr(), dq.data_ptr(), ne00, ne0, ncols, stream=s)
                g.mmvq(ty, ncols, dw.data_ptr(), dq.data_ptr(), dd.data_ptr(), 1024, 1024, stream=s)
                dx = dd.clone() / (dd.abs().max() + 1.0)
            torch.cuda.synchronize()
            outs.append(dd.cpu().numpy())
        assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
        assert np.isfinite(outs[0]).all()
    assert cw.stats()["stock_launches"] == 0
    cw.close()


def run(g, ty, ncols, w, x, nrows, ncols_x, ne00, ne0, s01, flush=None):
    s = torch.cuda.current_stream().cuda_stream
    dw, dx = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    dq = torch.full((ncols * ne0 // 32 * 36,), 0xAB, dtype=torch.uint8, device="cuda")
    dd = torch.full((ncols * nrows,), float("nan"), device="cuda")
    g.quantize_q8_1(dx.data_ptr(), dq.data_ptr(), ne00, ne0, ncols, s01=s01, stream=s)
    g.mmvq(ty, ncols, dw.data_ptr(), dq.data_ptr(), dd.data_ptr(), ncols_x, nrows, stride_col_y=ne0 // 32, stream=s)
    if flush:
        flush()
    torch.cuda.synchronize()
    assert cfi.lib().cfi_device_error() == 0
    return dq.cpu().numpy(), dd.cpu().numpy()


def case(ty, ncols, nrows, ncols_x, pad, seed):
    p, w, _, _, _ = O.mmvq_case(ty, ncols, nrows, ncols_x, 1, 1, 1, False, seed)
    ne00 = ncols_x
    ne0 = (ne00 + pad + 31) // 32 * 32
    s01 = ne00 + 3 if pad else ne00  # an unaligned row stride when padded
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, size=ncols * s01).astype(np.float32)
    return w, x, ne00, ne0, s01


@pytest.mark.parametrize("ty", TYPES)
@pytest.mark.parametrize("ncols", [1, 2, 3, 4])
@pytest.mark.parametrize("direct", ["0", "1"])
def test_fused_quantize_gemv_equals_separate_launches(ctxs, monkeypatch, ty, ncols, direct):
    monkeypatch.setenv("CFI_DEFER_MAX_VALUES", "1048576")  # absorb every case here
    monkeypatch.setenv("CFI_MMVQ_DIRECT", direct)
    # absorption is built on the decode-fast kernels (Q4_K with 3+ columns otherwise takes the
    # tensor-core GEMV, which does not absorb)
    monkeypatch.setenv("CFI_MMVQ_EXACT", "1")
    gp, gf, fctx = ctxs
    for nrows, ncols_x, pad in [(8192, 2048, 0), (300, 4096, 0), (37, 512, 512)]:
        w, x, ne00, ne0, s01 = case(ty, ncols, nrows, ncols_x, pad, 11 + ty + ncols + nrows)
        before = fctx.stats()["fused_q8_1"]
        q_ref, d_ref = run(gp, ty, ncols, w, x, nrows, ncols_x, ne00, ne0, s01)
        q, d = run(gf, ty, ncols, w, x, nrows, ncols_x, ne00, ne0, s01)
        assert fctx.stats()["fused_q8_1"] == before + 1
        assert np.array_equal(q, q_ref), "%d q8_1 bytes differ" % (q != q_ref).sum()
        assert np.array_equal(d.view(np.uint32), d_ref.view(np.uint32))
        if pad == 0 and s01 == ne00:
            assert np.array_equal(q, O.quantize_q8_1(x))  # the oracle's bytes


def test_fused_prologue_threshold(ctxs):
    """By default only one-pass prologues are absorbed (1 x 1024 values here, not 2 x 1024)."""
    gp, gf, fctx = ctxs
    for ncols, absorbed in ((1, 1), (2, 0)):
        w, x, ne00, ne0, s01 = case(cfi.Q4_K, ncols, 512, 1024, 0, 9)
        before = fctx.stats()["fused_q8_1"]
        q_ref, d_ref = run(gp, cfi.Q4_K, ncols, w, x, 512, 1024, ne00, ne0, s01)
        q, d = run(gf, cfi.Q4_K, ncols, w, x, 512, 1024, ne00, ne0, s01)
        assert fctx.stats()["fused_q8_1"] == before + absorbed
        assert np.array_equal(q, q_ref) and np.array_equal(d.view(np.uint32), d_ref.view(np.uint32))


def test_flush_and_unmatched_gemv(ctxs):
    gp, gf, fctx = ctxs
    w, x, ne00, ne0, s01 = case(cfi.Q4_K, 2, 512, 2048, 0, 5)
    q_ref, d_ref = run(gp, cfi.Q4_K, 2, w, x, 512, 2048, ne00, ne0, s01)
    # quantize alone, then flush: the buffer is the quantizer's
    s = torch.cuda.current_stream().cuda_stream
    dx = torch.from_numpy(x).cuda()
    dq = torch.zeros(q_ref.size, dtype=torch.uint8, device="cuda")
    gf.quantize_q8_1(dx.data_ptr(), dq.data_ptr(), ne00, ne0, 2, stream=s)
    fctx.flush()
    torch.cuda.synchronize()
    assert np.array_equal(dq.cpu().numpy(), q_ref)
    # a GEMV on another buffer: the quantize runs first, on its own
    dq.zero_()
    other = torch.from_numpy(q_ref).cuda()
    dw = torch.from_numpy(w).cuda()
    dd = torch.zeros(2 * 512, device="cuda")
    before = fctx.stats()["fused_q8_1"]
    gf.quantize_q8_1(dx.data_ptr(), dq.data_ptr(), ne00, ne0, 2, stream=s)
    gf.mmvq(cfi.Q4_K, 2, dw.data_ptr(), other.data_ptr(), dd.data_ptr(), 2048, 512, stream=s)
    torch.cuda.synchronize()
    assert fctx.stats()["fused_q8_1"] == before
    assert np.array_equal(dq.cpu().numpy(), q_ref)
    assert np.array_equal(dd.cpu().numpy().view(np.uint32), d_ref.view(np.uint32))


def test_fused_in_a_cuda_graph(ctxs):
    gp, gf, fctx = ctxs
    w, x, ne00, ne0, s01 = case(cfi.Q8_0, 1, 4864, 896, 128, 21)
    q_ref, d_ref = run(gp, cfi.Q8_0, 1, w, x, 4864, 896, ne00, ne0, s01)
    run(gf, cfi.Q8_0, 1, w, x, 4864, 896, ne00, ne0, s01)  # first use (probe) outside the capture
    dw, dx = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    dq = torch.zeros(q_ref.size, dtype=torch.uint8, device="cuda")
    dd = torch.zeros(4864, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        s = torch.cuda.current_stream().cuda_stream
        gf.quantize_q8_1(dx.data_ptr(), dq.data_ptr(), ne00, ne0, 1, s01=s01, stream=s)
        gf.mmvq(cfi.Q8_0, 1, dw.data_ptr(), dq.data_ptr(), dd.data_ptr(), 896, 4864, stride_col_y=ne0 // 32, stream=s)
        fctx.flush()
    for _ in range(3):
        dq.zero_()
        dd.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert np.array_equal(dq.cpu().numpy(), q_ref)
        assert np.array_equal(dd.cpu().numpy().view(np.uint32), d_ref.view(np.uint32))
    del graph
