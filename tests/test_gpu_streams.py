"""Calls on two streams of one GPU at the same time.

The kernels that combine partial results across CTAs (the split single-token attention and the
multi-CTA argmax of the decode glue, the GEMVs whose last CTA runs a fused decode step) and the
tensor-core GEMMs that split K or stage fp16 activations keep that scratch per (device, stream).
Each test enqueues the same entry point on two streams with different inputs, many times without
synchronising in between, and checks every result against the same call run alone: a shared
buffer or counter would mix the two streams' partials."""
import ctypes

import numpy as np
import pytest

import cfi_b200 as cfi
import oracle_py as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROUNDS = 12


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def streams():
    assert torch.cuda.is_available()
    torch.cuda.set_device(0)
    return torch.cuda.Stream(), torch.cuda.Stream()


def test_attention_and_argmax_on_two_streams(streams):
    L = cfi.lib()
    nh, nkvh, hd, n_ctx = 14, 2, 64, 8192  # 64 position ranges per head: many partials to combine
    cases = []
    for seed in (1, 2):
        gen = torch.Generator(device="cuda").manual_seed(seed)
        q = torch.randn(nh * hd, generator=gen, device="cuda")
        kc = torch.randn(nkvh, n_ctx, hd, generator=gen, device="cuda").half()
        vc = torch.randn(nkvh, hd, n_ctx, generator=gen, device="cuda").half()
        pos = torch.tensor([n_ctx - 1 - 37 * seed], dtype=torch.int32, device="cuda")
        logits = torch.randn(151936, generator=gen, device="cuda")
        cases.append(dict(q=q, kc=kc, vc=vc, pos=pos, logits=logits))
    torch.cuda.synchronize()
    scale = ctypes.c_float(1.0 / hd ** 0.5)

    def enqueue(c, st, out, tok, ppos):
        s = ctypes.c_void_p(st.cuda_stream)
        assert L.cfi_fused_attention_q8_1(_p(c["q"]), _p(c["kc"]), _p(c["vc"]), _p(c["pos"]), _p(out), nh, nkvh, hd,
                                          n_ctx, scale, s) == 0
        assert L.cfi_glue_argmax_next(_p(c["logits"]), 151936, _p(tok), _p(ppos), s) == 0

    # each case alone, one after the other
    want = []
    for c in cases:
        out = torch.zeros(nh * hd // 32 * 36, dtype=torch.uint8, device="cuda")
        tok = torch.zeros(1, dtype=torch.int32, device="cuda")
        ppos = torch.zeros(1, dtype=torch.int32, device="cuda")
        enqueue(c, streams[0], out, tok, ppos)
        torch.cuda.synchronize()
        want.append((out.clone(), int(tok.item())))
    assert want[0][1] == int(torch.argmax(cases[0]["logits"]).item())
    # both at once: ROUNDS launches on each stream, interleaved, no synchronisation in between
    outs = [[torch.zeros(nh * hd // 32 * 36, dtype=torch.uint8, device="cuda") for _ in range(ROUNDS)] for _ in cases]
    toks = [[torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(ROUNDS)] for _ in cases]
    ppos = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in cases]
    torch.cuda.synchronize()
    for r in range(ROUNDS):
        for i, c in enumerate(cases):
            enqueue(c, streams[i], outs[i][r], toks[i][r], ppos[i])
    torch.cuda.synchronize()
    assert L.cfi_device_error() == 0
    for i in range(len(cases)):
        for r in range(ROUNDS):
            assert torch.equal(outs[i][r], want[i][0]), (i, r)
            assert int(toks[i][r].item()) == want[i][1], (i, r)
        assert int(ppos[i].item()) == ROUNDS


def test_split_k_gemm_on_two_streams(streams):
    """mul_mat_q at 64 columns on a 1536-row Q4_K matrix splits K over partial tiles and stages
    fp16 activations: both per stream."""
    ctx = cfi.Ctx(0)
    g = cfi.GgmlCaller(ctx, "all")
    rows, k, n = 1536, 8960, 64
    cases = []
    for seed in (3, 4):
        w = torch.from_numpy(cfi.synthetic_weights(cfi.Q4_K, rows, k, seed=seed).ravel()).cuda()
        x = torch.from_numpy(np.random.default_rng(seed).normal(size=(n, k)).astype(np.float32)).cuda()
        q = torch.zeros(k // 128 * n * 144, dtype=torch.uint8, device="cuda")
        cases.append((w, x, q))
    torch.cuda.synchronize()

    def enqueue(c, st, d):
        w, x, q = c
        g.quantize_mmq(1, x.data_ptr(), q.data_ptr(), k, k, n, stream=st.cuda_stream)
        g.mmq(cfi.Q4_K, w.data_ptr(), q.data_ptr(), d.data_ptr(), k, rows, n, stream=st.cuda_stream)

    want = []
    for i, c in enumerate(cases):
        d = torch.zeros(n * rows, device="cuda")
        enqueue(c, streams[i], d)  # first call on each stream outside any capture
        torch.cuda.synchronize()
        want.append(d.clone())
    assert O.rel_l2(want[0].cpu().numpy(), want[1].cpu().numpy()) > 0.5  # the two problems differ
    outs = [[torch.zeros(n * rows, device="cuda") for _ in range(ROUNDS)] for _ in cases]
    torch.cuda.synchronize()
    for r in range(ROUNDS):
        for i, c in enumerate(cases):
            enqueue(c, streams[i], outs[i][r])
    torch.cuda.synchronize()
    assert cfi.lib().cfi_device_error() == 0
    for i in range(len(cases)):
        for r in range(ROUNDS):
            assert torch.equal(outs[i][r], want[i]), (i, r)
    assert ctx.stats()["stock_launches"] == 0
    ctx.close()


def test_gemv_with_fused_step_on_two_streams(streams):
    """cfi_fused_mmvq_swiglu_q8_1: the GEMV's last CTA (a per-stream counter) runs SwiGLU +
    quantize on the whole output."""
    L = cfi.lib()
    rows, k = 2 * 4864, 896
    cases = []
    for seed in (5, 6):
        w = torch.from_numpy(cfi.synthetic_weights(cfi.Q8_0, rows, k, seed=seed).ravel()).cuda()
        x = np.random.default_rng(seed).normal(size=k).astype(np.float32)
        xq = torch.from_numpy(O.quantize_q8_1(x[None, :])).cuda()
        cases.append((w, xq))
    torch.cuda.synchronize()

    def enqueue(c, st, y, out):
        w, xq = c
        assert L.cfi_fused_mmvq_swiglu_q8_1(_p(w), _p(xq), _p(y), rows, k, _p(out), ctypes.c_void_p(st.cuda_stream)) == 0

    want = []
    for i, c in enumerate(cases):
        y = torch.zeros(rows, device="cuda")
        out = torch.zeros(rows // 2 // 32 * 36, dtype=torch.uint8, device="cuda")
        enqueue(c, streams[i], y, out)
        torch.cuda.synchronize()
        want.append(out.clone())
    ys = [[torch.zeros(rows, device="cuda") for _ in range(ROUNDS)] for _ in cases]
    outs = [[torch.zeros(rows // 2 // 32 * 36, dtype=torch.uint8, device="cuda") for _ in range(ROUNDS)] for _ in cases]
    torch.cuda.synchronize()
    for r in range(ROUNDS):
        for i, c in enumerate(cases):
            enqueue(c, streams[i], ys[i][r], outs[i][r])
    torch.cuda.synchronize()
    assert L.cfi_device_error() == 0
    for i in range(len(cases)):
        for r in range(ROUNDS):
            assert torch.equal(outs[i][r], want[i]), (i, r)
