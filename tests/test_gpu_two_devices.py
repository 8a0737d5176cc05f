"""One process driving two GPUs, as ggml does with a split model: the library's once-per-device
state (the shared-memory attributes of its large kernels, the bounded-wait error words, the GEMV
and attention last-CTA counters, the per-stream scratch) must be set up on each device it runs on.

Every kernel family with such state runs on device 0, then on device 1, in one process; each
result is checked against the oracle (or, for the kernels whose fp32 order is exact, against
device 0's result bit for bit) and the device's error word.  Skipped with fewer than two GPUs."""
import ctypes as C

import numpy as np
import pytest

import cfi_b200 as cfi
import oracle_py as O

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs in one process")]

MMQ_WORDS = ("ncols_x", "nrows_x", "ncols_dst", "stride_row_x", "ncols_y", "stride_col_dst", "channel_ratio",
             "nchannels_y", "stride_channel_x", "stride_channel_y", "stride_channel_dst", "sample_ratio", "nsamples_y",
             "stride_sample_x", "stride_sample_y", "stride_sample_dst", "ncols_dst")


def _p(t):
    return C.c_void_p(t.data_ptr())


def on_device(d, fn):
    """fn(ctx, caller, stream) on device d with its own context; returns fn's result."""
    torch.cuda.set_device(d)
    ctx = cfi.Ctx(d)
    g = cfi.GgmlCaller(ctx, "all")
    try:
        out = fn(ctx, g, torch.cuda.current_stream(d).cuda_stream)
        torch.cuda.synchronize(d)
        assert cfi.lib().cfi_device_error() == 0, d
        return out
    finally:
        ctx.close()


def test_tensor_core_gemm_and_attention_on_both_devices():
    """mul_mat_q on tcgen05 (> 48 KB of dynamic shared memory, split K, fp16 scratch), the skinny
    mul_mat_q, and FlashAttention, each on device 0 then device 1."""
    p, x, y, n = O.mmq_case(cfi.Q8_0, 896, 4864, 631, 1, 1, 1, 21)
    want = O.mmq_ref(cfi.Q8_0, p, x, y, n)
    ps, xs, ys, ns = O.mmq_case(cfi.Q4_K, 1536, 1000, 64, 1, 1, 1, 22)
    want_s = O.mmq_ref(cfi.Q4_K, ps, xs, ys, ns)
    d, nq, nh, nkv = 64, 64, 4, 192
    q, k, v, m = O.fattn_case(d, nq, nh, 2, nkv, 1, True, 23)
    want_fa = O.fattn_reference(d, nq, nh, 2, nkv, 1, q, k, v, m, np.float32(1.0 / np.sqrt(d)))

    def work(ctx, g, st):
        res = []
        for ty, pp, xx, yy, nn in ((cfi.Q8_0, p, x, y, n), (cfi.Q4_K, ps, xs, ys, ns)):
            dx, dy = torch.from_numpy(xx).cuda(), torch.from_numpy(yy).cuda()
            dd = torch.full((nn,), float("nan"), device="cuda")
            g.mmq_words(ty, dx.data_ptr(), dy.data_ptr(), dd.data_ptr(), [getattr(pp, w) for w in MMQ_WORDS], stream=st)
            res.append(dd)
        dq = torch.from_numpy(q).cuda()
        dk, dv = torch.from_numpy(k.view(np.int16)).cuda(), torch.from_numpy(v.view(np.int16)).cuda()
        dm = torch.from_numpy(m.view(np.int16)).cuda()
        do = torch.full((d * nh * nq,), float("nan"), device="cuda")
        g.fattn(d, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dm.data_ptr(), do.data_ptr(), nq, nh, 2, nkv, 1,
                1.0 / np.sqrt(d), stream=st)
        res.append(do)
        torch.cuda.synchronize()
        return [r.cpu().numpy() for r in res]

    for dev in (0, 1):
        got, got_s, got_fa = on_device(dev, work)
        assert O.rel_l2(got, want) < 1e-3, dev
        assert O.rel_l2(got_s, want_s) < 1e-5, dev
        assert O.rel_l2(got_fa, want_fa) < 1e-3, dev


def test_gemv_epilogue_and_decode_glue_on_both_devices():
    """The GEMV whose last CTA runs SwiGLU + quantize (a per-device, per-stream counter), the split
    single-token attention and the multi-CTA argmax (per-device partial buffers): bit for bit the
    same on both devices."""
    rows, k = 2 * 4864, 896
    w = cfi.synthetic_weights(cfi.Q8_0, rows, k, seed=31).ravel()
    xq = O.quantize_q8_1(np.random.default_rng(31).normal(size=k).astype(np.float32)[None, :])
    nh, nkvh, hd, n_ctx = 14, 2, 64, 2048
    rng = np.random.default_rng(32)
    qv = rng.normal(size=nh * hd).astype(np.float32)
    kc = rng.normal(size=(nkvh, n_ctx, hd)).astype(np.float16)
    vc = rng.normal(size=(nkvh, hd, n_ctx)).astype(np.float16)
    logits = rng.normal(size=151936).astype(np.float32)
    L = cfi.lib()

    def work(ctx, g, st):
        s = C.c_void_p(st)
        dw, dxq = torch.from_numpy(w).cuda(), torch.from_numpy(xq).cuda()
        y = torch.zeros(rows, device="cuda")
        sw = torch.zeros(rows // 2 // 32 * 36, dtype=torch.uint8, device="cuda")
        assert L.cfi_fused_mmvq_swiglu_q8_1(_p(dw), _p(dxq), _p(y), rows, k, _p(sw), s) == 0
        dq, dk, dv = torch.from_numpy(qv).cuda(), torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
        pos = torch.tensor([n_ctx - 5], dtype=torch.int32, device="cuda")
        att = torch.zeros(nh * hd // 32 * 36, dtype=torch.uint8, device="cuda")
        assert L.cfi_fused_attention_q8_1(_p(dq), _p(dk), _p(dv), _p(pos), _p(att), nh, nkvh, hd, n_ctx,
                                          C.c_float(1.0 / hd ** 0.5), s) == 0
        lg = torch.from_numpy(logits).cuda()
        tok = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert L.cfi_glue_argmax_next(_p(lg), logits.size, _p(tok), _p(pos), s) == 0
        torch.cuda.synchronize()
        return y.cpu().numpy(), sw.cpu().numpy(), att.cpu().numpy(), int(tok.item()), int(pos.item())

    r0 = on_device(0, work)
    r1 = on_device(1, work)
    for a, b in zip(r0[:3], r1[:3]):
        assert np.array_equal(a, b)
    assert r0[3] == r1[3] == int(np.argmax(logits))
    assert r0[4] == r1[4] == n_ctx - 4
