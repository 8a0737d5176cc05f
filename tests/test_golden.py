"""Frozen fixtures (tests/golden/golden.npz, made by tests/golden/make_golden.py).

CPU: the oracle still reproduces every committed output bit for bit.  GPU: every native kernel
against the committed outputs -- bitwise for quantize, quantize_mmq and mmvq (the decode-fast
model, refs.rs:435-497), 1e-3 relative L2 for mmq (the stated bar), the reference tests' own
tolerances for the row ops."""
import ctypes as C
import os

import numpy as np
import pytest

import cfi_b200 as cfi
import oracle_py as O

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
NMMVQ = len([k for k in G.files if k.startswith("mmvq") and k.endswith("_p")])
NMMQ = len([k for k in G.files if k.startswith("mmq") and k.endswith("_p")])


def mmvq_params(i):
    p = O.Mmvq()
    for (n, _), v in zip(O.Mmvq._fields_, G["mmvq%d_p" % i]):
        setattr(p, n, int(v))
    return p


def mmq_params(i):
    p = O.Mmq()
    for (n, _), v in zip(O.Mmq._fields_, G["mmq%d_p" % i]):
        setattr(p, n, int(v))
    return p


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# ---------------------------------------------------------------- CPU: the oracle is unchanged
def test_oracle_reproduces_the_fixtures():
    n0, ne0, rows = (int(v) for v in G["q81_shape"])
    x, ref = O.quantize_case(n0, ne0, rows, 1, 1, 0x3171)
    assert np.array_equal(x, G["q81_x"]) and np.array_equal(ref, G["q81_y"])
    for i in range(NMMVQ):
        p = mmvq_params(i)
        ids = np.zeros(1, dtype=np.int32)
        n = G["mmvq%d_stock" % i].size
        assert np.array_equal(bits(O.mmvq_ref(p, G["mmvq%d_x" % i], G["mmvq%d_y" % i], ids, n)), bits(G["mmvq%d_stock" % i]))
        if p.ncols_dst == 1:
            got = O.mmvq_fast_ref(p, G["mmvq%d_x" % i], G["mmvq%d_y" % i], ids, n, 1, 1, True)
            assert np.array_equal(bits(got), bits(G["mmvq%d_fast" % i]))
    assert np.array_equal(O.quantize_mmq(8, G["qmmq_x"], 512, 7), G["qmmq_d4"])
    assert np.array_equal(O.quantize_mmq(12, G["qmmq_x"], 512, 7), G["qmmq_ds4"])
    for i in range(NMMQ):
        p = mmq_params(i)
        got = O.mmq_ref(int(G["mmq%d_ty" % i][0]), p, G["mmq%d_x" % i], G["mmq%d_y" % i], G["mmq%d_dst" % i].size)
        assert np.array_equal(bits(got), bits(G["mmq%d_dst" % i]))
    assert np.array_equal(bits(O.rms_norm(G["rms_x"], G["rms_w"], 4, 896, 1e-6)), bits(G["rms_y"]))
    assert np.array_equal(bits(O.soft_max(G["sm_x"], G["sm_mask"], None, 631, 2, 14, 28, 0.125)), bits(G["sm_y"]))
    assert np.array_equal(bits(O.rope_neox(G["rope_x"], 64, 16, 3, 64, G["rope_pos"], 1e6)), bits(G["rope_y"]))


# ---------------------------------------------------------------- GPU: the kernels vs the fixtures
@pytest.fixture(scope="module")
def dev():
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available()
    ctx = cfi.Ctx(0)
    yield torch, ctx, cfi.GgmlCaller(ctx, "all")
    ctx.close()


def d(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def finish(torch):
    torch.cuda.synchronize()
    assert cfi.lib().cfi_device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("exact", ["0", "1"])
def test_kernels_match_the_fixtures(dev, monkeypatch, exact):
    """Bitwise against the frozen outputs, except the tensor-core Q4_K GEMV of 3-8 columns (the
    default; exact int32 block dots, fp32 scales reassociated): nmse < 1e-10 there, bitwise again
    with CFI_MMVQ_EXACT=1."""
    torch, ctx, g = dev
    monkeypatch.setenv("CFI_MMVQ_EXACT", exact)
    s = torch.cuda.current_stream().cuda_stream
    n0, ne0, rows = (int(v) for v in G["q81_shape"])
    y = torch.zeros(G["q81_y"].size, dtype=torch.uint8, device="cuda")
    g.quantize_q8_1(d(torch, G["q81_x"]).data_ptr(), y.data_ptr(), n0, ne0, rows, stream=s)
    finish(torch)
    assert np.array_equal(y.cpu().numpy(), G["q81_y"])
    for i in range(NMMVQ):
        p = mmvq_params(i)
        want = G["mmvq%d_fast" % i]
        dx, dy = d(torch, G["mmvq%d_x" % i]), d(torch, G["mmvq%d_y" % i])
        out = torch.zeros(want.size, dtype=torch.float32, device="cuda")
        g.mmvq(p.ty, p.ncols_dst, dx.data_ptr(), dy.data_ptr(), out.data_ptr(), p.ncols_x, p.nrows_x,
               stride_row_x=p.stride_row_x, stride_col_y=p.stride_col_y, stride_col_dst=p.stride_col_dst, stream=s)
        finish(torch)
        if exact == "0" and p.ty == cfi.Q4_K and p.ncols_dst >= 3:
            assert O.nmse(out.cpu().numpy(), want) < 1e-10, "mmvq fixture %d" % i
        else:
            assert np.array_equal(bits(out.cpu().numpy()), bits(want)), "mmvq fixture %d" % i
    for lay, key in ((0, "qmmq_d4"), (1, "qmmq_ds4")):
        q = torch.zeros(G[key].size, dtype=torch.uint8, device="cuda")
        g.quantize_mmq(lay, d(torch, G["qmmq_x"]).data_ptr(), q.data_ptr(), 512, 512, 7, stream=s)
        finish(torch)
        assert np.array_equal(q.cpu().numpy(), G[key]), key
    for i in range(NMMQ):
        p = mmq_params(i)
        ty = int(G["mmq%d_ty" % i][0])
        want = G["mmq%d_dst" % i]
        out = torch.zeros(want.size, dtype=torch.float32, device="cuda")
        words = [p.ncols_x, p.nrows_x, p.ncols_dst, p.stride_row_x, p.ncols_y, p.stride_col_dst, p.channel_ratio,
                 p.nchannels_y, p.stride_channel_x, p.stride_channel_y, p.stride_channel_dst, p.sample_ratio,
                 p.nsamples_y, p.stride_sample_x, p.stride_sample_y, p.stride_sample_dst, p.ncols_dst]
        dx, dy = d(torch, G["mmq%d_x" % i]), d(torch, G["mmq%d_y" % i])
        g.mmq_words(ty, dx.data_ptr(), dy.data_ptr(), out.data_ptr(), words, stream=s)
        finish(torch)
        assert O.rel_l2(out.cpu().numpy(), want) < 1e-3, "mmq fixture %d" % i
    out = torch.zeros(4 * 896, dtype=torch.float32, device="cuda")
    dw = d(torch, G["rms_w"])
    g.rms_norm(d(torch, G["rms_x"]).data_ptr(), out.data_ptr(), 896, 4, mul=dw.data_ptr(), eps=1e-6, stream=s)
    finish(torch)
    assert O.rel_l2(out.cpu().numpy(), G["rms_y"].ravel()) < 1e-5
    out = torch.zeros(28 * 631, dtype=torch.float32, device="cuda")
    dm = d(torch, G["sm_mask"])
    g.soft_max(d(torch, G["sm_x"]).data_ptr(), dm.data_ptr(), out.data_ptr(), 631, 2, 14, 0.125, stream=s)
    finish(torch)
    assert O.rel_l2(out.cpu().numpy(), G["sm_y"].ravel()) < 1e-5
    out = torch.zeros(G["rope_y"].size, dtype=torch.float32, device="cuda")
    dp = d(torch, G["rope_pos"])
    g.rope_neox(d(torch, G["rope_x"]).data_ptr(), out.data_ptr(), 64, 16, 3, 64, dp.data_ptr(), freq_base=1e6, stream=s)
    finish(torch)
    assert O.rel_l2(out.cpu().numpy(), G["rope_y"].ravel()) < 1e-4
