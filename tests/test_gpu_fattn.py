"""GPU tests of the native FlashAttention (flash_attn_ext_f16 on tcgen05) through the substitution
C ABI, against the exact f64 softmax attention of the reference's probe (src/subst/probe.rs:405-489)
on its case generator (probe.rs:421-446).  Q and P are rounded to fp16 for the tensor cores, as
ggml's own tensor-core kernel does; that rounding alone gives about 2e-4 relative L2 (nmse about
4e-8, the same as a float64 model of the rounding), inside the 1e-3 relative L2 bound."""
import numpy as np
import pytest

import cfi_b200 as cfi
import oracle_py as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REL = 1e-3
NMSE = 1e-6


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available()
    ctx = cfi.Ctx(0)
    yield ctx, cfi.GgmlCaller(ctx, "all")
    ctx.close()


def run_case(g, d, nq, nh, nh_kv, nkv, ns, causal, seed):
    q, k, v, m = O.fattn_case(d, nq, nh, nh_kv, nkv, ns, causal, seed)
    scale = 1.0 / np.sqrt(d)
    dq = torch.from_numpy(q).cuda()
    dk = torch.from_numpy(k.view(np.int16)).cuda()
    dv = torch.from_numpy(v.view(np.int16)).cuda()
    dm = torch.from_numpy(m.view(np.int16)).cuda() if m is not None else None
    dd = torch.full((d * nh * nq * ns,), float("nan"), device="cuda")
    g.fattn(d, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dm.data_ptr() if dm is not None else 0, dd.data_ptr(), nq,
            nh, nh_kv, nkv, ns, scale, stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert cfi.lib().cfi_device_error() == 0
    want = O.fattn_reference(d, nq, nh, nh_kv, nkv, ns, q, k, v, m, np.float32(scale))
    return dd.cpu().numpy(), want


@pytest.mark.parametrize("d,nq,nh,nh_kv,nkv,ns,causal", [
    (64, 19, 4, 2, 70, 1, True),       # the reference's probe case: one partial tile, partial key chunk
    (128, 19, 4, 2, 70, 1, True),
    (64, 631, 14, 2, 960, 1, True),    # Qwen2.5-0.5B heads, a 631-token prompt, padded causal cache
    (128, 631, 12, 2, 960, 1, True),   # Qwen2.5-1.5B heads
    (128, 300, 12, 2, 300, 2, False),  # no mask, two sequences
    (64, 200, 8, 8, 300, 1, True),     # no GQA, keys not a multiple of 128 (every query sees a key)
])
def test_fattn_matches_exact_attention(dev, d, nq, nh, nh_kv, nkv, ns, causal):
    ctx, g = dev
    got, want = run_case(g, d, nq, nh, nh_kv, nkv, ns, causal, 0xfa77 + nq + d)
    assert np.isfinite(got).all()
    assert O.rel_l2(got, want) < REL, O.rel_l2(got, want)
    assert O.nmse(got, want) < NMSE, O.nmse(got, want)


def test_fattn_probe_and_fixup_skip(dev):
    ctx, g = dev
    for d in (64, 128):
        _, p, _ = cfi.decide(cfi.NAMES["fattn"].format(d=d), "fattn", "all")
        rc, why = ctx.probe(p, torch.cuda.current_stream().cuda_stream)
        assert rc == 0, why
    # the stream-k fixup after a native FlashAttention is skipped (the native kernel writes final results)
    d, nq, nh, nkv = 64, 40, 4, 128
    q, k, v, m = O.fattn_case(d, nq, nh, 2, nkv, 1, True, 5)
    dq, dk, dv = torch.from_numpy(q).cuda(), torch.from_numpy(k.view(np.int16)).cuda(), torch.from_numpy(v.view(np.int16)).cuda()
    dm = torch.from_numpy(m.view(np.int16)).cuda()
    dd = torch.zeros(d * nh * nq, device="cuda")
    meta = torch.zeros(2 * nh * nq * 8, device="cuda")
    before = ctx.stats()["fixups_skipped"]
    s = torch.cuda.current_stream().cuda_stream
    g.fattn(d, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dm.data_ptr(), dd.data_ptr(), nq, nh, 2, nkv, 1, 0.125,
            dst_meta=meta.data_ptr(), stream=s)
    out = dd.clone()
    g.fattn_fixup(d, dd.data_ptr(), meta.data_ptr(), nq, nh, 1, nkv, stream=s)
    torch.cuda.synchronize()
    assert ctx.stats()["fixups_skipped"] == before + 1
    assert torch.equal(dd, out)
    assert ctx.stats()["stock_launches"] == 0
