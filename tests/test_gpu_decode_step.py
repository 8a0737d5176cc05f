"""GPU test of cfi_decode_step_q8_0, the decode token step as one persistent launch: token by
token, its results equal the fused glue chain's (the decode driver's fused == 1 step, 9 launches
per layer) bit for bit -- the next token and position, the logits, the step's final x and hq, and
every layer's K and V caches after the steps."""
import pytest

import cfi_b200 as cfi

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

STEPS = 4


def test_persistent_step_equals_the_fused_chain():
    from decode import DecodeModel

    assert torch.cuda.is_available()
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    ctx_a, ctx_b = cfi.Ctx(0), cfi.Ctx(0)
    chain = DecodeModel(torch, ctx_a, dev, fused=1)
    pers = DecodeModel(torch, ctx_b, dev, fused=3)
    for m in (chain, pers):
        m.reset(token=1234)
    st = torch.cuda.Stream()
    for step in range(STEPS):
        for m in (chain, pers):
            m.step(st.cuda_stream)
        torch.cuda.synchronize()
        assert cfi.lib().cfi_device_error() == 0 and cfi.lib().cfi_decode_step_error() == 0
        assert int(pers.token.item()) == int(chain.token.item()), step
        assert int(pers.pos.item()) == int(chain.pos.item()) == chain.cfg.prompt + step + 1
        for name in ("logits", "x", "hq", "aq", "gq", "dn", "qr"):
            assert torch.equal(getattr(pers, name), getattr(chain, name)), (step, name)
    for i, (la, lb) in enumerate(zip(chain.layers, pers.layers)):
        assert torch.equal(la["kc"], lb["kc"]) and torch.equal(la["vc"], lb["vc"]), i
    assert pers.launches_per_step == 1
    ctx_a.close()
    ctx_b.close()


def test_persistent_step_refuses_unsupported_shapes():
    L = cfi.lib()
    s = cfi.DecodeStep()
    s.hidden, s.n_head, s.n_kv_head, s.head_dim, s.ffn, s.vocab, s.n_ctx, s.n_layers = 896, 14, 2, 64, 4864, 1000, 680, 1
    lay = torch.zeros(256, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    import ctypes as C
    for field, bad in (("hidden", 4096), ("head_dim", 96), ("n_ctx", 682), ("n_layers", 0), ("ffn", 4896)):
        old = getattr(s, field)
        setattr(s, field, bad)
        assert L.cfi_decode_step_q8_0(C.byref(s), C.c_void_p(lay.data_ptr()), C.c_void_p(st)) != 0, field
        setattr(s, field, old)
    torch.cuda.synchronize()
