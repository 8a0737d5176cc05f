"""The synthetic decode driver (BASELINE config 4 architecture) on the GPU against a plain PyTorch
float64 evaluation of the same layer math (weights dequantised from the same Q8_0 blocks,
activations put through the same q8_1 rounding, the attention operands through the same fp16
rounding), and captured-graph replays against eager steps.

Each operation is checked teacher-forced -- fed the inputs the kernels themselves produced -- at
1e-5 relative L2.  A float64 evaluation chained through a whole step drifts further: every q8_1
activation quantisation turns the ~1e-6 fp32/fp64 differences (rope at large angles, fp16
rounding of q and the probabilities) into whole-step rounding flips, 5-10x growth per
quantisation point (measured: attention output 4.5e-5, O projection 4.9e-4, FFN gate 2.3e-3), so
the chained logits are held to 5e-2."""
import math

import numpy as np
import pytest

import cfi_b200 as cfi

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from decode import Config, DecodeModel  # noqa: E402


def deq_q8_0(blocks, rows, k):
    b = blocks.view(-1, 34)
    d = b[:, 0:2].contiguous().view(torch.float16).float().double()
    q = b[:, 2:].contiguous().view(torch.int8).double()
    return (q * d).reshape(rows, k)


def q8_1_round(x):
    """quantize_q8_1 then dequantise (refs.rs:119-147): d = amax/127 stored as fp16, q = roundf(x/d)."""
    xb = x.float().reshape(-1, 32)
    amax = xb.abs().amax(dim=1, keepdim=True)
    d = amax / 127.0
    q = torch.where(amax > 0, torch.sign(xb / d) * torch.floor(torch.abs(xb / d) + 0.5), torch.zeros_like(xb))
    return (q.double() * d.half().double()).reshape(-1)


def rms(x, w, eps):
    return x / torch.sqrt((x * x).mean() + eps) * w.double()


def rope(x, nh, hd, pos, theta):
    x = x.reshape(nh, hd)
    half = hd // 2
    i = torch.arange(half, dtype=torch.float64, device=x.device)
    ang = pos * theta ** (-2.0 * i / hd)
    c, s = torch.cos(ang), torch.sin(ang)
    a, b = x[:, :half], x[:, half:]
    return torch.cat([a * c - b * s, a * s + b * c], dim=1).reshape(-1)


def reference_step(m, token, pos):
    c = m.cfg
    nq = c.n_head * c.head_dim
    grp = c.n_head // c.n_kv_head
    E = deq_q8_0(m.embd, c.vocab, c.hidden)
    x = E[token].clone()
    for lay in m.layers:
        W = lambda name, r, k: deq_q8_0(lay[name], r, k)
        h = q8_1_round(rms(x, lay["attn_norm"], c.eps))
        q = W("wq", nq, c.hidden) @ h + lay["bq"].double()
        k = W("wk", c.n_kv_head * c.head_dim, c.hidden) @ h + lay["bk"].double()
        v = W("wv", c.n_kv_head * c.head_dim, c.hidden) @ h + lay["bv"].double()
        q = rope(q, c.n_head, c.head_dim, pos, c.theta)
        k = rope(k, c.n_kv_head, c.head_dim, pos, c.theta)
        kc = lay["kc"].clone()
        vc = lay["vc"].clone()
        kc[:, pos] = k.reshape(c.n_kv_head, c.head_dim).half()
        vc[:, :, pos] = v.reshape(c.n_kv_head, c.head_dim).half()
        q16 = q.half().double().reshape(c.n_head, c.head_dim)
        out = torch.zeros(c.n_head, c.head_dim, dtype=torch.float64, device=x.device)
        for hh in range(c.n_head):
            g = hh // grp
            sc = kc[g].double() @ q16[hh] / math.sqrt(c.head_dim)
            sc[pos + 1:] = -math.inf
            p = torch.softmax(sc, dim=0).float().half().double()
            out[hh] = vc[g].double() @ p
        a = q8_1_round(out.reshape(-1))
        x = x + W("wo", c.hidden, nq) @ a
        h = q8_1_round(rms(x, lay["ffn_norm"], c.eps))
        gt = W("wg", c.ffn, c.hidden) @ h
        up = W("wu", c.ffn, c.hidden) @ h
        gu = q8_1_round(gt / (1 + torch.exp(-gt)) * up)
        x = x + W("wd", c.hidden, c.ffn) @ gu
    h = q8_1_round(rms(x, m.out_norm, c.eps))
    return E @ h


@pytest.fixture(scope="module")
def model():
    assert torch.cuda.is_available()
    ctx = cfi.Ctx(0)
    m = DecodeModel(torch, ctx, torch.device("cuda", 0), Config(layers=2, vocab=2048))
    yield m
    ctx.close()


@pytest.fixture(scope="module")
def model1():
    ctx = cfi.Ctx(0)
    m = DecodeModel(torch, ctx, torch.device("cuda", 0), Config(layers=1, vocab=2048), seed=0x1234)
    yield m
    ctx.close()


def rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


def test_each_operation_of_a_step_teacher_forced(model1):
    m = model1
    c = m.cfg
    lay = m.layers[0]
    nq, grp, pos = c.n_head * c.head_dim, c.n_head // c.n_kv_head, c.prompt
    m.reset(token=77)
    m.step(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert cfi.lib().cfi_device_error() == 0
    E = deq_q8_0(m.embd, c.vocab, c.hidden)
    W = lambda name, r, k: deq_q8_0(lay[name], r, k)
    tol = 1e-5
    h = q8_1_round(rms(E[77], lay["attn_norm"], c.eps))
    assert rel(m.q, W("wq", nq, c.hidden) @ h + lay["bq"].double()) < tol
    assert rel(m.k, W("wk", 128, c.hidden) @ h + lay["bk"].double()) < tol
    assert rel(m.v, W("wv", 128, c.hidden) @ h + lay["bv"].double()) < tol
    # fp32 angles near 631 rad: ~6e-6 (the rope kernel's own test bound is 1e-4)
    assert rel(m.qr, rope(m.q.double(), c.n_head, c.head_dim, pos, c.theta)) < 3e-5
    assert rel(m.kr, rope(m.k.double(), c.n_kv_head, c.head_dim, pos, c.theta)) < 3e-5
    kc, vc = lay["kc"].double(), lay["vc"].double()
    assert torch.equal(lay["kc"][:, pos], m.kr.reshape(2, 64).half())
    assert torch.equal(lay["vc"][:, :, pos], m.v.reshape(2, 64).half())
    q16 = m.qr.half().double().reshape(c.n_head, c.head_dim)
    sc = torch.stack([kc[hh // grp] @ q16[hh] for hh in range(c.n_head)])
    assert rel(m.scores.reshape(c.n_head, -1)[:, :pos + 1], sc[:, :pos + 1]) < tol
    sm = m.scores.double().reshape(c.n_head, -1) / math.sqrt(c.head_dim)
    sm[:, pos + 1:] = -math.inf
    assert rel(m.probs.reshape(c.n_head, -1), torch.softmax(sm, 1)) < tol
    p16 = m.probs.half().double().reshape(c.n_head, -1)
    out = torch.stack([vc[hh // grp] @ p16[hh] for hh in range(c.n_head)]).reshape(-1)
    assert rel(m.attn, out) < tol
    assert rel(m.o, W("wo", c.hidden, nq) @ q8_1_round(m.attn.double())) < tol
    x1 = E[77] + m.o.double()
    h2 = q8_1_round(rms(x1, lay["ffn_norm"], c.eps))
    assert rel(m.gate, W("wg", c.ffn, c.hidden) @ h2) < tol
    assert rel(m.up, W("wu", c.ffn, c.hidden) @ h2) < tol
    g, u = m.gate.double(), m.up.double()
    assert rel(m.gu, g / (1 + torch.exp(-g)) * u) < tol
    assert rel(m.dn, W("wd", c.hidden, c.ffn) @ q8_1_round(m.gu.double())) < tol
    assert rel(m.x, x1 + m.dn.double()) < tol
    assert rel(m.logits, E @ q8_1_round(rms(m.x.double(), m.out_norm, c.eps))) < tol
    assert int(m.token.item()) == int(torch.argmax(m.logits).item())
    assert int(m.pos.item()) == pos + 1


def test_whole_step_against_the_chained_evaluation(model):
    m = model
    m.reset(token=77)
    m.step(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert cfi.lib().cfi_device_error() == 0
    want = reference_step(m, 77, m.cfg.prompt)
    assert rel(m.logits, want) < 5e-2


def test_graph_replay_equals_eager_steps(model):
    m = model
    s = torch.cuda.current_stream()
    for lay in m.layers:
        lay["kc"][:, m.cfg.prompt:] = 0
        lay["vc"][:, :, m.cfg.prompt:] = 0
    m.reset(token=5)
    eager = []
    for _ in range(3):
        m.step(s.cuda_stream)
        eager.append((int(m.token.item()), m.logits.clone()))
    torch.cuda.synchronize()
    # rewind the KV caches to the prompt (the eager steps wrote positions prompt .. prompt+2)
    for lay in m.layers:
        lay["kc"][:, m.cfg.prompt:] = 0
        lay["vc"][:, :, m.cfg.prompt:] = 0
    m.reset(token=5)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        m.step(torch.cuda.current_stream().cuda_stream)
    m.reset(token=5)
    for tok, logits in eager:
        gr.replay()
        torch.cuda.synchronize()
        assert int(m.token.item()) == tok
        assert torch.equal(m.logits, logits)
    assert cfi.lib().cfi_device_error() == 0
    del gr


# ------------------------------------------------------------------------------------------
# fused decode steps (include/cfi_glue.h) against the unfused kernel chain they replace
# ------------------------------------------------------------------------------------------
def _p(t):
    import ctypes
    return ctypes.c_void_p(t.data_ptr())


def _s():
    import ctypes
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("n", [896, 1536, 4864])
def test_fused_add_rmsnorm_quantize_equals_the_chain(n):
    import ctypes
    L = cfi.lib()
    ctx = cfi.Ctx(0)
    g = cfi.GgmlCaller(ctx, "all")
    gen = torch.Generator(device="cuda").manual_seed(n)
    x0 = torch.randn(n, generator=gen, device="cuda")
    y = torch.randn(n, generator=gen, device="cuda")
    w = 1.0 + 0.1 * torch.randn(n, generator=gen, device="cuda")
    xa, xb = x0.clone(), x0.clone()
    h = torch.zeros(n, device="cuda")
    qa = torch.zeros(n // 32 * 36, dtype=torch.uint8, device="cuda")
    qb = torch.zeros_like(qa)
    s = torch.cuda.current_stream().cuda_stream
    assert L.cfi_glue_add(_p(xa), _p(y), n, _s()) == 0
    g.rms_norm(xa.data_ptr(), h.data_ptr(), n, 1, mul=w.data_ptr(), eps=1e-6, stream=s)
    g.quantize_q8_1(h.data_ptr(), qa.data_ptr(), n, n, 1, stream=s)
    assert L.cfi_fused_add_rmsnorm_q8_1(_p(xb), _p(y), _p(w), _p(qb), n, ctypes.c_float(1e-6), _s()) == 0
    torch.cuda.synchronize()
    assert torch.equal(xa, xb)
    assert torch.equal(qa, qb)
    # without the residual add
    assert L.cfi_fused_add_rmsnorm_q8_1(_p(xb), None, _p(w), _p(qb), n, ctypes.c_float(1e-6), _s()) == 0
    torch.cuda.synchronize()
    assert torch.equal(qa, qb) and torch.equal(xa, xb)
    ctx.close()


@pytest.mark.parametrize("pos", [0, 631, 679])
def test_fused_qkv_rope_store_equals_the_chain(pos):
    import ctypes
    L = cfi.lib()
    ctx = cfi.Ctx(0)
    g = cfi.GgmlCaller(ctx, "all")
    nh, nkvh, hd, n_ctx, theta = 14, 2, 64, 680, 1e6
    nq, nkv = nh * hd, nkvh * hd
    gen = torch.Generator(device="cuda").manual_seed(pos)
    qkv = torch.randn(nq + 2 * nkv, generator=gen, device="cuda")
    bias = 0.1 * torch.randn(nq + 2 * nkv, generator=gen, device="cuda")
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    # unfused: bias, rope q and k, cache store
    q, k, v = qkv[:nq].clone(), qkv[nq:nq + nkv].clone(), qkv[nq + nkv:].clone()
    qr, kr = torch.zeros(nq, device="cuda"), torch.zeros(nkv, device="cuda")
    kc_a = torch.zeros(nkvh, n_ctx, hd, dtype=torch.float16, device="cuda")
    vc_a = torch.zeros(nkvh, hd, n_ctx, dtype=torch.float16, device="cuda")
    q16 = torch.zeros(nq, dtype=torch.float16, device="cuda")
    assert L.cfi_glue_qkv_bias(_p(q), _p(k), _p(v), _p(bias[:nq]), _p(bias[nq:nq + nkv]), _p(bias[nq + nkv:]), nq, nkv,
                               _s()) == 0
    g.rope_neox(q.data_ptr(), qr.data_ptr(), hd, nh, 1, hd, p.data_ptr(), freq_base=theta, stream=s)
    g.rope_neox(k.data_ptr(), kr.data_ptr(), hd, nkvh, 1, hd, p.data_ptr(), freq_base=theta, stream=s)
    assert L.cfi_glue_kv_store(_p(qr), _p(kr), _p(v), _p(q16), _p(kc_a), _p(vc_a), _p(p), nq, nkv, hd, n_ctx, _s()) == 0
    # fused
    q_out = torch.zeros(nq, device="cuda")
    kc_b, vc_b = torch.zeros_like(kc_a), torch.zeros_like(vc_a)
    assert L.cfi_fused_qkv_rope_store(_p(qkv), _p(bias), _p(q_out), _p(kc_b), _p(vc_b), _p(p), nq, nkv, hd, n_ctx,
                                      ctypes.c_float(theta), _s()) == 0
    torch.cuda.synchronize()
    assert torch.equal(q_out, qr)
    assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)
    ctx.close()


@pytest.mark.parametrize("nh,nkvh,hd,pos", [(14, 2, 64, 631), (14, 2, 64, 0), (12, 2, 128, 679)])
def test_fused_attention_against_float64(nh, nkvh, hd, pos):
    import ctypes
    L = cfi.lib()
    n_ctx = 680
    gen = torch.Generator(device="cuda").manual_seed(nh + hd + pos)
    q = torch.randn(nh * hd, generator=gen, device="cuda")
    kc = torch.randn(nkvh, n_ctx, hd, generator=gen, device="cuda").half()
    vc = torch.randn(nkvh, hd, n_ctx, generator=gen, device="cuda").half()
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    out = torch.zeros(nh * hd // 32 * 36, dtype=torch.uint8, device="cuda")
    scale = 1.0 / math.sqrt(hd)
    assert L.cfi_fused_attention_q8_1(_p(q), _p(kc), _p(vc), _p(p), _p(out), nh, nkvh, hd, n_ctx,
                                      ctypes.c_float(scale), _s()) == 0
    torch.cuda.synchronize()
    assert cfi.lib().cfi_device_error() == 0
    grp = nh // nkvh
    qd = q.double().reshape(nh, hd)
    want = []
    for h in range(nh):
        s_ = kc[h // grp, :pos + 1].double() @ qd[h] * scale
        pr = torch.softmax(s_, 0)
        want.append(vc[h // grp, :, :pos + 1].double() @ pr)
    want = torch.cat(want)
    # the q8_1 blocks of the exact output: the kernel's fp32 output is within ~1e-6 of it, so
    # scales agree closely and quants differ by at most one step (round-half cases), rarely
    import oracle_py as O
    ref = torch.from_numpy(O.quantize_q8_1(want.float().cpu().numpy().reshape(1, -1))).reshape(-1, 36)
    blk = out.cpu().reshape(-1, 36)
    d = blk[:, 0:2].contiguous().view(torch.float16).double()
    dr = ref[:, 0:2].contiguous().view(torch.float16).double()
    assert torch.allclose(d, dr, rtol=2e-3, atol=0)
    qv = blk[:, 4:].contiguous().view(torch.int8).int()
    qr = ref[:, 4:].contiguous().view(torch.int8).int()
    assert int((qv - qr).abs().max()) <= 1
    assert float((qv != qr).float().mean()) < 0.02


def test_fused_swiglu_quantize_equals_the_chain():
    L = cfi.lib()
    ctx = cfi.Ctx(0)
    g = cfi.GgmlCaller(ctx, "all")
    n = 4864
    gen = torch.Generator(device="cuda").manual_seed(3)
    gu = 3 * torch.randn(2 * n, generator=gen, device="cuda")
    out = torch.zeros(n, device="cuda")
    qa = torch.zeros(n // 32 * 36, dtype=torch.uint8, device="cuda")
    qb = torch.zeros_like(qa)
    assert L.cfi_glue_swiglu(_p(gu[:n]), _p(gu[n:]), _p(out), n, _s()) == 0
    g.quantize_q8_1(out.data_ptr(), qa.data_ptr(), n, n, 1, stream=torch.cuda.current_stream().cuda_stream)
    assert L.cfi_fused_swiglu_q8_1(_p(gu), _p(qb), n, _s()) == 0
    torch.cuda.synchronize()
    assert torch.equal(qa, qb)
    ctx.close()


def test_fused_step_tracks_the_unfused_step_and_replays():
    """The fused step runs the same model (same weights, the unfused step's views): its logits stay
    within the drift the attention's fp16 rounding points allow, and graph replays equal eager steps."""
    ctx = cfi.Ctx(0)
    cfg = Config(layers=2, vocab=2048)
    mu = DecodeModel(torch, ctx, torch.device("cuda", 0), cfg)
    mf = DecodeModel(torch, ctx, torch.device("cuda", 0), cfg, fused=True)
    s = torch.cuda.current_stream()
    mu.reset(token=77)
    mu.step(s.cuda_stream)
    mf.reset(token=77)
    mf.step(s.cuda_stream)
    torch.cuda.synchronize()
    assert cfi.lib().cfi_device_error() == 0
    assert rel(mf.logits, mu.logits) < 5e-2
    assert mf.launches_per_step == 2 + 9 * cfg.layers + 2
    # graph replay of the fused step == eager fused steps
    for lay in mf.layers:
        lay["kc"][:, cfg.prompt:] = 0
        lay["vc"][:, :, cfg.prompt:] = 0
    mf.reset(token=5)
    eager = []
    for _ in range(3):
        mf.step(s.cuda_stream)
        eager.append((int(mf.token.item()), mf.logits.clone()))
    for lay in mf.layers:
        lay["kc"][:, cfg.prompt:] = 0
        lay["vc"][:, :, cfg.prompt:] = 0
    mf.reset(token=5)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        mf.step(torch.cuda.current_stream().cuda_stream)
    mf.reset(token=5)
    for tok, logits in eager:
        gr.replay()
        torch.cuda.synchronize()
        assert int(mf.token.item()) == tok
        assert torch.equal(mf.logits, logits)
    del gr
    ctx.close()


def test_gguf_export_and_load_give_the_same_model(tmp_path):
    """A model written as a qwen2 GGUF file (include/cfi_gguf.h reader) and loaded back steps to
    bit-identical logits, fused and unfused; a separate output.weight becomes the lm_head."""
    from decode import load_gguf, save_gguf

    ctx = cfi.Ctx(0)
    cfg = Config(layers=2, vocab=2048)
    m0 = DecodeModel(torch, ctx, torch.device("cuda", 0), cfg)
    path = tmp_path / "qwen2-mini.gguf"
    save_gguf(m0, path)
    # another seed: every weight differs until the file's are loaded; the caches are copied over
    m1 = load_gguf(torch, ctx, torch.device("cuda", 0), path, seed=1234)
    assert m1.cfg.hidden == cfg.hidden and m1.cfg.layers == 2 and m1.cfg.vocab == 2048
    assert torch.equal(m1.layers[1]["wqkv"], m0.layers[1]["wqkv"]) and torch.equal(m1.layers[0]["bqkv"], m0.layers[0]["bqkv"])
    s = torch.cuda.current_stream().cuda_stream
    for fused in (False, True):
        m0.fused = m1.fused = fused
        for l0, l1 in zip(m0.layers, m1.layers):
            l0["kc"][:, cfg.prompt:] = 0
            l0["vc"][:, :, cfg.prompt:] = 0
            l1["kc"].copy_(l0["kc"])
            l1["vc"].copy_(l0["vc"])
        for m in (m0, m1):
            m.reset(token=11)
            m.step(s)
        torch.cuda.synchronize()
        assert torch.equal(m0.logits, m1.logits)
    # a separate lm_head
    m0.head = m0.embd.clone()
    m0.head[:34] = 0  # first block of row 0 zeroed: d = 0
    save_gguf(m0, tmp_path / "b.gguf")
    m2 = load_gguf(torch, ctx, torch.device("cuda", 0), tmp_path / "b.gguf")
    assert m2.head is not m2.embd and torch.equal(m2.head, m0.head)
    ctx.close()


def test_gemv_epilogue_step_equals_the_fused_step():
    """fused=2 (add + rms_norm + quantize in the O and down GEMVs' last CTAs, 7 launches per layer;
    with the QKV and gate/up steps too, 5) gives the same bits as fused=1 (separate launches), over
    three graph-replayed tokens."""
    ctx = cfi.Ctx(0)
    cfg = Config(layers=2, vocab=2048)
    ms = [DecodeModel(torch, ctx, torch.device("cuda", 0), cfg, fused=f) for f in (1, 2, 2)]
    ms[2].epi_qkv = ms[2].epi_swiglu = True
    out = []
    for m in ms:
        for lay in m.layers:
            lay["kc"][:, cfg.prompt:] = 0
            lay["vc"][:, :, cfg.prompt:] = 0
        m.reset(token=9)
        m.step(torch.cuda.current_stream().cuda_stream)  # first-use probes, eager
        for lay in m.layers:
            lay["kc"][:, cfg.prompt:] = 0
            lay["vc"][:, :, cfg.prompt:] = 0
        m.reset(token=9)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            m.step(torch.cuda.current_stream().cuda_stream)
        m.reset(token=9)
        toks = []
        for _ in range(3):
            gr.replay()
            torch.cuda.synchronize()
            toks.append((int(m.token.item()), m.logits.clone()))
        out.append(toks)
        del gr
    assert cfi.lib().cfi_device_error() == 0
    assert ms[1].launches_per_step == 1 + 1 + 7 * cfg.layers + 2
    assert ms[2].launches_per_step == 1 + 1 + 5 * cfg.layers + 2
    for k in (1, 2):
        for (t1, l1), (t2, l2) in zip(out[0], out[k]):
            assert t1 == t2 and torch.equal(l1, l2)
    ctx.close()
