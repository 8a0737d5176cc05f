"""Synthetic decode driver: a Qwen2-architecture layer stack (Qwen2.5-0.5B
shape, random Q8_0 weights) stepping one token at a time through this library's kernels only.

Per layer, in ggml's order: rms_norm (x attn_norm) -> quantize_q8_1 -> Q/K/V mul_mat_vec_q (+bias)
-> rope_neox on q and k -> K/V cache store (f16) -> KQ = K^T q (GemmStridedBatchedEx, GQA groups)
-> soft_max (scale 1/sqrt(d), causal mask) -> KQV = V P -> quantize -> O projection -> residual ->
rms_norm (x ffn_norm) -> quantize -> gate/up -> swiglu -> quantize -> down -> residual.  Then the
output norm, the tied Q8_0 embedding as lm_head, and a device-side greedy argmax that advances the
position.  The substituted kernels (quantize_q8_1, mul_mat_vec_q, rms_norm, rope_neox, soft_max)
run through the substitution C ABI with ggml's kernelParams; the attention products through the
cuBLAS-compatible GemmEx; the element-wise steps through include/cfi_glue.h.  Position and token
live in device memory, so one captured step graph replays for every token.

The model weights are random (seeded), so the generated tokens are meaningless; the KV cache of the
prompt positions is filled with seeded random values instead of running a prefill.
"""
import ctypes as C
import math
from dataclasses import dataclass

import cfi_b200 as cfi


@dataclass
class Config:
    hidden: int = 896
    layers: int = 24
    n_head: int = 14
    n_kv_head: int = 2
    head_dim: int = 64
    ffn: int = 4864
    vocab: int = 151936
    eps: float = 1e-6
    theta: float = 1e6
    prompt: int = 631
    n_ctx: int = 680  # >= prompt + generated tokens, a multiple of 8

    def weight_bytes_per_token(self):
        per_layer = (self.hidden * (self.n_head * self.head_dim) * 2 + self.hidden * self.n_kv_head * self.head_dim * 2
                     + self.hidden * self.ffn * 3)
        return (per_layer * self.layers + self.vocab * self.hidden) * 34 // 32


def random_q8_0(torch, rows, k, gen, device):
    """Valid Q8_0 blocks of a random matrix with values about N(0, 0.02) (device-side, seeded)."""
    nb = rows * k // 32
    q = torch.clamp(torch.round(torch.randn(nb, 32, generator=gen, device=device) * 42.0), -127, 127).to(torch.int8)
    d = (0.02 / 42.0 * (0.75 + 0.5 * torch.rand(nb, 1, generator=gen, device=device))).to(torch.float16)
    blk = torch.empty(nb, 34, dtype=torch.uint8, device=device)
    blk[:, 0:2] = d.view(torch.uint8)
    blk[:, 2:] = q.view(torch.uint8)
    return blk.reshape(-1)


def random_q4_k(torch, rows, k, gen, device):
    """Valid Q4_K superblocks (144 B: fp16 d and dmin, 12 bytes of 6-bit scales/mins, 128 bytes of
    nibbles) with random scales, mins and quants (device-side, seeded); d, dmin about 2e-4, so
    weights fall in about [-0.8, 0.9] with most near +-0.1."""
    nsb = rows * k // 256
    blk = torch.randint(0, 256, (nsb, 144), generator=gen, device=device, dtype=torch.int32).to(torch.uint8)
    dd = (2e-4 * (0.75 + 0.5 * torch.rand(nsb, 2, generator=gen, device=device))).to(torch.float16)
    blk[:, 0:4] = dd.view(torch.uint8)
    return blk.reshape(-1)


class DecodeModel:
    """fused=False: the ggml op sequence above, kernel by kernel.  fused=True: the same model with
    Q/K/V and gate/up as stacked weights (one GEMV each) and the include/cfi_glue.h fused steps
    (add + rms_norm + quantize, bias + rope + cache store, single-token attention to q8_1, SwiGLU +
    quantize): 9 launches per layer instead of 25."""

    def __init__(self, torch, ctx, device, cfg=None, seed=0x5eed, fused=False):
        self.t = torch
        self.cfg = cfg or Config()
        self.dev = device
        self.fused = fused
        self.row_gemv_below_kb = 8192
        # fused == 2: which GEMVs also carry their element-wise step (the add + rms_norm ones always)
        self.epi_qkv = self.epi_swiglu = False
        self.g = cfi.GgmlCaller(ctx, "all")
        self.blas = cfi.Blas()
        self.L = cfi.lib()
        c, tt = self.cfg, torch
        gen = tt.Generator(device=device)
        gen.manual_seed(seed)
        f32 = dict(dtype=tt.float32, device=device)
        nq, nkv = c.n_head * c.head_dim, c.n_kv_head * c.head_dim
        self.layers = []
        for _ in range(c.layers):
            self.layers.append(dict(
                wq=random_q8_0(tt, nq, c.hidden, gen, device), wk=random_q8_0(tt, nkv, c.hidden, gen, device),
                wv=random_q8_0(tt, nkv, c.hidden, gen, device), wo=random_q8_0(tt, c.hidden, nq, gen, device),
                wg=random_q8_0(tt, c.ffn, c.hidden, gen, device), wu=random_q8_0(tt, c.ffn, c.hidden, gen, device),
                wd=random_q8_0(tt, c.hidden, c.ffn, gen, device),
                bq=tt.randn(nq, generator=gen, **f32) * 0.1, bk=tt.randn(nkv, generator=gen, **f32) * 0.1,
                bv=tt.randn(nkv, generator=gen, **f32) * 0.1,
                attn_norm=1.0 + 0.1 * tt.randn(c.hidden, generator=gen, **f32),
                ffn_norm=1.0 + 0.1 * tt.randn(c.hidden, generator=gen, **f32),
                kc=tt.zeros(c.n_kv_head, c.n_ctx, c.head_dim, dtype=tt.float16, device=device),
                vc=tt.zeros(c.n_kv_head, c.head_dim, c.n_ctx, dtype=tt.float16, device=device)))
            lay = self.layers[-1]
            # stacked Q/K/V and gate/up weights (the per-matrix entries become views of them)
            lay["wqkv"] = tt.cat([lay["wq"], lay["wk"], lay["wv"]])
            nqb, nkb = lay["wq"].numel(), lay["wk"].numel()
            lay["wq"], lay["wk"], lay["wv"] = (lay["wqkv"][:nqb], lay["wqkv"][nqb:nqb + nkb],
                                               lay["wqkv"][nqb + nkb:])
            lay["wgu"] = tt.cat([lay["wg"], lay["wu"]])
            ngb = lay["wg"].numel()
            lay["wg"], lay["wu"] = lay["wgu"][:ngb], lay["wgu"][ngb:]
            lay["bqkv"] = tt.cat([lay["bq"], lay["bk"], lay["bv"]])
            lay["bq"], lay["bk"], lay["bv"] = lay["bqkv"][:nq], lay["bqkv"][nq:nq + nkv], lay["bqkv"][nq + nkv:]
            lay["kc"][:, :c.prompt] = (tt.randn(c.n_kv_head, c.prompt, c.head_dim, generator=gen, **f32)).half()
            lay["vc"][:, :, :c.prompt] = (tt.randn(c.n_kv_head, c.head_dim, c.prompt, generator=gen, **f32)).half()
        self.embd = random_q8_0(tt, c.vocab, c.hidden, gen, device)
        self.head = self.embd  # tied lm_head (a GGUF file with output.weight replaces it)
        self.out_norm = 1.0 + 0.1 * tt.randn(c.hidden, generator=gen, **f32)
        # activations and device-side state
        z = lambda n: tt.zeros(n, **f32)
        self.x, self.h, self.q, self.k, self.v = z(c.hidden), z(c.hidden), z(nq), z(nkv), z(nkv)
        self.qr, self.kr = z(nq), z(nkv)
        self.attn, self.o = z(nq), z(c.hidden)
        self.gate, self.up, self.gu, self.dn = z(c.ffn), z(c.ffn), z(c.ffn), z(c.hidden)
        self.qkv, self.gu2 = z(nq + 2 * nkv), z(2 * c.ffn)
        self.logits = z(c.vocab)
        self.scores, self.probs = z(c.n_head * c.n_ctx), z(c.n_head * c.n_ctx)
        self.mask = z(c.n_ctx)
        self.q16 = tt.zeros(nq, dtype=tt.float16, device=device)
        self.p16 = tt.zeros(c.n_head * c.n_ctx, dtype=tt.float16, device=device)
        qb = lambda n: tt.zeros(n // 32 * 36, dtype=tt.uint8, device=device)
        self.hq, self.aq, self.gq = qb(c.hidden), qb(nq), qb(c.ffn)
        self.token = tt.zeros(1, dtype=tt.int32, device=device)
        self.pos = tt.zeros(1, dtype=tt.int32, device=device)
        self.launches_per_step = 0
        # the weights and state above were written on torch's current stream; steps may run on
        # another one
        tt.cuda.current_stream().synchronize()

    def reset(self, token, pos=None):
        """Sets the token and position (on torch's current stream) and waits for them: the step
        may be enqueued on another stream, whose kernels must not read them half-written."""
        self.token.fill_(int(token))
        self.pos.fill_(self.cfg.prompt if pos is None else int(pos))
        self.t.cuda.current_stream().synchronize()

    def _chk(self, rc, what):
        if rc != 0:
            raise RuntimeError("%s failed: %d" % (what, rc))
        self.launches_per_step += 1

    def step(self, stream):
        """Enqueue one token step on `stream` (a cudaStream_t).  GEMVs over weight matrices under
        `row_gemv_below_kb` (default 8 MB) take the substitution layer's row kernel
        (CFI_MMVQ_STREAM_MIN_KB, set for the duration of the call unless the environment sets it):
        between the short kernels of a decode step it measured faster than the streaming kernel,
        which serves the stacked gate/up matrix (9 MB, its weights fetched before the dependent-launch
        wait on a const-weights context) and the lm_head."""
        import os

        key = "CFI_MMVQ_STREAM_MIN_KB"
        prev = os.environ.get(key)
        if prev is None and self.row_gemv_below_kb:
            os.environ[key] = str(int(self.row_gemv_below_kb))
        try:
            return self._step(stream)
        finally:
            if prev is None and self.row_gemv_below_kb:
                del os.environ[key]

    def _step(self, stream):
        if self.fused == 3:
            return self.step_persistent(stream)
        if self.fused:
            return self.step_fused(stream)
        c, g, L, s = self.cfg, self.g, self.L, stream
        P = lambda t: C.c_void_p(t.data_ptr())
        sv = C.c_void_p(s)
        nq, nkv, grp = c.n_head * c.head_dim, c.n_kv_head * c.head_dim, c.n_head // c.n_kv_head
        self.launches_per_step = 0
        self._chk(L.cfi_glue_get_rows_q8_0(P(self.embd), P(self.token), P(self.x), c.hidden, sv), "get_rows")
        self._chk(L.cfi_glue_causal_mask(P(self.mask), P(self.pos), c.n_ctx, sv), "mask")

        def gemv(w, xq, out, rows, k):
            g.mmvq(cfi.Q8_0, 1, w.data_ptr(), xq.data_ptr(), out.data_ptr(), k, rows, stream=s)
            self.launches_per_step += 1

        def quant(x, xq, k):
            g.quantize_q8_1(x.data_ptr(), xq.data_ptr(), k, k, 1, stream=s)
            self.launches_per_step += 1

        B = cfi.Blas
        self.blas.set_stream(s)
        for lay in self.layers:
            g.rms_norm(self.x.data_ptr(), self.h.data_ptr(), c.hidden, 1, mul=lay["attn_norm"].data_ptr(), eps=c.eps,
                       stream=s)
            quant(self.h, self.hq, c.hidden)
            gemv(lay["wq"], self.hq, self.q, nq, c.hidden)
            gemv(lay["wk"], self.hq, self.k, nkv, c.hidden)
            gemv(lay["wv"], self.hq, self.v, nkv, c.hidden)
            self._chk(L.cfi_glue_qkv_bias(P(self.q), P(self.k), P(self.v), P(lay["bq"]), P(lay["bk"]), P(lay["bv"]),
                                          nq, nkv, sv), "bias")
            g.rope_neox(self.q.data_ptr(), self.qr.data_ptr(), c.head_dim, c.n_head, 1, c.head_dim, self.pos.data_ptr(),
                        freq_base=c.theta, stream=s)
            g.rope_neox(self.k.data_ptr(), self.kr.data_ptr(), c.head_dim, c.n_kv_head, 1, c.head_dim,
                        self.pos.data_ptr(), freq_base=c.theta, stream=s)
            self._chk(L.cfi_glue_kv_store(P(self.qr), P(self.kr), P(self.v), P(self.q16), P(lay["kc"]), P(lay["vc"]),
                                          P(self.pos), nq, nkv, c.head_dim, c.n_ctx, sv), "kv_store")
            # KQ: per KV head, scores[h][j] = K[j] . q_h for its `grp` query heads
            rc = self.blas.gemm_strided_batched_ex(
                B.OP_T, B.OP_N, c.n_ctx, grp, c.head_dim, 1.0, lay["kc"].data_ptr(), B.R_16F, c.head_dim,
                c.n_ctx * c.head_dim, self.q16.data_ptr(), B.R_16F, c.head_dim, grp * c.head_dim, 0.0,
                self.scores.data_ptr(), B.R_32F, c.n_ctx, grp * c.n_ctx, c.n_kv_head)
            self._chk(rc, "KQ")
            g.soft_max(self.scores.data_ptr(), self.mask.data_ptr(), self.probs.data_ptr(), c.n_ctx, 1, c.n_head,
                       1.0 / math.sqrt(c.head_dim), stream=s)
            self._chk(L.cfi_glue_to_f16(P(self.probs), P(self.p16), c.n_head * c.n_ctx, sv), "to_f16")
            # KQV: out_h = V P_h
            rc = self.blas.gemm_strided_batched_ex(
                B.OP_T, B.OP_N, c.head_dim, grp, c.n_ctx, 1.0, lay["vc"].data_ptr(), B.R_16F, c.n_ctx,
                c.head_dim * c.n_ctx, self.p16.data_ptr(), B.R_16F, c.n_ctx, grp * c.n_ctx, 0.0,
                self.attn.data_ptr(), B.R_32F, c.head_dim, grp * c.head_dim, c.n_kv_head)
            self._chk(rc, "KQV")
            quant(self.attn, self.aq, nq)
            gemv(lay["wo"], self.aq, self.o, c.hidden, nq)
            self._chk(L.cfi_glue_add(P(self.x), P(self.o), c.hidden, sv), "add")
            g.rms_norm(self.x.data_ptr(), self.h.data_ptr(), c.hidden, 1, mul=lay["ffn_norm"].data_ptr(), eps=c.eps,
                       stream=s)
            quant(self.h, self.hq, c.hidden)
            gemv(lay["wg"], self.hq, self.gate, c.ffn, c.hidden)
            gemv(lay["wu"], self.hq, self.up, c.ffn, c.hidden)
            self._chk(L.cfi_glue_swiglu(P(self.gate), P(self.up), P(self.gu), c.ffn, sv), "swiglu")
            quant(self.gu, self.gq, c.ffn)
            gemv(lay["wd"], self.gq, self.dn, c.hidden, c.ffn)
            self._chk(L.cfi_glue_add(P(self.x), P(self.dn), c.hidden, sv), "add")
            self.launches_per_step += 5  # rms_norm x2, rope x2, soft_max
        g.rms_norm(self.x.data_ptr(), self.h.data_ptr(), c.hidden, 1, mul=self.out_norm.data_ptr(), eps=c.eps, stream=s)
        quant(self.h, self.hq, c.hidden)
        gemv(self.head, self.hq, self.logits, c.vocab, c.hidden)
        self._chk(L.cfi_glue_argmax_next(P(self.logits), c.vocab, P(self.token), P(self.pos), sv), "argmax")
        self.launches_per_step += 1  # the output rms_norm

    def step_fused(self, stream):
        """One token step with the stacked weights and the fused glue kernels.  fused == 2: the
        element-wise steps after the QKV, O, gate/up and down GEMVs run in those GEMVs' last CTAs
        (5 launches per layer); fused == 1: as separate launches (9 per layer)."""
        if self.fused == 2:
            return self.step_fused_epi(stream)
        c, g, L, s = self.cfg, self.g, self.L, stream
        P = lambda t: C.c_void_p(t.data_ptr())
        sv = C.c_void_p(s)
        nq, nkv = c.n_head * c.head_dim, c.n_kv_head * c.head_dim
        eps, theta, scale = C.c_float(c.eps), C.c_float(c.theta), C.c_float(1.0 / math.sqrt(c.head_dim))
        self.launches_per_step = 0

        def gemv(w, xq, out, rows, k):
            g.mmvq(cfi.Q8_0, 1, w.data_ptr(), xq.data_ptr(), out.data_ptr(), k, rows, stream=s)
            self.launches_per_step += 1

        self._chk(L.cfi_glue_get_rows_q8_0(P(self.embd), P(self.token), P(self.x), c.hidden, sv), "get_rows")
        resid = None
        for lay in self.layers:
            self._chk(L.cfi_fused_add_rmsnorm_q8_1(P(self.x), resid, P(lay["attn_norm"]), P(self.hq), c.hidden, eps, sv),
                      "add_rmsnorm")
            gemv(lay["wqkv"], self.hq, self.qkv, nq + 2 * nkv, c.hidden)
            self._chk(L.cfi_fused_qkv_rope_store(P(self.qkv), P(lay["bqkv"]), P(self.qr), P(lay["kc"]), P(lay["vc"]),
                                                 P(self.pos), nq, nkv, c.head_dim, c.n_ctx, theta, sv), "qkv_rope")
            self._chk(L.cfi_fused_attention_q8_1(P(self.qr), P(lay["kc"]), P(lay["vc"]), P(self.pos), P(self.aq),
                                                 c.n_head, c.n_kv_head, c.head_dim, c.n_ctx, scale, sv), "attention")
            gemv(lay["wo"], self.aq, self.o, c.hidden, nq)
            self._chk(L.cfi_fused_add_rmsnorm_q8_1(P(self.x), P(self.o), P(lay["ffn_norm"]), P(self.hq), c.hidden, eps,
                                                   sv), "add_rmsnorm")
            gemv(lay["wgu"], self.hq, self.gu2, 2 * c.ffn, c.hidden)
            self._chk(L.cfi_fused_swiglu_q8_1(P(self.gu2), P(self.gq), c.ffn, sv), "swiglu")
            gemv(lay["wd"], self.gq, self.dn, c.hidden, c.ffn)
            resid = P(self.dn)
        self._chk(L.cfi_fused_add_rmsnorm_q8_1(P(self.x), resid, P(self.out_norm), P(self.hq), c.hidden, eps, sv),
                  "add_rmsnorm")
        gemv(self.head, self.hq, self.logits, c.vocab, c.hidden)
        self._chk(L.cfi_glue_argmax_next(P(self.logits), c.vocab, P(self.token), P(self.pos), sv), "argmax")

    def step_persistent(self, stream):
        """fused == 3: the whole step of fused == 1 as one persistent launch (cfi_decode_step_q8_0,
        grid-wide barriers between the phases), its results equal to that chain's bit for bit."""
        c, L = self.cfg, self.L
        if getattr(self, "_ds", None) is None:
            a = lambda t: t.data_ptr()
            lays = (cfi.DecodeLayer * c.layers)()
            for i, lay in enumerate(self.layers):
                lays[i] = cfi.DecodeLayer(a(lay["wqkv"]), a(lay["bqkv"]), a(lay["wo"]), a(lay["wgu"]), a(lay["wd"]),
                                          a(lay["attn_norm"]), a(lay["ffn_norm"]), a(lay["kc"]), a(lay["vc"]))
            raw = bytes(lays)
            self._ds_layers = self.t.frombuffer(bytearray(raw), dtype=self.t.uint8).to(self.dev)
            self.t.cuda.current_stream().synchronize()
            self._ds = cfi.DecodeStep(c.hidden, c.n_head, c.n_kv_head, c.head_dim, c.ffn, c.vocab, c.n_ctx, c.layers,
                                      c.eps, c.theta, a(self.embd), a(self.head), a(self.out_norm), a(self.x), a(self.qkv),
                                      a(self.qr), a(self.o), a(self.gu2), a(self.dn), a(self.logits), a(self.hq), a(self.aq),
                                      a(self.gq), a(self.token), a(self.pos))
        self.launches_per_step = 1
        rc = L.cfi_decode_step_q8_0(C.byref(self._ds), C.c_void_p(self._ds_layers.data_ptr()), C.c_void_p(stream))
        if rc != 0:
            raise RuntimeError("cfi_decode_step_q8_0 failed: %d" % rc)

    def step_fused_epi(self, stream):
        c, L = self.cfg, self.L
        P = lambda t: C.c_void_p(t.data_ptr())
        sv = C.c_void_p(stream)
        nq, nkv = c.n_head * c.head_dim, c.n_kv_head * c.head_dim
        eps, theta, scale = C.c_float(c.eps), C.c_float(c.theta), C.c_float(1.0 / math.sqrt(c.head_dim))
        self.launches_per_step = 0
        self._chk(L.cfi_glue_get_rows_q8_0(P(self.embd), P(self.token), P(self.x), c.hidden, sv), "get_rows")
        self._chk(L.cfi_fused_add_rmsnorm_q8_1(P(self.x), None, P(self.layers[0]["attn_norm"]), P(self.hq), c.hidden, eps,
                                               sv), "add_rmsnorm")
        for i, lay in enumerate(self.layers):
            if self.epi_qkv:
                self._chk(L.cfi_fused_mmvq_qkv_rope_store(P(lay["wqkv"]), P(self.hq), P(self.qkv), c.hidden,
                                                          P(lay["bqkv"]), P(self.qr), P(lay["kc"]), P(lay["vc"]),
                                                          P(self.pos), nq, nkv, c.head_dim, c.n_ctx, theta, sv), "qkv")
            else:
                self.g.mmvq(cfi.Q8_0, 1, lay["wqkv"].data_ptr(), self.hq.data_ptr(), self.qkv.data_ptr(), c.hidden,
                            nq + 2 * nkv, stream=stream)
                self.launches_per_step += 1
                self._chk(L.cfi_fused_qkv_rope_store(P(self.qkv), P(lay["bqkv"]), P(self.qr), P(lay["kc"]), P(lay["vc"]),
                                                     P(self.pos), nq, nkv, c.head_dim, c.n_ctx, theta, sv), "qkv_rope")
            self._chk(L.cfi_fused_attention_q8_1(P(self.qr), P(lay["kc"]), P(lay["vc"]), P(self.pos), P(self.aq),
                                                 c.n_head, c.n_kv_head, c.head_dim, c.n_ctx, scale, sv), "attention")
            self._chk(L.cfi_fused_mmvq_add_rmsnorm_q8_1(P(lay["wo"]), P(self.aq), P(self.o), c.hidden, nq, P(self.x),
                                                        P(lay["ffn_norm"]), P(self.hq), eps, sv), "o")
            if self.epi_swiglu:
                self._chk(L.cfi_fused_mmvq_swiglu_q8_1(P(lay["wgu"]), P(self.hq), P(self.gu2), 2 * c.ffn, c.hidden,
                                                       P(self.gq), sv), "gate_up")
            else:
                self.g.mmvq(cfi.Q8_0, 1, lay["wgu"].data_ptr(), self.hq.data_ptr(), self.gu2.data_ptr(), c.hidden,
                            2 * c.ffn, stream=stream)
                self.launches_per_step += 1
                self._chk(L.cfi_fused_swiglu_q8_1(P(self.gu2), P(self.gq), c.ffn, sv), "swiglu")
            nxt = self.layers[i + 1]["attn_norm"] if i + 1 < len(self.layers) else self.out_norm
            self._chk(L.cfi_fused_mmvq_add_rmsnorm_q8_1(P(lay["wd"]), P(self.gq), P(self.dn), c.hidden, c.ffn, P(self.x),
                                                        P(nxt), P(self.hq), eps, sv), "down")
        self.g.mmvq(cfi.Q8_0, 1, self.head.data_ptr(), self.hq.data_ptr(), self.logits.data_ptr(), c.hidden, c.vocab,
                    stream=stream)
        self.launches_per_step += 1
        self._chk(L.cfi_glue_argmax_next(P(self.logits), c.vocab, P(self.token), P(self.pos), sv), "argmax")


# ---- GGUF (llama.cpp's qwen2 tensor names; include/cfi_gguf.h reads the file) ----
GGUF_LAYER = {"attn_norm.weight": "attn_norm", "attn_q.weight": "wq", "attn_q.bias": "bq", "attn_k.weight": "wk",
              "attn_k.bias": "bk", "attn_v.weight": "wv", "attn_v.bias": "bv", "attn_output.weight": "wo",
              "ffn_norm.weight": "ffn_norm", "ffn_gate.weight": "wg", "ffn_up.weight": "wu", "ffn_down.weight": "wd"}
_Q8_0, _F32 = 8, 0


def _gguf_shape(name, c):
    """(ggml type, dims with ne[0] innermost) of a per-layer tensor of config c."""
    nq, nkv = c.n_head * c.head_dim, c.n_kv_head * c.head_dim
    mats = {"wq": (c.hidden, nq), "wk": (c.hidden, nkv), "wv": (c.hidden, nkv), "wo": (nq, c.hidden),
            "wg": (c.hidden, c.ffn), "wu": (c.hidden, c.ffn), "wd": (c.ffn, c.hidden)}
    vecs = {"bq": nq, "bk": nkv, "bv": nkv, "attn_norm": c.hidden, "ffn_norm": c.hidden}
    return (_Q8_0, mats[name]) if name in mats else (_F32, (vecs[name],))


def save_gguf(model, path):
    """Writes the model's weights (Q8_0 matrices, f32 norms and biases) as a qwen2 GGUF file."""
    import gguf as G

    c = model.cfg
    kv = {"general.architecture": (G.STRING, "qwen2"), "qwen2.block_count": (G.U32, c.layers),
          "qwen2.embedding_length": (G.U32, c.hidden), "qwen2.feed_forward_length": (G.U32, c.ffn),
          "qwen2.attention.head_count": (G.U32, c.n_head), "qwen2.attention.head_count_kv": (G.U32, c.n_kv_head),
          "qwen2.attention.layer_norm_rms_epsilon": (G.F32, c.eps), "qwen2.rope.freq_base": (G.F32, c.theta),
          "qwen2.context_length": (G.U32, c.n_ctx)}
    host = lambda t: t.detach().contiguous().cpu().numpy().tobytes()
    ts = [("token_embd.weight", _Q8_0, (c.hidden, c.vocab), host(model.embd))]
    for i, lay in enumerate(model.layers):
        for gname, key in GGUF_LAYER.items():
            ty, dims = _gguf_shape(key, c)
            ts.append(("blk.%d.%s" % (i, gname), ty, dims, host(lay[key])))
    ts.append(("output_norm.weight", _F32, (c.hidden,), host(model.out_norm)))
    if model.head is not model.embd:
        ts.append(("output.weight", _Q8_0, (c.hidden, c.vocab), host(model.head)))
    G.write_gguf(path, kv, ts)


def load_gguf(torch, ctx, device, path, fused=False, prompt=None, n_ctx=None, seed=0x5eed):
    """A DecodeModel with the weights of a qwen2 GGUF file (Q8_0 matrices, f32 norms and biases,
    as in a Q8_0 model export; other matrix types are refused).  The KV cache of the prompt
    positions stays seeded random (no prefill is run)."""
    import gguf as G

    with G.GGUFFile(path) as f:
        if f.get("general.architecture") != "qwen2":
            raise G.GGUFError("not a qwen2 model: %r" % f.get("general.architecture"))
        a = lambda k, default=None: f.get("qwen2." + k, default)
        _, edims, _ = f.tensor("token_embd.weight")
        hidden, nh = int(a("embedding_length")), int(a("attention.head_count"))
        cfg = Config(hidden=hidden, layers=int(a("block_count")), n_head=nh, n_kv_head=int(a("attention.head_count_kv")),
                     head_dim=hidden // nh, ffn=int(a("feed_forward_length")), vocab=int(edims[1]),
                     eps=float(a("attention.layer_norm_rms_epsilon")), theta=float(a("rope.freq_base", 1e6)))
        if prompt is not None:
            cfg.prompt = prompt
        if n_ctx is not None:
            cfg.n_ctx = n_ctx
        m = DecodeModel(torch, ctx, device, cfg, seed=seed, fused=fused)

        def put(dst, name, ty, dims):
            gty, gdims, data = f.tensor(name)
            if gty != ty or tuple(gdims) != tuple(dims):
                raise G.GGUFError("%s: type %d dims %s, this driver needs type %d dims %s" % (name, gty, gdims, ty, dims))
            src = torch.from_numpy(data.copy()).to(device)
            dst.view(torch.uint8).reshape(-1).copy_(src)

        put(m.embd, "token_embd.weight", _Q8_0, (hidden, cfg.vocab))
        for i, lay in enumerate(m.layers):
            for gname, key in GGUF_LAYER.items():
                ty, dims = _gguf_shape(key, cfg)
                put(lay[key], "blk.%d.%s" % (i, gname), ty, dims)
        put(m.out_norm, "output_norm.weight", _F32, (hidden,))
        names = f.tensor_names()
        if "output.weight" in names:
            m.head = torch.empty_like(m.embd)
            put(m.head, "output.weight", _Q8_0, (hidden, cfg.vocab))
    torch.cuda.current_stream().synchronize()  # the copies above, before steps on any stream
    return m

