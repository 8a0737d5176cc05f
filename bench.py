"""Benchmark of the substitution hot path on B200 (one JSON line on rank 0).

Workload: quantize_q8_1 of fp32 activations + Q4_K mul_mat_vec_q over an
8192 x 2048 Q4_K weight matrix at batch 1, 2, 4 and 8 columns.  One step = the four
(quantize, GEMV) pairs.  Metric: GB/s of algorithmic bytes (weights + q8_1 activations + fp32
outputs + quantizer traffic) against the measured HBM peak.  Weights rotate over enough copies
that every GEMV reads from HBM (inputs larger than L2).  Kernels are launched through the
substitution C ABI (cfi_subst_launch with ggml kernelParams) and each step is replayed as a
CUDA graph.  With --gpus N (torchrun) every rank owns an 8192-row shard of an (8192 N) x 2048
matrix (weak scaling) and the outputs are all-gathered over NCCL each step (step i gathers
step i-1's outputs on a second stream while its own kernels run, all inside the step's graph).

--impl reference times the CPU evaluation of the same step (the oracle port of the reference's
host math, row-parallel over every host core) on rank 0.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cuda-for-intel_b200"))

ROWS, K, BATCHES = 8192, 2048, (1, 2, 4, 8)
W_BYTES = ROWS * K // 256 * 144                       # 9,437,184
Q81 = lambda b: b * K // 32 * 36                       # q8_1 bytes of b columns
MMVQ_BYTES = lambda b: W_BYTES + b * (Q81(1) + ROWS * 4)
QUANT_BYTES = lambda b: b * (K * 4 + Q81(1))
STEP_BYTES = sum(MMVQ_BYTES(b) + QUANT_BYTES(b) for b in BATCHES)
L2_BYTES = 126 * 1024 * 1024
METRIC = "Q4_K decode GEMV + quantize_q8_1 throughput (8192x2048, batch 1/2/4/8)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + q,
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def traffic_per_launch(fused=False):
    """dram bytes per launch of the roofline kernel (the GEMV, or the GEMV that absorbed its
    quantize_q8_1) from the committed ncu summary, if one exists."""
    p = os.path.join(ROOT, "profiles", "mmvq_q4k_8192x2048_traffic.json")
    try:
        with open(p) as f:
            return float(json.load(f)["dram_bytes_per_launch_b1_fused" if fused else "dram_bytes_per_launch_b1"])
    except Exception:
        return None


def prefill_gemm(cfi, g, stream, dev, peak_tf):
    """Q8_0 weights (4864x896 and 896x4864) x 631 tokens quantised to
    q8_1_mmq, through the native mul_mat_q (tcgen05).  CUDA graph of back-to-back calls."""
    import torch

    out = {}
    for m, k in ((4864, 896), (896, 4864)):
        n = 631
        w = torch.from_numpy(cfi.synthetic_weights(cfi.Q8_0, m, k, seed=m)).to(dev)
        xf = torch.from_numpy(np.random.default_rng(k).normal(size=(n, k)).astype(np.float32)).to(dev)
        q = torch.zeros(k // 128 * n * 144, dtype=torch.uint8, device=dev)
        d = torch.zeros(n * m, dtype=torch.float32, device=dev)
        with torch.cuda.stream(stream):
            g.quantize_mmq(0, xf.data_ptr(), q.data_ptr(), k, k, n, stream=stream.cuda_stream)
            g.mmq(cfi.Q8_0, w.data_ptr(), q.data_ptr(), d.data_ptr(), k, m, n, stream=stream.cuda_stream)
        torch.cuda.synchronize()
        reps, calls = 5, 20
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for _ in range(calls):
                g.mmq(cfi.Q8_0, w.data_ptr(), q.data_ptr(), d.data_ptr(), k, m, n,
                      stream=torch.cuda.current_stream().cuda_stream)
        with torch.cuda.stream(stream):
            gr.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                gr.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * calls)
        out["%dx%dx%d" % (m, k, n)] = {"us": round(us, 2), "tflops": round(2.0 * m * n * k / us / 1e6, 1)}
        del gr
    # the cuBLAS-compatible GemmEx path on the same shapes (ggml's T,N f16 -> f32 call)
    blas = cfi.Blas(stream.cuda_stream)
    gemm = {}
    for m, k in ((4864, 896), (896, 4864)):
        n = 631
        A = torch.randn(m, k, device=dev).half()
        B = torch.randn(n, k, device=dev).half()
        C = torch.zeros(n, m, device=dev)
        def call(st):
            blas.set_stream(st)
            blas.gemm_ex(1, 0, m, n, k, 1.0, A.data_ptr(), 2, k, B.data_ptr(), 2, k, 0.0, C.data_ptr(), 0, m)
        with torch.cuda.stream(stream):
            call(stream.cuda_stream)
        torch.cuda.synchronize()
        reps, calls = 5, 20
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for _ in range(calls):
                call(torch.cuda.current_stream().cuda_stream)
        with torch.cuda.stream(stream):
            gr.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                gr.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * calls)
        gemm["%dx%dx%d" % (m, n, k)] = {"us": round(us, 2), "tflops": round(2.0 * m * n * k / us / 1e6, 1),
                                         "path": "tcgen05" if blas.last_path() == 1 else "simt"}
        del gr
    blas.close()
    best = max(v["tflops"] for v in out.values())
    return {"workload": "config3: Q8_0 W x 631 q8_1_mmq tokens -> f32 (mul_mat_q on tcgen05, incl. activation pre-pass)",
            "shapes": out, "gemm_ex_f16": gemm,
            "roofline": {"bound": "tensor", "achieved": best, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": round(best / peak_tf, 4), "peak_kind": "measured bf16 dense (burst)"}}


def graph_time_us(stream, body, reps=5, calls=1):
    """Capture `calls` x body(stream_handle) in one CUDA graph; mean device time per body call (µs)
    over `reps` replays after one warm replay, CUDA events on the launching stream."""
    import torch

    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        for i in range(calls):
            body(i, torch.cuda.current_stream().cuda_stream)
    with torch.cuda.stream(stream):
        gr.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            gr.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * calls)
    del gr
    return us


def config1_bench(cfi, g, stream, dev, peak, gf=None):
    """Q8_0 mul_mat_vec_q 4864x896 on its own (batch 1), and with its
    quantize_q8_1 in front, back to back over rotated weight copies (> 3x L2)."""
    import torch

    rows, k = 4864, 896
    wb = rows * k // 32 * 34
    ncopy = int(np.ceil(3 * L2_BYTES / wb))
    w = torch.from_numpy(cfi.synthetic_weights(cfi.Q8_0, rows, k, seed=11).ravel()).to(dev)
    wd = torch.empty((ncopy, w.numel()), dtype=torch.uint8, device=dev)
    wd[:] = w
    x = torch.from_numpy(np.random.default_rng(3).normal(size=k).astype(np.float32)).to(dev)
    q = torch.zeros(k // 32 * 36, dtype=torch.uint8, device=dev)
    y = torch.zeros(rows, dtype=torch.float32, device=dev)
    with torch.cuda.stream(stream):
        g.quantize_q8_1(x.data_ptr(), q.data_ptr(), k, k, 1, stream=stream.cuda_stream)
        g.mmvq(cfi.Q8_0, 1, wd[0].data_ptr(), q.data_ptr(), y.data_ptr(), k, rows, stream=stream.cuda_stream)
    torch.cuda.synchronize()
    mm = lambda i, st: g.mmvq(cfi.Q8_0, 1, wd[i].data_ptr(), q.data_ptr(), y.data_ptr(), k, rows, stream=st)

    def pair(i, st):
        g.quantize_q8_1(x.data_ptr(), q.data_ptr(), k, k, 1, stream=st)
        mm(i, st)
    us = graph_time_us(stream, mm, calls=ncopy)
    us_pair = graph_time_us(stream, pair, calls=ncopy)
    mbytes = wb + k // 32 * 36 + rows * 4                 # 4,650,992
    qbytes = k * 4 + k // 32 * 36
    fused = {}
    if gf is not None:
        def fpair(i, st):
            gf.quantize_q8_1(x.data_ptr(), q.data_ptr(), k, k, 1, stream=st)
            gf.mmvq(cfi.Q8_0, 1, wd[i].data_ptr(), q.data_ptr(), y.data_ptr(), k, rows, stream=st)
        with torch.cuda.stream(stream):
            fpair(0, stream.cuda_stream)  # first use outside the capture
        torch.cuda.synchronize()
        us_f = graph_time_us(stream, fpair, calls=ncopy)
        fused = {"fused_quantize_plus_mmvq_us": round(us_f, 3),
                 "fused_quantize_plus_mmvq_gbs": round((mbytes + qbytes) / us_f / 1e3, 1)}
    return {**fused, "workload": "config1: Q8_0 mul_mat_vec_q 4864x896, batch 1 (weights rotated over %d copies, %.0f MB)"
                        % (ncopy, ncopy * wb / 1e6),
            "mmvq_us": round(us, 3), "mmvq_gbs": round(mbytes / us / 1e3, 1),
            "mmvq_frac": round(mbytes / us / 1e3 / peak, 4),
            "quantize_plus_mmvq_us": round(us_pair, 3), "quantize_plus_mmvq_gbs": round((mbytes + qbytes) / us_pair / 1e3, 1),
            "bytes_per_call": mbytes}


def config5_bench(cfi, g, stream, dev, peak_gbs, peak_tf):
    """Qwen2.5-1.5B-architecture weight products, 28 layers of Q4_K matrices
    (q, o 1536x1536; k, v 256x1536; gate, up 8960x1536; down 1536x8960) and the Q8_0 head
    151936x1536: (a) a 631-token prefill -- per layer the activations quantised to q8_1_mmq once
    per distinct input (attention input, attention output, FFN input, FFN hidden) and the seven
    mul_mat_q products; the head on the last token only (quantize_q8_1 + mul_mat_vec_q), as ggml
    does; (b) one batch-64 decode step of 64 independent sequences -- the same products with 64
    columns (mul_mat_q, as ggml uses above 8 columns), the head included.  Attention and the
    element-wise ops are not in this leg.  Weights random, device-side (seeded)."""
    import torch

    from decode import random_q4_k, random_q8_0

    H, F, KV, L, V = 1536, 8960, 256, 28, 151936
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    shapes = {"q": (H, H), "k": (KV, H), "v": (KV, H), "o": (H, H), "g": (F, H), "u": (F, H), "d": (H, F)}
    layers = [{n: random_q4_k(torch, r, c, gen, dev) for n, (r, c) in shapes.items()} for _ in range(L)]
    head = random_q8_0(torch, V, H, gen, dev)
    wbytes = sum(t.numel() for lay in layers for t in lay.values()) + head.numel()
    params = L * sum(r * c for r, c in shapes.values())

    def buffers(n):
        xf = {kk: torch.randn(n * kk, generator=gen, device=dev) for kk in (H, F)}
        xq = {kk: torch.zeros(kk // 128 * n * 144, dtype=torch.uint8, device=dev) for kk in (H, F)}
        out = {nm: torch.zeros(n * r, dtype=torch.float32, device=dev) for nm, (r, c) in shapes.items()}
        return xf, xq, out

    def layer_products(n, xf, xq, out, st):
        for lay in layers:
            for inputs, k in ((("q", "k", "v"), H), (("o",), H), (("g", "u"), H), (("d",), F)):
                g.quantize_mmq(1, xf[k].data_ptr(), xq[k].data_ptr(), k, k, n, stream=st)
                for nm in inputs:
                    r = shapes[nm][0]
                    g.mmq(cfi.Q4_K, lay[nm].data_ptr(), xq[k].data_ptr(), out[nm].data_ptr(), k, r, n, stream=st)

    # (a) prefill, 631 tokens
    n = 631
    xf, xq, out = buffers(n)
    hq = torch.zeros(H // 32 * 36, dtype=torch.uint8, device=dev)
    logits = torch.zeros(V, dtype=torch.float32, device=dev)

    def prefill(i, st):
        layer_products(n, xf, xq, out, st)
        g.quantize_q8_1(xf[H].data_ptr() + (n - 1) * H * 4, hq.data_ptr(), H, H, 1, stream=st)
        g.mmvq(cfi.Q8_0, 1, head.data_ptr(), hq.data_ptr(), logits.data_ptr(), H, V, stream=st)
    with torch.cuda.stream(stream):
        prefill(0, stream.cuda_stream)
    torch.cuda.synchronize()
    us_pf = graph_time_us(stream, prefill, reps=3)
    pf_ops = 2.0 * params * n + 2.0 * V * H
    # (b) batch-64 decode step
    n = 64
    xf, xq, out = buffers(n)
    hq64 = torch.zeros(H // 128 * n * 144, dtype=torch.uint8, device=dev)
    logits64 = torch.zeros(n * V, dtype=torch.float32, device=dev)

    def decode64(i, st):
        layer_products(n, xf, xq, out, st)
        g.quantize_mmq(0, xf[H].data_ptr(), hq64.data_ptr(), H, H, n, stream=st)
        g.mmq(cfi.Q8_0, head.data_ptr(), hq64.data_ptr(), logits64.data_ptr(), H, V, n, stream=st)
    with torch.cuda.stream(stream):
        decode64(0, stream.cuda_stream)
    torch.cuda.synchronize()
    us_dc = graph_time_us(stream, decode64, reps=5)
    launches = L * (4 + 7) + 2
    res = {"workload": "config5: Qwen2.5-1.5B-architecture weight products (28 layers Q4_K + Q8_0 head, %d B of "
                       "weights), 631-token prefill and a batch-64 decode step; attention not included" % wbytes,
           "prefill": {"ms": round(us_pf / 1e3, 3), "tok_per_s": round(631 / (us_pf * 1e-6), 1),
                       "tflops": round(pf_ops / us_pf / 1e6, 1), "frac": round(pf_ops / us_pf / 1e6 / peak_tf, 4),
                       "launches": launches},
           "decode_b64": {"ms": round(us_dc / 1e3, 3), "tok_per_s": round(64 / (us_dc * 1e-6), 1),
                          "weights_gbs": round(wbytes / us_dc / 1e3, 1),
                          "frac": round(wbytes / us_dc / 1e3 / peak_gbs, 4), "launches": launches}}
    del layers, head
    return res


def fattn_bench(cfi, g, stream, dev, peak_tf):
    """The native flash_attn_ext_f16 (tcgen05) on the prefill attention of BASELINE configs 4 and 5:
    631 queries against a 640-key padded causal cache (14 heads x 64 over 2 KV heads; 12 x 128 over
    2), CUDA graph of back-to-back calls.  FLOPs counted for the whole score matrix (4 nq nkv D H):
    masked keys are computed, not skipped."""
    import torch

    out = {}
    for d, nh, nhk in ((64, 14, 2), (128, 12, 2)):
        nq, nkv = 631, 640
        gen = torch.Generator(device=dev).manual_seed(d)
        q = torch.randn(nh * nq * d, generator=gen, device=dev)
        k = torch.randn(nhk * nkv * d, generator=gen, device=dev).half()
        v = torch.randn(nhk * nkv * d, generator=gen, device=dev).half()
        nq_pad = (nq + 15) // 16 * 16
        i = torch.arange(nq_pad, device=dev)[:, None]
        j = torch.arange(nkv, device=dev)[None, :]
        mask = torch.where(j <= i, 0.0, float("-inf")).half().contiguous()
        dst = torch.zeros(nq * nh * d, device=dev)
        call = lambda n, st: g.fattn(d, q.data_ptr(), k.data_ptr(), v.data_ptr(), mask.data_ptr(), dst.data_ptr(), nq,
                                     nh, nhk, nkv, 1, 1.0 / d ** 0.5, stream=st)
        with torch.cuda.stream(stream):
            call(0, stream.cuda_stream)
        torch.cuda.synchronize()
        us = graph_time_us(stream, call, reps=5, calls=20)
        fl = 4.0 * nq * nkv * d * nh
        out["d%d_h%d" % (d, nh)] = {"us": round(us, 2), "tflops": round(fl / us / 1e6, 1),
                                   "frac": round(fl / us / 1e6 / peak_tf, 4)}
    return {"workload": "flash_attn_ext_f16, 631 queries x 640 keys, causal mask (configs 4 / 5 prefill attention)",
            "shapes": out}


def decode_bench(stream, dev, ntok=48, warm=3, fused=False, defer=False, const_weights=False):
    """Qwen2.5-0.5B-architecture decode (24 layers, Q8_0 random weights, 631-token
    seeded KV cache), one CUDA graph per token step replayed for `ntok` greedy tokens.  fused: the
    stacked-weight step with the fused glue kernels (9 launches per layer instead of 25).  defer:
    ggml's sequence on a context that holds each quantize_q8_1 back for the GEMV reading it (every
    GEMV on the streaming kernel, which is the one that absorbs it).  const_weights: the GEMVs copy
    their weights before waiting on the previous kernel (CFI_CTX_CONST_WEIGHTS)."""
    import torch

    import cfi_b200 as cfi
    from decode import DecodeModel

    ctx = cfi.Ctx(dev.index or 0, defer_q8_1=defer, const_weights=const_weights)
    m = DecodeModel(torch, ctx, dev, fused=fused)
    if defer:
        m.row_gemv_below_kb = 0
    m.reset(token=1234)
    with torch.cuda.stream(stream):
        m.step(stream.cuda_stream)  # first-use probes outside the capture
    torch.cuda.synchronize()
    m.reset(token=1234)
    gr = torch.cuda.CUDAGraph()
    before = ctx.stats()["fused_q8_1"]
    with torch.cuda.graph(gr, stream=stream):
        m.step(torch.cuda.current_stream().cuda_stream)
        ctx.flush()
    fused_in_capture = ctx.stats()["fused_q8_1"] - before
    m.reset(token=1234)
    with torch.cuda.stream(stream):
        for _ in range(warm):
            gr.replay()
    torch.cuda.synchronize()
    m.reset(token=1234)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(ntok):
            gr.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    assert int(m.pos.item()) == m.cfg.prompt + ntok and cfi.lib().cfi_device_error() == 0
    bpt = m.cfg.weight_bytes_per_token()
    out = {"workload": "config4: Qwen2.5-0.5B-architecture decode, 24 layers, Q8_0 random weights, 631-token seeded "
                       "KV cache, %d greedy tokens, one CUDA graph per token%s"
                       % (ntok, {0: "; ggml's kernel sequence through the substitution ABI",
                                 1: "; stacked QKV / gate-up weights and fused glue kernels",
                                 2: "; stacked weights, element-wise steps in the GEMVs' last CTAs"}[int(fused)]
                          + ("; quantize_q8_1 held back into the GEMVs (CFI_CTX_DEFER_Q8_1)" if defer else "")
                          + ("; weights fetched before the dependent-launch wait (CFI_CTX_CONST_WEIGHTS)"
                             if const_weights else "")),
           "tok_per_s": round(ntok / (ms * 1e-3), 1), "ms_per_token": round(ms / ntok, 4),
           "launches_per_token": m.launches_per_step, "weight_bytes_per_token": bpt,
           "weights_gbs": round(bpt * ntok / (ms * 1e-3) / 1e9, 1)}
    if defer:
        out["launches_per_token"] -= fused_in_capture
    del gr
    ctx.close()
    return out


def cpu_baseline(seconds, threads=0):
    """The oracle's CPU decode step (reference host math, row-parallel) on a bounded sample."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import cfi_b200 as cfi
    import oracle_py as O

    w = cfi.synthetic_weights(cfi.Q4_K, ROWS, K, seed=7)
    xs = {b: np.random.default_rng(b).normal(size=(b, K)).astype(np.float32) for b in BATCHES}
    O.cpu_decode_step(cfi.Q4_K, w, ROWS, K, xs[1], 1, threads)
    n, t0, used = 0, time.perf_counter(), 1
    while True:
        for b in BATCHES:
            _, _, used = O.cpu_decode_step(cfi.Q4_K, w, ROWS, K, xs[b], b, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return STEP_BYTES * n / el / 1e9, used, n, el


def run_reference(args, rank, world):
    if rank != 0:
        return
    gbs, used, n, el = cpu_baseline(max(1.0, min(20.0, 0.5 * (args.steps + args.warmup))))
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * el / n, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "config": {"workload": "config2: Q4_K 8192x2048 GEMV + quantize_q8_1, batch 1/2/4/8"},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": used, "kind": "port",
                             "sample": "%d full steps in %.1f s" % (n, el)},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_gpu(args, rank, world):
    import torch

    import cfi_b200 as cfi

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        os.environ.setdefault("NCCL_DEBUG", "WARN")  # rank 0's stdout carries only the JSON line
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    # the step's router holds each quantize_q8_1 back for the GEMV that reads it (one kernel per
    # pair); --separate-quantize keeps them two launches
    defer = not args.separate_quantize
    ctx = cfi.Ctx(local, defer_q8_1=defer, const_weights=True)
    g = cfi.GgmlCaller(ctx, "all")
    # comparison legs (1 GPU): the same step launched separately, with and without the early
    # weight copies
    ctx_sep = cfi.Ctx(local, const_weights=True) if world == 1 else None
    g_sep = cfi.GgmlCaller(ctx_sep, "all") if ctx_sep else None
    ctx_plain = cfi.Ctx(local) if world == 1 else None
    g_plain = cfi.GgmlCaller(ctx_plain, "all") if ctx_plain else None
    stream = torch.cuda.Stream(device=dev)

    ncopy = max(8, int(np.ceil(3 * L2_BYTES / W_BYTES / 4.0)) * 4)   # > 3x L2 of weight copies
    w = cfi.synthetic_weights(cfi.Q4_K, ROWS, K, seed=7 + rank)
    wd = torch.empty((ncopy, w.size), dtype=torch.uint8, device=dev)
    wd[0].copy_(torch.from_numpy(w.ravel()))
    for i in range(1, ncopy):
        wd[i].copy_(wd[0])
    xs_host = {b: torch.from_numpy(np.random.default_rng(b).normal(size=(b, K)).astype(np.float32)).pin_memory()
               for b in BATCHES}
    xs = {b: xs_host[b].to(dev) for b in BATCHES}
    qs = {b: torch.zeros(Q81(b), dtype=torch.uint8, device=dev) for b in BATCHES}
    ys = {b: torch.zeros(b * ROWS, dtype=torch.float32, device=dev) for b in BATCHES}
    # two output sets: with N > 1 step i all-gathers step i-1's outputs while it computes its own
    y_sets = [torch.zeros(sum(b for b in BATCHES) * ROWS, dtype=torch.float32, device=dev) for _ in range(2)]
    y_all = y_sets[0]
    offs, o = {}, 0
    for b in BATCHES:
        offs[b] = o
        o += b * ROWS
    y_views_p = [{b: ya[offs[b]:offs[b] + b * ROWS] for b in BATCHES} for ya in y_sets]
    y_views = y_views_p[0]
    gathered = torch.zeros(world * y_all.numel(), dtype=torch.float32, device=dev) if world > 1 else None
    ys_host = torch.zeros(y_all.numel(), dtype=torch.float32).pin_memory()
    comm = torch.cuda.Stream(device=dev) if world > 1 else None

    def step(phase, s, parity=0, gg=None, xsrc=None):
        gg = gg or g
        xsrc = xsrc or xs
        for j, b in enumerate(BATCHES):
            gg.quantize_q8_1(xsrc[b].data_ptr(), qs[b].data_ptr(), K, K, b, stream=s)
            wcopy = wd[(phase * len(BATCHES) + j) % ncopy]
            gg.mmvq(cfi.Q4_K, b, wcopy.data_ptr(), qs[b].data_ptr(), y_views_p[parity][b].data_ptr(), K, ROWS, stream=s)
        gg.ctx.flush()

    def step_pipelined(phase, parity):
        """Inside a capture: the all-gather of the other output set on the comm stream (one exchange
        per step for the step's four sharded GEMVs) overlapping this step's kernels."""
        cur = torch.cuda.current_stream()
        if dist:
            fork = torch.cuda.Event()
            fork.record(cur)
            comm.wait_event(fork)
            with torch.cuda.stream(comm):
                dist.all_gather_into_tensor(gathered, y_sets[1 - parity])
        step(phase, cur.cuda_stream, parity)
        if dist:
            join = torch.cuda.Event()
            join.record(comm)
            cur.wait_event(join)

    nphase = ncopy // len(BATCHES)
    # warm-up (first-use probes run here, outside any capture)
    with torch.cuda.stream(stream):
        for i in range(max(1, args.warmup)):
            step(i % nphase, stream.cuda_stream)
            if dist:
                dist.all_gather_into_tensor(gathered, y_all)
    torch.cuda.synchronize()
    # Step i uses weight phase i % nphase and output set i % 2; that pattern repeats every
    # `period` steps, so one CUDA graph holds a whole period (programmatic dependent launch then
    # overlaps consecutive steps too, which separate graph launches would not) and a second graph
    # the first K % period steps, so the timed region runs exactly K steps.
    period = nphase if nphase % 2 == 0 else 2 * nphase

    def capture(nsteps):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for i in range(nsteps):
                step_pipelined(i % nphase, i % 2)
        return gr

    fused_before = ctx.stats()["fused_q8_1"]
    graph_period = capture(period)
    # GEMVs that absorbed their quantize, per captured step
    launches_per_step = 2 * len(BATCHES) - (ctx.stats()["fused_q8_1"] - fused_before) // period
    fused_step = launches_per_step < 2 * len(BATCHES)
    rest = args.steps % period
    graph_rest = capture(rest) if rest else None
    with torch.cuda.stream(stream):
        for _ in range((args.warmup + period - 1) // period):
            graph_period.replay()
    torch.cuda.synchronize()

    # ---- timed region: device time, max over ranks ----
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps // period):
                graph_period.replay()
            if graph_rest is not None:
                graph_rest.replay()
            e1.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = world * STEP_BYTES / (ms_step * 1e-3) / 1e9

    legs = {}
    for leg, gg, note in (("separate_launches", g_sep, "quantize_q8_1 and mul_mat_vec_q launched separately, "
                           "weights fetched before the wait (CFI_CTX_CONST_WEIGHTS)"),
                          ("plain_router", g_plain, "separate launches, no context flags (weights fetched "
                           "after the wait)")):
        if gg is None:
            continue
        with torch.cuda.stream(stream):
            step(0, stream.cuda_stream, 0, gg)  # first use outside the capture
        torch.cuda.synchronize()
        us_l = graph_time_us(stream, lambda i, st: step(i % nphase, st, 0, gg), reps=max(3, args.steps // 10),
                             calls=nphase)
        legs[leg] = {"value": round(STEP_BYTES / us_l / 1e3, 2), "ms_per_step": round(us_l * 1e-3, 5),
                     "launches_per_step": 2 * len(BATCHES), "router": note}

    # ---- dominant kernel: mmvq Q4_K batch 1, back to back (one graph of ncopy launches over the
    # rotated weight copies), CUDA events on the launching stream around the replays ----
    gk = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gk, stream=stream):
        for i in range(ncopy):
            if fused_step:  # the step's kernel: quantize_q8_1 absorbed by the GEMV
                g.quantize_q8_1(xs[1].data_ptr(), qs[1].data_ptr(), K, K, 1, stream=torch.cuda.current_stream().cuda_stream)
            g.mmvq(cfi.Q4_K, 1, wd[i].data_ptr(), qs[1].data_ptr(), y_views[1].data_ptr(), K, ROWS,
                   stream=torch.cuda.current_stream().cuda_stream)
        ctx.flush()
    reps = max(3, args.steps // 10)
    with torch.cuda.stream(stream):
        gk.replay()
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(stream)
        for _ in range(reps):
            gk.replay()
        k1.record(stream)
    torch.cuda.synchronize()
    kms = k0.elapsed_time(k1) / (reps * ncopy)
    peak, peak_kind = peaks()
    kbytes = MMVQ_BYTES(1) + (QUANT_BYTES(1) if fused_step else 0)
    achieved = kbytes / (kms * 1e-3) / 1e9

    # ---- end to end: host activations in, outputs back to the host, every step ----
    h2d = sum(xs_host[b].numel() * 4 for b in BATCHES)
    d2h = y_all.numel() * 4
    # Pipelined as a serving loop would run it: step i's activation copy and output copy run on
    # copy streams (one per direction) while steps i-1 / i+1 compute, with double-buffered device inputs and
    # outputs (parity i % 2) and event edges: H2D(i) after step i-2 has read its input buffer,
    # step i after H2D(i) and after D2H(i-2) has read its output buffer, D2H(i) after step i.
    # One CUDA graph holds a whole rotation period; the timed region ends when the last output
    # is on the host.
    nx = sum(b * K for b in BATCHES)
    x_host_all = torch.empty(nx, dtype=torch.float32).pin_memory()
    o = 0
    for b in BATCHES:
        x_host_all[o:o + b * K].copy_(xs_host[b].reshape(-1))
        o += b * K
    x_dev = [torch.empty(nx, dtype=torch.float32, device=dev) for _ in range(2)]
    x_views = []
    for xd in x_dev:
        vv, o = {}, 0
        for b in BATCHES:
            vv[b] = xd[o:o + b * K]
            o += b * K
        x_views.append(vv)
    y_host = [torch.empty(y_all.numel(), dtype=torch.float32).pin_memory() for _ in range(2)]
    copy_s = torch.cuda.Stream(device=dev)   # host -> device
    copy_o = torch.cuda.Stream(device=dev)   # device -> host (the other direction's copy engine)
    ev_h2d = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_d2h = [torch.cuda.Event() for _ in range(2)]
    # with N > 1 GPUs: step i's outputs are all-gathered on the comm stream after its kernels;
    # step i+2 waits for that collective before it rewrites the same output buffer
    ev_ag = [torch.cuda.Event() for _ in range(2)]
    gathered2 = [gathered, torch.zeros_like(gathered)] if dist else None

    def capture_e2e(nsteps):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            cur = torch.cuda.current_stream()
            fork = torch.cuda.Event()
            fork.record(cur)
            copy_s.wait_event(fork)
            copy_o.wait_event(fork)
            if dist:
                comm.wait_event(fork)
            for i in range(nsteps):
                p = i % 2
                with torch.cuda.stream(copy_s):
                    if i >= 2:
                        copy_s.wait_event(ev_comp[p])
                    x_dev[p].copy_(x_host_all, non_blocking=True)
                    ev_h2d[p].record(copy_s)
                cur.wait_event(ev_h2d[p])
                if i >= 2:
                    cur.wait_event(ev_d2h[p])
                    if dist:
                        cur.wait_event(ev_ag[p])
                step(i % nphase, cur.cuda_stream, p, xsrc=x_views[p])
                ev_comp[p].record(cur)
                if dist:
                    comm.wait_event(ev_comp[p])
                    with torch.cuda.stream(comm):
                        dist.all_gather_into_tensor(gathered2[p], y_sets[p])
                    ev_ag[p].record(comm)
                with torch.cuda.stream(copy_o):
                    copy_o.wait_event(ev_comp[p])
                    y_host[p].copy_(y_sets[p], non_blocking=True)
                    ev_d2h[p].record(copy_o)
            for cs in (copy_s, copy_o) + ((comm,) if dist else ()):
                join = torch.cuda.Event()
                join.record(cs)
                cur.wait_event(join)
        return gr

    ge = [capture_e2e(period)]
    e_rest = args.steps % period
    if e_rest:
        ge.append(capture_e2e(e_rest))
    with torch.cuda.stream(stream):
        ge[0].replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(args.steps // period):
            ge[0].replay()
        if e_rest:
            ge[1].replay()
    stream.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_note = ("host fp32 activations in (one pinned buffer) and fp32 outputs out (two pinned buffers) every "
                "step, weights resident; the copies (one stream per direction) overlap the neighbouring steps' kernels "
                "(double-buffered device inputs and outputs, event-ordered)%s, %d steps per CUDA graph, wall clock "
                "until the last output is on the host" % (", outputs all-gathered over NCCL on a third stream" if dist
                                                           else "", period))
    ge = []
    if dist:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * STEP_BYTES * args.steps / e2e_s / 1e9

    stats = ctx.stats()
    ok = stats["stock_launches"] == 0 and stats["native_failures"] == 0
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded N(0,0.02) weights quantized to Q4_K, "
                "N(0,1) activations)",
                "config": {"workload": "config2: Q4_K 8192x2048 GEMV + quantize_q8_1, batch 1/2/4/8",
                           "rows_per_gpu": ROWS, "k": K, "batches": list(BATCHES), "weight_copies": ncopy,
                           "l2": "inputs larger than L2: %d weight copies (%.0f MB) rotated" % (ncopy, ncopy * W_BYTES / 1e6),
                           "parallelism": "row-sharded x%d + NCCL all-gather" % world if world > 1 else "single GPU",
                           "bytes_per_step_per_gpu": STEP_BYTES,
                           "cuda_graph": "%d steps per graph (one period of the weight rotation)" % period,
                           "router": ("weights fetched before the dependent-launch wait (CFI_CTX_CONST_WEIGHTS)"
                                      + ("; quantize_q8_1 held back into its GEMV where the prologue is small "
                                         "(CFI_CTX_DEFER_Q8_1)" if defer else ""))},
                "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "note": e2e_note},
                "gpu_launches": launches_per_step * args.steps,
                "collectives_per_step": 1 if world > 1 else 0,
                "roofline": {"bound": "hbm",
                             "kernel": ("cfi_mmvq_stream_q81<Q4_K,1> (quantize_q8_1 + mul_mat_vec_q) 8192x2048"
                                        if fused_step else "cfi_mmvq_stream<Q4_K,1> (mul_mat_vec_q) 8192x2048"),
                             "achieved": round(achieved, 1),
                             "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                             "traffic": traffic_per_launch(fused_step), "launch_us": round(kms * 1e3, 3),
                             "bytes_per_launch": kbytes},
                "clocks": clk.summary(), "native_only": ok}
        line.update(legs)
        if not args.no_prefill and world == 1:
            line["prefill"] = prefill_gemm(cfi, g, stream, dev, tensor_peak())
        if not args.no_decode and world == 1:
            line["decode"] = decode_bench(stream, dev)
            line["decode"]["const_weights"] = decode_bench(stream, dev, const_weights=True)
            line["decode"]["deferred_quantize"] = decode_bench(stream, dev, defer=True, const_weights=True)
            line["decode"]["fused"] = decode_bench(stream, dev, fused=1, const_weights=True)
        if not args.no_configs and world == 1:
            line["config1"] = config1_bench(cfi, g_sep or g, stream, dev, peak, gf=g if defer else None)
            line["config5"] = config5_bench(cfi, g, stream, dev, peak, tensor_peak())
            line["fattn"] = fattn_bench(cfi, g, stream, dev, tensor_peak())
        if not args.no_cpu and world == 1:
            gbs, used, n, el = cpu_baseline(args.cpu_seconds)
            gbs1, _, n1, el1 = cpu_baseline(max(1.0, args.cpu_seconds / 2), threads=1)
            line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": used, "kind": "port",
                                    "sample": "%d full steps (4 batches each) in %.1f s, rows split over %d threads"
                                              % (n, el, used),
                                    "single_thread": {"value": round(gbs1, 3), "unit": "GB/s", "cores": 1,
                                                      "sample": "%d full steps in %.1f s" % (n1, el1)}}
        print(json.dumps(line), flush=True)
    del graph_period, graph_rest, ge
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    for c in (ctx_sep, ctx_plain):
        if c:
            c.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the config 1 and config 5 legs")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--separate-quantize", action="store_true",
                    help="launch quantize_q8_1 and mul_mat_vec_q separately (no CFI_CTX_DEFER_Q8_1)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_gpu(args, rank, world)


if __name__ == "__main__":
    main()
