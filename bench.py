"""Benchmark of the substitution hot path on B200 (one JSON line on rank 0).

Workload: quantize_q8_1 of fp32 activations + Q4_K mul_mat_vec_q over an
8192 x 2048 Q4_K weight matrix at batch 1, 2, 4 and 8 columns.  One step = the four
(quantize, GEMV) pairs.  Metric: GB/s of algorithmic bytes (weights + q8_1 activations + fp32
outputs + quantizer traffic) against the measured HBM peak.  Weights rotate over enough copies
that every GEMV reads from HBM (inputs larger than L2).  Kernels are launched through the
substitution C ABI (cfi_subst_launch with ggml kernelParams); the timed region replays one CUDA
graph of exactly --steps steps, replayed once before timing.  With --gpus N (torchrun) every rank
owns an 8192-row shard of an (8192 N) x 2048 matrix (weak scaling) and the outputs are
all-gathered each step (step i gathers step i-1's outputs on a second stream while its own
kernels run, all inside the graph) by cfi_peer_all_gather (a few CTAs storing each rank's slice
into every rank's IPC-mapped buffer over NVLink, bounded signal and wait), or over NCCL with
--exchange nccl.  Every N also runs config 5's batch-64 decode step with
the rows of every matrix split over the ranks and an all-gather of every product's outputs.

Further legs (1 GPU): per-batch GEMV kernel times, large GEMV shapes (65536 x 2048 Q4_K, the
151936 x 896 Q8_0 lm_head), the row kernels (rms_norm, rope_neox, soft_max, quantize_q8_1),
config 1, config 3 (prefill mul_mat_q and GemmEx), config 4 decode, config 5 prefill, the prefill
FlashAttention and the CPU baseline.  --legs selects them.

--impl reference times the CPU evaluation of the same step (the oracle port of the reference's
host math, built -O3 -march=native on the host, row-parallel over every host core) on rank 0.
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
ALL_LEGS = ("gemv", "rowops", "prefill", "decode", "config1", "config5", "fattn", "cpu")


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


def graph_time_us(stream, body, reps=5, calls=1):
    """Capture `calls` x body(i, stream_handle) in one CUDA graph; mean device time per body call
    (µs) over `reps` replays after one warm replay, CUDA events on the launching stream."""
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


def rotated(torch, dev, host_bytes, min_total):
    """Copies of one weight matrix on the device, enough that they exceed `min_total` bytes."""
    n = max(2, int(np.ceil(min_total / host_bytes.size)))
    wd = torch.empty((n, host_bytes.size), dtype=torch.uint8, device=dev)
    wd[0].copy_(torch.from_numpy(np.ascontiguousarray(host_bytes).ravel()))
    for i in range(1, n):
        wd[i].copy_(wd[0])
    return wd


def prefill_gemm(cfi, g, stream, dev, peak_tf):
    """Q8_0 weights (4864x896 and 896x4864) x 631 tokens quantised to
    q8_1_mmq, through the native mul_mat_q (tcgen05), plus the reference's own mmq throughput shape
    4096x4096x512 (Q8_0 and Q4_K) and the cuBLAS-compatible GemmEx path on config 3's shapes.
    CUDA graph of back-to-back calls.  Flat keys: <type>_<rows>x<k>x<cols>_us / _tflops."""
    import torch

    out = {}
    for ty, m, k, n in ((cfi.Q8_0, 4864, 896, 631), (cfi.Q8_0, 896, 4864, 631), (cfi.Q8_0, 4096, 4096, 512),
                        (cfi.Q4_K, 4096, 4096, 512)):
        w = torch.from_numpy(cfi.synthetic_weights(ty, m, k, seed=m).ravel()).to(dev)
        xf = torch.from_numpy(np.random.default_rng(k).normal(size=(n, k)).astype(np.float32)).to(dev)
        q = torch.zeros(k // 128 * n * 144, dtype=torch.uint8, device=dev)
        d = torch.zeros(n * m, dtype=torch.float32, device=dev)
        ds4 = 1 if ty == cfi.Q4_K else 0
        torch.cuda.synchronize()  # inputs written on torch's stream, used on `stream`
        with torch.cuda.stream(stream):
            g.quantize_mmq(ds4, xf.data_ptr(), q.data_ptr(), k, k, n, stream=stream.cuda_stream)
            g.mmq(ty, w.data_ptr(), q.data_ptr(), d.data_ptr(), k, m, n, stream=stream.cuda_stream)
        torch.cuda.synchronize()
        us = graph_time_us(stream, lambda i, st: g.mmq(ty, w.data_ptr(), q.data_ptr(), d.data_ptr(), k, m, n,
                                                        stream=st), reps=5, calls=20)
        tag = "%s_%dx%dx%d" % ("q8_0" if ty == cfi.Q8_0 else "q4_k", m, k, n)
        out[tag + "_us"] = round(us, 2)
        out[tag + "_tflops"] = round(2.0 * m * n * k / us / 1e6, 1)
    # the cuBLAS-compatible GemmEx path on the same shapes (ggml's T,N f16 -> f32 call)
    blas = cfi.Blas(stream.cuda_stream)
    for m, k in ((4864, 896), (896, 4864)):
        n = 631
        A = torch.randn(m, k, device=dev).half()
        B = torch.randn(n, k, device=dev).half()
        Cm = torch.zeros(n, m, device=dev)
        torch.cuda.synchronize()

        def call(i, st):
            blas.set_stream(st)
            blas.gemm_ex(1, 0, m, n, k, 1.0, A.data_ptr(), 2, k, B.data_ptr(), 2, k, 0.0, Cm.data_ptr(), 0, m)
        with torch.cuda.stream(stream):
            call(0, stream.cuda_stream)
        torch.cuda.synchronize()
        us = graph_time_us(stream, call, reps=5, calls=20)
        tag = "gemm_ex_f16_%dx%dx%d" % (m, n, k)
        out[tag + "_us"] = round(us, 2)
        out[tag + "_tflops"] = round(2.0 * m * n * k / us / 1e6, 1)
        out[tag + "_path"] = "tcgen05" if blas.last_path() == 1 else "simt"
    blas.close()
    c3 = max(out["q8_0_4864x896x631_tflops"], out["q8_0_896x4864x631_tflops"])
    return {"workload": "config3: Q8_0 W x 631 q8_1_mmq tokens -> f32 (mul_mat_q on tcgen05, incl. activation "
                        "pre-pass); also 4096x4096x512",
            "config3_best_tflops": c3, "config3_frac": round(c3 / peak_tf, 4),
            "peak_tflops": peak_tf, "peak_kind": "measured bf16 dense (burst)", **out}


GEMV_SHAPES = ((12, ROWS, K, BATCHES, "q4k_8192x2048"), (12, 65536, 2048, (1, 8), "q4k_65536x2048"),
               (8, 151936, 896, (1,), "q8_0_151936x896"))


def gemv_legs(cfi, g, stream, dev, peak, shapes=GEMV_SHAPES):
    """Q4_K mul_mat_vec_q 8192x2048 at batch 1/2/4/8 on their own, and the large shapes (65536 x
    2048 Q4_K at batch 1 and 8, the 151936 x 896 Q8_0 lm_head at batch 1): graphs of back-to-back
    launches over rotated weight copies (> 3x L2), on a context that fetches weights before the
    dependent-launch wait.  µs per launch and the fraction of HBM of the algorithmic bytes."""
    import torch

    out = {}
    for ty, rows, k, batches, tag in shapes:
        w = cfi.synthetic_weights(ty, rows, k, seed=rows)
        wd = rotated(torch, dev, w, 3 * L2_BYTES)
        ncopy = wd.shape[0]
        for b in batches:
            x = torch.from_numpy(np.random.default_rng(b).normal(size=(b, k)).astype(np.float32)).to(dev)
            q = torch.zeros(b * k // 32 * 36, dtype=torch.uint8, device=dev)
            y = torch.zeros(b * rows, dtype=torch.float32, device=dev)
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                g.quantize_q8_1(x.data_ptr(), q.data_ptr(), k, k, b, stream=stream.cuda_stream)
                g.mmvq(ty, b, wd[0].data_ptr(), q.data_ptr(), y.data_ptr(), k, rows, stream=stream.cuda_stream)
            torch.cuda.synchronize()
            calls = max(ncopy, 8)
            us = graph_time_us(stream, lambda i, st: g.mmvq(ty, b, wd[i % ncopy].data_ptr(), q.data_ptr(), y.data_ptr(),
                                                            k, rows, stream=st), reps=5, calls=calls)
            byts = w.size + b * (k // 32 * 36 + rows * 4)
            out["%s_b%d_us" % (tag, b)] = round(us, 3)
            out["%s_b%d_frac" % (tag, b)] = round(byts / us / 1e3 / peak, 4)
        del wd
    return out


def rowops_bench(cfi, g, stream, dev, peak, big_only=False):
    """The row kernels at the decode shapes of configs 4/5 (µs per launch: one row or one token, the
    reference's profiled launches) and at a batched shape that streams from HBM (GB/s of
    read + write bytes, inputs rotated over > 2x L2): rms_norm_f32 with the weight multiply (rows of
    896 and 1536), rope_neox (14 heads x 64 and 12 heads x 128, theta 1e6), soft_max_f32 (rows of
    632 keys with an f32 mask, 14 heads), quantize_q8_1 (896 / 1536 values)."""
    import torch

    out = {}

    def timed(fn, nbuf):
        torch.cuda.synchronize()  # inputs written on torch's stream, used on `stream`
        with torch.cuda.stream(stream):
            fn(0, stream.cuda_stream)
        torch.cuda.synchronize()
        return graph_time_us(stream, lambda i, st: fn(i % nbuf, st), reps=5, calls=max(nbuf, 32))

    for ncols in (896, 1536):
        wv = torch.randn(ncols, device=dev)
        for nrows, tag in ((1, "dec"), (16384, "big"))[1 if big_only else 0:]:
            nbuf = 1 if nrows == 1 else max(2, int(np.ceil(2 * L2_BYTES / (nrows * ncols * 8))))
            xs = torch.randn(nbuf, nrows * ncols, device=dev)
            ys = torch.zeros_like(xs)
            us = timed(lambda i, st: g.rms_norm(xs[i].data_ptr(), ys[i].data_ptr(), ncols, nrows, mul=wv.data_ptr(),
                                                stream=st), nbuf)
            out["rms_norm_%d_%s_us" % (ncols, tag)] = round(us, 3)
            if nrows > 1:
                byts = nrows * ncols * 8 + ncols * 4
                out["rms_norm_%d_big_gbs" % ncols] = round(byts / us / 1e3, 1)
                out["rms_norm_%d_big_frac" % ncols] = round(byts / us / 1e3 / peak, 4)
    for nh, hd in ((14, 64), (12, 128)):
        for ntok, tag in ((1, "dec"), (4096, "big"))[1 if big_only else 0:]:
            n = nh * hd * ntok
            nbuf = 1 if ntok == 1 else max(2, int(np.ceil(2 * L2_BYTES / (n * 8))))
            xs = torch.randn(nbuf, n, device=dev)
            ys = torch.zeros_like(xs)
            pos = torch.arange(ntok, dtype=torch.int32, device=dev) + 631
            us = timed(lambda i, st: g.rope_neox(xs[i].data_ptr(), ys[i].data_ptr(), hd, nh, ntok, hd, pos.data_ptr(),
                                                 stream=st), nbuf)
            out["rope_%dx%d_%s_us" % (nh, hd, tag)] = round(us, 3)
            if ntok > 1:
                byts = n * 8 + ntok * 4
                out["rope_%dx%d_big_gbs" % (nh, hd)] = round(byts / us / 1e3, 1)
                out["rope_%dx%d_big_frac" % (nh, hd)] = round(byts / us / 1e3 / peak, 4)
    ncols, nh = 632, 14
    for ne01, tag in ((1, "dec"), (631 * 8, "big"))[1 if big_only else 0:]:
        nbuf = 1 if ne01 == 1 else max(2, int(np.ceil(2 * L2_BYTES / (ne01 * nh * ncols * 8))))
        xs = torch.randn(nbuf, ne01 * nh * ncols, device=dev)
        ys = torch.zeros_like(xs)
        mask = torch.zeros(ne01 * ncols, device=dev)
        us = timed(lambda i, st: g.soft_max(xs[i].data_ptr(), mask.data_ptr(), ys[i].data_ptr(), ncols, ne01, nh, 0.125,
                                            stream=st), nbuf)
        out["soft_max_%s_us" % tag] = round(us, 3)
        if ne01 > 1:
            byts = ne01 * nh * ncols * 8 + ne01 * ncols * 4
            out["soft_max_big_gbs"] = round(byts / us / 1e3, 1)
            out["soft_max_big_frac"] = round(byts / us / 1e3 / peak, 4)
    for k in (896, 1536):
        for ncol, tag in ((1, "dec"), (16384, "big"))[1 if big_only else 0:]:
            nbuf = 1 if ncol == 1 else max(2, int(np.ceil(2 * L2_BYTES / (ncol * k * 5))))
            xs = torch.randn(nbuf, ncol * k, device=dev)
            qs = torch.zeros(nbuf, ncol * k // 32 * 36, dtype=torch.uint8, device=dev)
            us = timed(lambda i, st: g.quantize_q8_1(xs[i].data_ptr(), qs[i].data_ptr(), k, k, ncol, stream=st), nbuf)
            out["quantize_q8_1_%d_%s_us" % (k, tag)] = round(us, 3)
            if ncol > 1:
                byts = ncol * k * 4 + ncol * k // 32 * 36
                out["quantize_q8_1_%d_big_gbs" % k] = round(byts / us / 1e3, 1)
                out["quantize_q8_1_%d_big_frac" % k] = round(byts / us / 1e3 / peak, 4)
    return out


def config1_bench(cfi, g, stream, dev, peak, gf=None):
    """Q8_0 mul_mat_vec_q 4864x896 on its own (batch 1), and with its
    quantize_q8_1 in front, back to back over rotated weight copies (> 3x L2)."""
    import torch

    rows, k = 4864, 896
    wb = rows * k // 32 * 34
    wd = rotated(torch, dev, cfi.synthetic_weights(cfi.Q8_0, rows, k, seed=11), 3 * L2_BYTES)
    ncopy = wd.shape[0]
    x = torch.from_numpy(np.random.default_rng(3).normal(size=k).astype(np.float32)).to(dev)
    q = torch.zeros(k // 32 * 36, dtype=torch.uint8, device=dev)
    y = torch.zeros(rows, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
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


C5_H, C5_F, C5_KV, C5_L, C5_V = 1536, 8960, 256, 28, 151936
C5_SHAPES = {"q": (C5_H, C5_H), "k": (C5_KV, C5_H), "v": (C5_KV, C5_H), "o": (C5_H, C5_H), "g": (C5_F, C5_H),
             "u": (C5_F, C5_H), "d": (C5_H, C5_F)}
# products grouped by the activation they read, in model order: each group's input depends on the
# previous group's outputs (attention input -> q, k, v; attention output -> o; FFN input -> gate,
# up; FFN hidden -> down; the next layer's attention input)
C5_GROUPS = ((("q", "k", "v"), C5_H), (("o",), C5_H), (("g", "u"), C5_H), (("d",), C5_F))


def config5_prefill(cfi, g, stream, dev, peak_tf):
    """BASELINE config 5 prefill: Qwen2.5-1.5B-architecture weight products, 28 layers of Q4_K
    matrices (q, o 1536x1536; k, v 256x1536; gate, up 8960x1536; down 1536x8960) and the Q8_0 head
    151936x1536, over a 631-token prompt: per layer the activations quantised to q8_1_mmq once per
    distinct input and the seven mul_mat_q products; the head on the last token only
    (quantize_q8_1 + mul_mat_vec_q), as ggml does.  Attention and the element-wise ops are not in
    this leg.  Weights random, device-side (seeded)."""
    import torch

    from decode import random_q4_k, random_q8_0

    H, F, L, V = C5_H, C5_F, C5_L, C5_V
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    layers = [{nm: random_q4_k(torch, r, c, gen, dev) for nm, (r, c) in C5_SHAPES.items()} for _ in range(L)]
    head = random_q8_0(torch, V, H, gen, dev)
    params = L * sum(r * c for r, c in C5_SHAPES.values())
    n = 631
    xf = {kk: torch.randn(n * kk, generator=gen, device=dev) for kk in (H, F)}
    xq = {kk: torch.zeros(kk // 128 * n * 144, dtype=torch.uint8, device=dev) for kk in (H, F)}
    out = {nm: torch.zeros(n * r, dtype=torch.float32, device=dev) for nm, (r, c) in C5_SHAPES.items()}
    hq = torch.zeros(H // 32 * 36, dtype=torch.uint8, device=dev)
    logits = torch.zeros(V, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()

    def prefill(i, st):
        for lay in layers:
            for inputs, k in C5_GROUPS:
                g.quantize_mmq(1, xf[k].data_ptr(), xq[k].data_ptr(), k, k, n, stream=st)
                for nm in inputs:
                    g.mmq(cfi.Q4_K, lay[nm].data_ptr(), xq[k].data_ptr(), out[nm].data_ptr(), k, C5_SHAPES[nm][0], n,
                          stream=st)
        g.quantize_q8_1(xf[H].data_ptr() + (n - 1) * H * 4, hq.data_ptr(), H, H, 1, stream=st)
        g.mmvq(cfi.Q8_0, 1, head.data_ptr(), hq.data_ptr(), logits.data_ptr(), H, V, stream=st)
    with torch.cuda.stream(stream):
        prefill(0, stream.cuda_stream)
    torch.cuda.synchronize()
    us = graph_time_us(stream, prefill, reps=3)
    ops = 2.0 * params * n + 2.0 * V * H
    del layers, head
    return {"ms": round(us / 1e3, 3), "tok_per_s": round(631 / (us * 1e-6), 1), "tflops": round(ops / us / 1e6, 1),
            "frac": round(ops / us / 1e6 / peak_tf, 4), "launches": L * (4 + 7) + 2}


def config5_b64(cfi, g, stream, dev, peak_gbs, world, rank, dist, comm):
    """BASELINE config 5 decode: one batch-64 step (64 independent sequences) over the 28 Q4_K
    layers and the Q8_0 head, the rows of every matrix split over the `world` ranks
    (shard.row_split, weak in memory, strong in work).  Per product: quantize_q8_1_mmq of its input
    (once per group), the native mul_mat_q on the rank's rows, and with N > 1 one NCCL all-gather
    per group of products that share an input (their 64-column outputs back to back) on a comm
    stream, followed by cfi_glue_gather_row_shards of each product into ggml's column-major dst.  A group's quantize waits for the previous group's gathers (its input is
    computed from them in a real model), so collective latency is exposed as it would be.
    Reported: the step time, the same step without collectives (kernels only), the collectives
    alone, the step with the products of a group as parallel graph branches (side streams), and a
    check of rank 0's gathered logits against the unsharded head product on rank 0.  With N > 1
    also `peer_ms`: the all-gather fused into the products over NVLink peer memory (each group in
    one cfi_mmq_skinny_group_peers launch that stores every rank's rows into every rank's
    gathered dst and ends once the peers' rows are in; cfi_peer.h), its logits checked against
    the NCCL path's."""
    import torch

    import shard
    from decode import random_q4_k, random_q8_0

    H, F, L, V, n = C5_H, C5_F, C5_L, C5_V, 64
    L_ = cfi.lib()
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)

    def rows_of(full, rows, sh):
        return full.view(rows, -1)[sh.row0:sh.row0 + sh.rows].contiguous().view(-1)

    sh = {nm: shard.row_split(r, world, rank) for nm, (r, c) in C5_SHAPES.items()}
    sh["head"] = shard.row_split(V, world, rank)
    layers = []
    for _ in range(L):
        lay = {}
        for nm, (r, c) in C5_SHAPES.items():
            lay[nm] = rows_of(random_q4_k(torch, r, c, gen, dev), r, sh[nm])  # the same draws on every rank
        layers.append(lay)
    head_full = random_q8_0(torch, V, H, gen, dev)
    head = rows_of(head_full, V, sh["head"])
    if rank != 0:
        del head_full
        head_full = None
    wbytes = L * sum(r * c // 256 * 144 for r, c in C5_SHAPES.values()) + V * H // 32 * 34
    xf = {kk: torch.randn(n * kk, generator=gen, device=dev) for kk in (H, F)}
    xq = {kk: torch.zeros(kk // 128 * n * 144, dtype=torch.uint8, device=dev) for kk in (H, F)}
    hq = torch.zeros(H // 128 * n * 144, dtype=torch.uint8, device=dev)
    names = list(C5_SHAPES) + ["head"]
    nrows = {**{nm: r for nm, (r, c) in C5_SHAPES.items()}, "head": V}
    # the outputs of the products that share an input are back to back in one buffer per group, so
    # one all-gather per group carries them (each rank's slices of a group contiguous)
    groups = [inputs for inputs, _ in C5_GROUPS] + [("head",)]
    gsize, goff = {}, {}
    for grp in groups:
        o = 0
        for nm in grp:
            goff[nm] = o
            o += n * sh[nm].rows_padded
        gsize[grp] = o
    gbuf = {grp: torch.zeros(gsize[grp], dtype=torch.float32, device=dev) for grp in groups}
    out = {nm: gbuf[grp][goff[nm]:goff[nm] + n * sh[nm].rows_padded] for grp in groups for nm in grp}
    gath = {grp: torch.zeros(world * gsize[grp], dtype=torch.float32, device=dev) for grp in groups} \
        if world > 1 else None
    full = {nm: torch.zeros(n * nrows[nm], dtype=torch.float32, device=dev) for nm in names} if world > 1 else None

    def gathers(cur, grp):
        """all-gather of one group's outputs + assembly of each product into ggml's layout, on the
        comm stream after `cur`'s work so far; returns the event that marks their completion."""
        ev = torch.cuda.Event()
        ev.record(cur)
        comm.wait_event(ev)
        with torch.cuda.stream(comm):
            dist.all_gather_into_tensor(gath[grp], gbuf[grp])
            for nm in grp:
                rc = L_.cfi_glue_gather_row_shards(gath[grp].data_ptr() + 4 * goff[nm], full[nm].data_ptr(), nrows[nm],
                                                   n, world, gsize[grp], comm.cuda_stream)
                assert rc == 0, rc
        done = torch.cuda.Event()
        done.record(comm)
        return done

    side = [torch.cuda.Stream(device=dev) for _ in range(2)]
    # the all-gather over NVLink peer memory: every product's gathered ggml dst (n x nrows) in
    # one peer buffer per rank, mapped into every rank (cfi_peer.h)
    pg, poff = None, {}
    if world > 1:
        o = 0
        for nm in names:
            poff[nm] = o
            o += (n * nrows[nm] * 4 + 255) // 256 * 256

        def exchange(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got

        pg = cfi.PeerGroup(rank, world, o, exchange)

    def peer_step():
        """Each group of products in one skinny launch that stores every rank's rows into every
        rank's gathered output (peer stores over NVLink) and ends once the peers' rows have
        arrived (its last CTA's bounded wait for their signals): no collective, no assembly
        kernel, no extra launch."""
        st = torch.cuda.current_stream().cuda_stream
        for lay in layers:
            for inputs, k in C5_GROUPS:
                g.quantize_mmq(1, xf[k].data_ptr(), xq[k].data_ptr(), k, k, n, stream=st)
                cfi.mmq_skinny_group_peers(cfi.Q4_K, [lay[nm].data_ptr() for nm in inputs], xq[k].data_ptr(),
                                           [pg.data + poff[nm] + 4 * sh[nm].row0 for nm in inputs],
                                           [sh[nm].rows for nm in inputs], k, n, pg,
                                           stride_col_dst=[nrows[nm] for nm in inputs], stream=st)
        g.quantize_mmq(0, xf[H].data_ptr(), hq.data_ptr(), H, H, n, stream=st)
        cfi.mmq_skinny_group_peers(cfi.Q8_0, [head.data_ptr()], hq.data_ptr(), [pg.data + poff["head"] + 4 * sh["head"].row0],
                                   [sh["head"].rows], H, n, pg, stride_col_dst=[V], stream=st)

    def step(kernels=True, collectives=True, parallel=False, grouped=False, peer=False):
        if peer:
            return peer_step()
        """parallel: the products of a group after the first run on side streams, as parallel
        branches (each product depends only on the group's quantized input); every stream has
        its own split-K workspace and scratch.  grouped: the products of a group in one launch
        (cfi_mmq_skinny_group) instead of one mul_mat_q each."""
        cur = torch.cuda.current_stream()
        st = cur.cuda_stream
        coll = collectives and world > 1
        prev = None
        if coll:
            fork = torch.cuda.Event()
            fork.record(cur)
            comm.wait_event(fork)
        for lay in layers:
            for inputs, k in C5_GROUPS:
                if kernels:
                    if prev is not None:
                        cur.wait_event(prev)
                    g.quantize_mmq(1, xf[k].data_ptr(), xq[k].data_ptr(), k, k, n, stream=st)
                    branches = []
                    if parallel and len(inputs) > 1:
                        ev = torch.cuda.Event()
                        ev.record(cur)
                        for sd in side[:len(inputs) - 1]:
                            sd.wait_event(ev)
                    if grouped and len(inputs) > 1:
                        cfi.mmq_skinny_group(cfi.Q4_K, [lay[nm].data_ptr() for nm in inputs], xq[k].data_ptr(),
                                             [out[nm].data_ptr() for nm in inputs], [sh[nm].rows for nm in inputs], k, n,
                                             stride_col_dst=[sh[nm].rows_padded for nm in inputs], stream=st)
                    for i, nm in enumerate(inputs):
                        if grouped and len(inputs) > 1:
                            break
                        on = side[i - 1] if parallel and i > 0 else cur
                        g.mmq(cfi.Q4_K, lay[nm].data_ptr(), xq[k].data_ptr(), out[nm].data_ptr(), k, sh[nm].rows, n,
                              stream=on.cuda_stream, stride_col_dst=sh[nm].rows_padded)
                        if on is not cur:
                            done = torch.cuda.Event()
                            done.record(on)
                            branches.append(done)
                    for done in branches:
                        cur.wait_event(done)
                if coll:
                    prev = gathers(cur, tuple(inputs))
        if kernels:
            if prev is not None:
                cur.wait_event(prev)
            g.quantize_mmq(0, xf[H].data_ptr(), hq.data_ptr(), H, H, n, stream=st)
            g.mmq(cfi.Q8_0, head.data_ptr(), hq.data_ptr(), out["head"].data_ptr(), H, sh["head"].rows, n, stream=st,
                  stride_col_dst=sh["head"].rows_padded)
        if coll:
            prev = gathers(cur, ("head",))
            cur.wait_event(prev)

    def timed(**kw):
        torch.cuda.synchronize()  # inputs written on torch's stream, used on `stream`
        with torch.cuda.stream(stream):
            step(**kw)  # first use (probes) outside the capture
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            step(**kw)
        with torch.cuda.stream(stream):
            gr.replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        reps = 5
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                gr.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        if dist:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        del gr
        return ms

    ms_step = timed()
    ms_kern = timed(collectives=False) if world > 1 else ms_step
    ms_coll = timed(kernels=False) if world > 1 else 0.0
    ms_par = timed(parallel=True)
    ms_grp = timed(grouped=True)
    ms_peer = timed(peer=True) if world > 1 else None
    # check: rank 0's gathered logits (the NCCL path's, and the peer path's) against the
    # unsharded head product on rank 0
    check = {}
    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    peer_head = None
    if world > 1:
        with torch.cuda.stream(stream):
            step(peer=True)
        torch.cuda.synchronize()
        if rank == 0:
            peer_head = torch.empty(n * V, dtype=torch.float32, device=dev)
            rc = L_.cfi_glue_gather_row_shards(pg.data + poff["head"], peer_head.data_ptr(), V, n, 1, 0,
                                               torch.cuda.current_stream().cuda_stream)  # one rank's "gather": a copy
            assert rc == 0, rc
            torch.cuda.synchronize()
    if rank == 0:
        got = (full["head"] if world > 1 else out["head"]).view(n, V)
        ref = torch.zeros(n * V, dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            g.quantize_mmq(0, xf[H].data_ptr(), hq.data_ptr(), H, H, n, stream=stream.cuda_stream)
            g.mmq(cfi.Q8_0, head_full.data_ptr(), hq.data_ptr(), ref.data_ptr(), H, V, n, stream=stream.cuda_stream)
        torch.cuda.synchronize()
        ref = ref.view(n, V)
        diff = (got.double() - ref.double()).norm() / ref.double().norm()
        check = {"logits_bitwise_equal": bool(torch.equal(got, ref)), "logits_rel_l2": float(diff),
                 "logits_nonfinite": int((~torch.isfinite(got)).sum()), "ref_nonfinite": int((~torch.isfinite(ref)).sum())}
        if peer_head is not None:
            ph = peer_head.view(n, V)
            check["peer_logits_equal_nccl_path"] = bool(torch.equal(ph, got))
            check["peer_logits_rel_l2"] = float((ph.double() - ref.double()).norm() / ref.double().norm())
            check["peer_logits_nonfinite"] = int((~torch.isfinite(ph)).sum())
    err = int(L_.cfi_device_error())
    if dist:
        dist.barrier()
    if pg is not None:
        pg.close()
    launches = L * (4 + 7) + 2 + (L * 7 + 1 if world > 1 else 0)  # + one assembly per product
    res = {"ms": round(ms_step, 4), "tok_per_s": round(64 / (ms_step * 1e-3), 1),
           "weights_gbs": round(wbytes / ms_step / 1e6, 1),
           "frac": round(wbytes / ms_step / 1e6 / (peak_gbs * world), 4),
           "parallel_products_ms": round(ms_par, 4),
           "parallel_products_frac": round(wbytes / ms_par / 1e6 / (peak_gbs * world), 4),
           "grouped_products_ms": round(ms_grp, 4),
           "grouped_products_frac": round(wbytes / ms_grp / 1e6 / (peak_gbs * world), 4),
           "grouped_launches": launches - L * sum(len(i) - 1 for i, _ in C5_GROUPS),
           "kernels_only_ms": round(ms_kern, 4), "collectives_only_ms": round(ms_coll, 4),
           "all_gathers_per_step": (L * len(C5_GROUPS) + 1) if world > 1 else 0,
           "gathered_bytes_per_gpu": (world - 1) * n * 4 * (L * sum(sh[nm].rows_padded for nm in C5_SHAPES) +
                                                            sh["head"].rows_padded),
           "launches": launches, "gpus": world, "device_error": err, **check}
    if ms_peer is not None:
        res.update({"peer_ms": round(ms_peer, 4), "peer_tok_per_s": round(64 / (ms_peer * 1e-3), 1),
                    "peer_frac": round(wbytes / ms_peer / 1e6 / (peak_gbs * world), 4),
                    "peer_launches": 2 * (L * len(C5_GROUPS) + 1)})
    del layers, head, head_full, out, gbuf, gath, full
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
        torch.cuda.synchronize()
        call = lambda n, st: g.fattn(d, q.data_ptr(), k.data_ptr(), v.data_ptr(), mask.data_ptr(), dst.data_ptr(), nq,
                                     nh, nhk, nkv, 1, 1.0 / d ** 0.5, stream=st)
        with torch.cuda.stream(stream):
            call(0, stream.cuda_stream)
        torch.cuda.synchronize()
        us = graph_time_us(stream, call, reps=5, calls=20)
        fl = 4.0 * nq * nkv * d * nh
        out["d%d_h%d_us" % (d, nh)] = round(us, 2)
        out["d%d_h%d_tflops" % (d, nh)] = round(fl / us / 1e6, 1)
        out["d%d_h%d_frac" % (d, nh)] = round(fl / us / 1e6 / peak_tf, 4)
    return {"workload": "flash_attn_ext_f16, 631 queries x 640 keys, causal mask (configs 4 / 5 prefill attention)",
            **out}


def decode_bench(stream, dev, ntok=48, warm=3, fused=False, defer=False, const_weights=False):
    """Qwen2.5-0.5B-architecture decode (24 layers, Q8_0 random weights, 631-token
    seeded KV cache), one CUDA graph per token step replayed for `ntok` greedy tokens.  fused: the
    stacked-weight step with the fused glue kernels (9 launches per layer instead of 25); fused=3: that
    step as one persistent cooperative launch (cfi_decode_step_q8_0).  defer:
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
    out = {"tok_per_s": round(ntok / (ms * 1e-3), 1), "ms_per_token": round(ms / ntok, 4),
           "launches_per_token": m.launches_per_step - (fused_in_capture if defer else 0),
           "weights_gbs": round(bpt * ntok / (ms * 1e-3) / 1e9, 1)}
    del gr
    ctx.close()
    return out


def cpu_baseline(seconds, threads=0):
    """The oracle's CPU decode step (reference host math, row-parallel) on a bounded sample, from
    the copy of the oracle built -O3 -march=native on this host."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import cfi_b200 as cfi
    import oracle_py as O

    if O._o is None:
        O.use_native_build()
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
                             "sample": "%d full steps in %.1f s (oracle built -O3 -march=native)" % (n, el)},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_gpu(args, rank, world):
    import torch

    import cfi_b200 as cfi

    legs_on = set(ALL_LEGS if args.legs == "all" else [x for x in args.legs.split(",") if x])
    for flag, leg in (("no_cpu", "cpu"), ("no_prefill", "prefill"), ("no_decode", "decode")):
        if getattr(args, flag):
            legs_on.discard(leg)
    if args.no_configs:
        legs_on -= {"config1", "config5", "fattn"}
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
    wd = rotated(torch, dev, w, ncopy * W_BYTES)
    ncopy = wd.shape[0]
    xs_host = {b: torch.from_numpy(np.random.default_rng(b).normal(size=(b, K)).astype(np.float32)).pin_memory()
               for b in BATCHES}
    xs = {b: xs_host[b].to(dev) for b in BATCHES}
    qs = {b: torch.zeros(Q81(b), dtype=torch.uint8, device=dev) for b in BATCHES}
    # two output sets: with N > 1 step i all-gathers step i-1's outputs while it computes its own
    y_sets = [torch.zeros(sum(b for b in BATCHES) * ROWS, dtype=torch.float32, device=dev) for _ in range(2)]
    y_all = y_sets[0]
    offs, o = {}, 0
    for b in BATCHES:
        offs[b] = o
        o += b * ROWS
    y_views_p = [{b: ya[offs[b]:offs[b] + b * ROWS] for b in BATCHES} for ya in y_sets]
    y_views = y_views_p[0]
    gathered_sets = [torch.zeros(world * y_all.numel(), dtype=torch.float32, device=dev) for _ in range(2)] \
        if world > 1 and args.exchange == "nccl" else None
    comm = torch.cuda.Stream(device=dev) if world > 1 else None
    # the peer exchange: one gathered range per output set (world slices of y_all each) in a
    # buffer every rank maps (cfi_peer.h)
    ybytes = y_all.numel() * 4
    pgx = None
    if world > 1 and args.exchange == "peer":
        def exchange_obj(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got
        pgx = cfi.PeerGroup(rank, world, 2 * world * ybytes, exchange_obj)

    def all_gather(ysrc, parity, st):
        """step outputs ysrc (output set `parity`) gathered over the ranks on stream st"""
        if pgx is not None:
            pgx.all_gather(ysrc.data_ptr(), ybytes, parity * world * ybytes, stream=st.cuda_stream)
        else:
            with torch.cuda.stream(st):
                dist.all_gather_into_tensor(gathered_sets[parity], ysrc)
    torch.cuda.synchronize()  # everything above was written on torch's stream; the steps run on `stream`

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
            all_gather(y_sets[1 - parity], 1 - parity, comm)
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
                all_gather(y_all, 0, stream)
    torch.cuda.synchronize()
    # One CUDA graph holds exactly the K timed steps (step i: weight phase i % nphase, output set
    # i % 2; programmatic dependent launch overlaps consecutive steps inside it).  It is replayed
    # once before the timed replay, so the timed region runs a warmed graph.
    fused_before = ctx.stats()["fused_q8_1"]
    graph_k = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_k, stream=stream):
        for i in range(args.steps):
            step_pipelined(i % nphase, i % 2)
    # GEMVs that absorbed their quantize, per captured step
    launches_per_step = 2 * len(BATCHES) - (ctx.stats()["fused_q8_1"] - fused_before) // args.steps
    fused_step = launches_per_step < 2 * len(BATCHES)
    with torch.cuda.stream(stream):
        graph_k.replay()
    torch.cuda.synchronize()

    # ---- timed region: device time, max over ranks ----
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            e0.record(stream)
            graph_k.replay()
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
    del graph_k

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

    # ---- the same step with its four independent (quantize, GEMV) pairs on four streams as
    # parallel graph branches (1 GPU): the throughput of independent decode batches served together;
    # the headline value above keeps ggml's one-stream order ----
    if g_sep is not None:
        pair_streams = [torch.cuda.Stream(device=dev) for _ in BATCHES]

        def step_concurrent(phase, st):
            cur = torch.cuda.current_stream()
            fork = torch.cuda.Event()
            fork.record(cur)
            joins = []
            for j, b in enumerate(BATCHES):
                ps = pair_streams[j]
                ps.wait_event(fork)
                g_sep.quantize_q8_1(xs[b].data_ptr(), qs[b].data_ptr(), K, K, b, stream=ps.cuda_stream)
                g_sep.mmvq(cfi.Q4_K, b, wd[(phase * len(BATCHES) + j) % ncopy].data_ptr(), qs[b].data_ptr(),
                           y_views[b].data_ptr(), K, ROWS, stream=ps.cuda_stream)
                done = torch.cuda.Event()
                done.record(ps)
                joins.append(done)
            for done in joins:
                cur.wait_event(done)
        with torch.cuda.stream(stream):
            step_concurrent(0, stream.cuda_stream)  # first use on each stream outside the capture
        torch.cuda.synchronize()
        us_c = graph_time_us(stream, lambda i, st: step_concurrent(i % nphase, st), reps=max(3, args.steps // 10),
                             calls=nphase)
        legs["concurrent_streams"] = {"value": round(STEP_BYTES / us_c / 1e3, 2), "ms_per_step": round(us_c * 1e-3, 5),
                                      "launches_per_step": 2 * len(BATCHES),
                                      "router": "the four (quantize_q8_1, mul_mat_vec_q) pairs on four streams (parallel "
                                                "graph branches), CFI_CTX_CONST_WEIGHTS"}

    # ---- dominant kernel: mmvq Q4_K batch 1, back to back (one graph of ncopy launches over the
    # rotated weight copies), CUDA events on the launching stream around the replays ----
    def roof_body(i, st):
        if fused_step:  # the step's kernel: quantize_q8_1 absorbed by the GEMV
            g.quantize_q8_1(xs[1].data_ptr(), qs[1].data_ptr(), K, K, 1, stream=st)
        g.mmvq(cfi.Q4_K, 1, wd[i].data_ptr(), qs[1].data_ptr(), y_views[1].data_ptr(), K, ROWS, stream=st)
        if i == ncopy - 1:
            ctx.flush()
    kms = graph_time_us(stream, roof_body, reps=max(3, args.steps // 10), calls=ncopy) * 1e-3
    peak, peak_kind = peaks()
    kbytes = MMVQ_BYTES(1) + (QUANT_BYTES(1) if fused_step else 0)
    achieved = kbytes / (kms * 1e-3) / 1e9

    # ---- end to end: host activations in, outputs back to the host, every step ----
    h2d = sum(xs_host[b].numel() * 4 for b in BATCHES)
    d2h = y_all.numel() * 4
    # Pipelined as a serving loop would run it: step i's activation copy and output copy run on
    # copy streams (one per direction) while steps i-1 / i+1 compute, with double-buffered device
    # inputs and outputs (parity i % 2) and event edges: H2D(i) after step i-2 has read its input
    # buffer, step i after H2D(i) and after D2H(i-2) has read its output buffer, D2H(i) after step
    # i.  One CUDA graph holds exactly the K steps (replayed once before timing); the timed region
    # ends when the last output is on the host.
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
    torch.cuda.synchronize()
    copy_s = torch.cuda.Stream(device=dev)   # host -> device
    copy_o = torch.cuda.Stream(device=dev)   # device -> host (the other direction's copy engine)
    ev_h2d = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_d2h = [torch.cuda.Event() for _ in range(2)]
    # with N > 1 GPUs: step i's outputs are all-gathered on the comm stream after its kernels;
    # step i+2 waits for that collective before it rewrites the same output buffer
    ev_ag = [torch.cuda.Event() for _ in range(2)]

    ge = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ge, stream=stream):
        cur = torch.cuda.current_stream()
        fork = torch.cuda.Event()
        fork.record(cur)
        copy_s.wait_event(fork)
        copy_o.wait_event(fork)
        if dist:
            comm.wait_event(fork)
        for i in range(args.steps):
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
                all_gather(y_sets[p], p, comm)
                ev_ag[p].record(comm)
            with torch.cuda.stream(copy_o):
                copy_o.wait_event(ev_comp[p])
                y_host[p].copy_(y_sets[p], non_blocking=True)
                ev_d2h[p].record(copy_o)
        for cs in (copy_s, copy_o) + ((comm,) if dist else ()):
            join = torch.cuda.Event()
            join.record(cs)
            cur.wait_event(join)
    with torch.cuda.stream(stream):
        ge.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        ge.replay()
    stream.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_note = ("host fp32 activations in (one pinned buffer) and fp32 outputs out (two pinned buffers) every "
                "step, weights resident; copies on one stream per direction overlap the neighbouring steps' kernels%s; "
                "one CUDA graph of the K steps, replayed once before timing; wall clock until the last output is on "
                "the host" % ((", outputs all-gathered on a third stream (%s)" % ("NCCL" if pgx is None else "cfi_peer_all_gather"))
                              if dist else ""))
    del ge
    if dist:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * STEP_BYTES * args.steps / e2e_s / 1e9

    stats = ctx.stats()
    ok = stats["stock_launches"] == 0 and stats["native_failures"] == 0
    line = {}
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded N(0,0.02) weights quantized to Q4_K, "
                "N(0,1) activations)",
                "config": {"workload": "config2: Q4_K 8192x2048 GEMV + quantize_q8_1, batch 1/2/4/8",
                           "rows_per_gpu": ROWS, "k": K, "batches": "1,2,4,8", "weight_copies": ncopy,
                           "l2": "inputs larger than L2: %d weight copies (%.0f MB) rotated" % (ncopy, ncopy * W_BYTES / 1e6),
                           "parallelism": ("row-sharded x%d + %s all-gather" % (world, "NCCL" if pgx is None else "peer-memory (NVLink)"))
                           if world > 1 else "single GPU",
                           "bytes_per_step_per_gpu": STEP_BYTES,
                           "cuda_graph": "one graph of exactly the K timed steps, replayed once before timing",
                           "router": "CFI_CTX_CONST_WEIGHTS" + (" + CFI_CTX_DEFER_Q8_1" if defer else "")},
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
    summary = {}
    if world == 1:
        if "gemv" in legs_on:
            line["gemv"] = gemv_legs(cfi, g_sep, stream, dev, peak)
            summary.update({k: v for k, v in line["gemv"].items() if k.endswith("_us")})
        if "rowops" in legs_on:
            line["rowops"] = rowops_bench(cfi, g_sep, stream, dev, peak)
        if "prefill" in legs_on:
            line["prefill"] = prefill_gemm(cfi, g, stream, dev, tensor_peak())
            summary["config3_tflops"] = line["prefill"]["config3_best_tflops"]
        if "decode" in legs_on:
            dec = {"workload": "config4: Qwen2.5-0.5B-architecture decode, 24 layers, Q8_0 random weights, 631-token "
                               "seeded KV cache, 48 greedy tokens, one CUDA graph per token"}
            dec["ggml_sequence"] = decode_bench(stream, dev)
            dec["ggml_const_weights"] = decode_bench(stream, dev, const_weights=True)
            dec["ggml_deferred_quantize"] = decode_bench(stream, dev, defer=True, const_weights=True)
            dec["fused"] = decode_bench(stream, dev, fused=1, const_weights=True)
            dec["persistent"] = decode_bench(stream, dev, fused=3)
            line["decode"] = dec
            summary["config4_tok_s"] = dec["fused"]["tok_per_s"]
        if "config1" in legs_on:
            line["config1"] = config1_bench(cfi, g_sep or g, stream, dev, peak, gf=g if defer else None)
        if "fattn" in legs_on:
            line["fattn"] = fattn_bench(cfi, g, stream, dev, tensor_peak())
    if "config5" in legs_on:
        c5 = {"workload": "config5: Qwen2.5-1.5B-architecture weight products (28 layers Q4_K + Q8_0 head, "
                          "984944640 B of weights); attention not included"}
        if world == 1:
            c5["prefill_631"] = config5_prefill(cfi, g, stream, dev, tensor_peak())
            summary["config5_prefill_ms"] = c5["prefill_631"]["ms"]
        c5["decode_b64"] = config5_b64(cfi, g, stream, dev, peak, world, rank, dist, comm)
        summary["config5_b64_ms"] = c5["decode_b64"]["ms"]
        summary["config5_b64_kernels_ms"] = c5["decode_b64"]["kernels_only_ms"]
        summary["config5_b64_parallel_ms"] = c5["decode_b64"]["parallel_products_ms"]
        if "peer_ms" in c5["decode_b64"]:
            summary["config5_b64_peer_ms"] = c5["decode_b64"]["peer_ms"]
        line["config5"] = c5
    if world == 1 and "cpu" in legs_on:
        gbs, used, n, el = cpu_baseline(args.cpu_seconds)
        gbs1, _, n1, el1 = cpu_baseline(max(1.0, args.cpu_seconds / 2), threads=1)
        line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": used, "kind": "port",
                                "sample": "%d full steps (4 batches each) in %.1f s, rows split over %d threads, "
                                          "oracle built -O3 -march=native" % (n, el, used),
                                "single_thread": {"value": round(gbs1, 3), "unit": "GB/s", "cores": 1,
                                                  "sample": "%d full steps in %.1f s" % (n1, el1)}}
    if rank == 0:
        summary.update({"value": line["value"], "e2e": line["e2e"]["value"], "frac": line["roofline"]["frac"]})
        line["summary"] = summary
        print(json.dumps(line), flush=True)
    if dist:
        torch.cuda.synchronize()
        dist.barrier()  # no rank still stores into another's exchange buffer
        if pgx is not None:
            pgx.close()
        dist.destroy_process_group()
    ctx.close()
    for c in (ctx_sep, ctx_plain):
        if c:
            c.close()


def only_gemv(spec):
    """One GEMV shape alone (the gemv leg's timing loop), printed as one JSON line: the profiling
    entry of the kernel summaries."""
    import torch

    import cfi_b200 as cfi

    tname, rows, k, b = spec.split(":")
    ty = {"q4k": cfi.Q4_K, "q8_0": cfi.Q8_0}[tname]
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    ctx = cfi.Ctx(0, const_weights=True)
    g = cfi.GgmlCaller(ctx, "all")
    stream = torch.cuda.Stream(device=dev)
    res = gemv_legs(cfi, g, stream, dev, peaks()[0],
                    shapes=((ty, int(rows), int(k), (int(b),), "%s_%sx%s" % (tname, rows, k)),))
    print(json.dumps({"only_gemv": spec, **res}), flush=True)
    ctx.close()


def only_mmq(spec):
    """One mul_mat_q shape alone (type:rows:k:cols, e.g. q8_0:151936:1536:64 for the batch-64
    head), timed like the prefill leg (graph of back-to-back calls over rotated weight copies) and
    printed as one JSON line: the profiling entry of the mul_mat_q summaries."""
    import torch

    import cfi_b200 as cfi

    tname, rows, k, n = spec.split(":")
    ty = {"q4k": cfi.Q4_K, "q8_0": cfi.Q8_0}[tname]
    rows, k, n = int(rows), int(k), int(n)
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    ctx = cfi.Ctx(0)
    g = cfi.GgmlCaller(ctx, "all")
    stream = torch.cuda.Stream(device=dev)
    w = cfi.synthetic_weights(ty, rows, k, seed=rows)
    wd = rotated(torch, dev, w, 3 * L2_BYTES)
    ncopy = wd.shape[0]
    xf = torch.from_numpy(np.random.default_rng(k).normal(size=(n, k)).astype(np.float32)).to(dev)
    q = torch.zeros(k // 128 * n * 144, dtype=torch.uint8, device=dev)
    d = torch.zeros(n * rows, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        g.quantize_mmq(1 if ty == cfi.Q4_K else 0, xf.data_ptr(), q.data_ptr(), k, k, n, stream=stream.cuda_stream)
        g.mmq(ty, wd[0].data_ptr(), q.data_ptr(), d.data_ptr(), k, rows, n, stream=stream.cuda_stream)
    torch.cuda.synchronize()
    us = graph_time_us(stream, lambda i, st: g.mmq(ty, wd[i % ncopy].data_ptr(), q.data_ptr(), d.data_ptr(), k, rows, n,
                                                    stream=st), reps=5, calls=max(ncopy, 8))
    wbytes = w.size
    print(json.dumps({"only_mmq": spec, "us": round(us, 3), "weights_gbs": round(wbytes / us / 1e3, 1),
                      "weights_frac": round(wbytes / us / 1e3 / peaks()[0], 4),
                      "tflops": round(2.0 * rows * k * n / us / 1e6, 1), "weight_copies": ncopy,
                      "device_error": int(cfi.lib().cfi_device_error())}), flush=True)
    ctx.close()


def only_rowops():
    """The row kernels at their batched shapes alone (the rowops leg without the decode shapes),
    printed as one JSON line: the profiling entry of the row-kernel summaries."""
    import torch

    import cfi_b200 as cfi

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    ctx = cfi.Ctx(0)
    g = cfi.GgmlCaller(ctx, "all")
    stream = torch.cuda.Stream(device=dev)
    print(json.dumps({"only_rowops": rowops_bench(cfi, g, stream, dev, peaks()[0], big_only=True)}), flush=True)
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--legs", default="all", help="comma list of %s (default all)" % ",".join(ALL_LEGS))
    ap.add_argument("--exchange", default="peer", choices=("peer", "nccl"),
                    help="N > 1: the headline step's all-gather over peer memory (default) or NCCL")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the config 1, config 5 and FlashAttention legs")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--separate-quantize", action="store_true",
                    help="launch quantize_q8_1 and mul_mat_vec_q separately (no CFI_CTX_DEFER_Q8_1)")
    ap.add_argument("--only-mmq", default="",
                    help="time one mul_mat_q shape type:rows:k:cols (q4k or q8_0) and exit (profiling entry)")
    ap.add_argument("--only-rowops", action="store_true",
                    help="time only the row kernels at their batched shapes (for profiling) and exit")
    ap.add_argument("--only-gemv", default="",
                    help="type:rows:k:batch (e.g. q4k:65536:2048:8): time only that mul_mat_vec_q (for profiling) and exit")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.only_gemv:
        only_gemv(args.only_gemv)
        return
    if args.only_mmq:
        only_mmq(args.only_mmq)
        return
    if args.only_rowops:
        only_rowops()
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_gpu(args, rank, world)


if __name__ == "__main__":
    main()
