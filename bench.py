#!/usr/bin/env python
"""Benchmark of the quantized-linear hot path on B200.

Workload: the FLUX.1-dev-shaped Q8 double-stream block
linears, group 64, bf16, batch 1, M = 4608 tokens:
    QKV 3072->9216 (+bias), attn-out 3072->3072 (+bias),
    MLP up 3072->12288 (+bias, GELU-tanh fused), MLP down 12288->3072 (+bias)
One step = those four quantized_matmul calls (the down projection consumes the up
projection's output) = 1043.7 GFLOP.  Weights ~N(0, 0.02) quantized on the device,
activations ~N(0, 1), seeded synthetic data (no checkpoint or dataset involved).
Each step touches ~300 MB (> the 126 MB L2), so no explicit L2 flush is needed.

N > 1 GPUs (torchrun, one rank per GPU, NCCL): Megatron tensor parallelism of the same
block -- QKV / up column-parallel, out / down row-parallel with one all-reduce each, run
in M-slices that overlap the neighbouring GEMM slices, every GEMM reading the reduced
data -- so total work is fixed ("scaling": "strong").

Also reported (rank 0, N = 1):
  * "roofline": the tcgen05 GEMM kernel's achieved TFLOP/s (algorithmic 2*M*N*K per
    launch / CUDA-event launch time) against the measured bf16 peak;
  * "e2e": the same metric through the public API with host buffers (pinned H2D of x,
    D2H of the block output inside the timed region);
  * "cpu_baseline": the CPU oracle (oracle/qref.c, fast mode, all host threads) on a
    bounded sample of the workload;
  * "decode_gemv": the Llama-3.2-3B Q4 decode step at M = 1 in HBM GB/s,
    with the lm_head alone and the step at M = 4 and 8;
  * "other_configs": cfg1 and the Z-Image block with LoRA at full size;
  * "wan_block": the Wan2.2-shaped block (configs[4], M = 32760 Q4), the multi-GPU scaling
    workload, timed with the same tensor parallelism at every N.

`--impl reference` times the reference path's CPU implementation instead (the oracle
restatement of MLX's affine quantized_matmul; MLX itself cannot be built here).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mlx-gen_b200"))

FLUX = dict(M=4608, hidden=3072, mlp=12288, bits=8, gs=64)
METRIC = "quantized_matmul TFLOP/s (DiT M) and HBM GB/s (M=1) vs B200 peak"


WAN = dict(M=32760, hidden=5120, mlp=13824, bits=4, gs=64)

# DRAM traffic (read + write) of one launch of the dominant kernel, the GEMM's FLUX MLP-up
# launch (M=4608, N=12288, K=3072, Q8 g64, bias + GELU-tanh), from an ncu capture of the
# committed kernel (dram__bytes_read.sum + dram__bytes_write.sum); the algorithmic bytes of
# that launch are 180.4 MB.  Re-captured whenever the GEMM changes.
PROFILED_TRAFFIC = {"bytes": 179216384, "source": "ncu capture of the up launch (python bench_case.py 4608 12288 3072 8 gelu_tanh 2 gemm), not measured in this run"}


def flux_linears(cfg):
    """(name, N, K, act, tensor-parallel style, input).  The input is "x" (the block input),
    "attn" (a stand-in for the attention output, which is not part of this path) or the
    name of an earlier linear: each linear waits for the one it reads, all-reduce
    included, as in a real forward pass."""
    h, f = cfg["hidden"], cfg["mlp"]
    return [("qkv", 3 * h, h, None, "col", "x"), ("out", h, h, None, "row", "attn"),
            ("up", f, h, "gelu_tanh", "col", "out"), ("down", h, f, None, "row", "up")]


def wan_linears(cfg):
    """Wan2.2 block linears: self-attention q, k, v, o, cross-attention q, o (its k, v act
    on the 512 text tokens and are left out), FFN up (+GELU-tanh) and down: three
    row-parallel linears, so three all-reduces per block under TP."""
    h, f = cfg["hidden"], cfg["mlp"]
    return [("q", h, h, None, "col", "x"), ("k", h, h, None, "col", "x"), ("v", h, h, None, "col", "x"),
            ("o", h, h, None, "row", "v"), ("cq", h, h, None, "col", "o"), ("co", h, h, None, "row", "cq"),
            ("up", f, h, "gelu_tanh", "col", "co"), ("down", h, f, None, "row", "up")]


def block_flops(cfg, linears):
    return sum(2.0 * cfg["M"] * N * K for _, N, K, _, _, _ in linears(cfg))


def flux_flops(cfg):
    return block_flops(cfg, flux_linears)


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200", "-i", str(gpu_index)], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.seek(0)
        rows = [r.split(", ") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------- reference arm

def run_reference(args):
    """Times the CPU implementation of the path (oracle fast mode) on a bounded sample."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O  # CPU restatement of MLX's affine quantized_matmul

    cfg = dict(FLUX)
    Ms = 256  # bounded sample: 256 of the 4608 tokens per step
    rng = np.random.default_rng(0)
    lin = []
    for name, N, K, act, _, _ in flux_linears(cfg):
        w = O.to_bf16((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
        wq, s, b = O.quantize(w, cfg["gs"], cfg["bits"])
        lin.append((name, wq, s, b, O.to_bf16((rng.standard_normal(N) * 0.02).astype(np.float32))))
    x = O.to_bf16(rng.standard_normal((Ms, cfg["hidden"])).astype(np.float32))
    u_in = O.to_bf16(rng.standard_normal((Ms, cfg["mlp"])).astype(np.float32))
    threads = os.cpu_count() or 1

    def step():
        for name, wq, s, b, bias in lin:
            O.quantized_matmul_fast(u_in if name == "down" else x, wq, s, b, cfg["gs"], cfg["bits"], bias=bias,
                                    threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    flops = flux_flops(dict(cfg, M=Ms))
    v = flops / dt / 1e12
    out = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": "flux_q8_block_linears", "M": cfg["M"], "sample_tokens": Ms, "bits": 8,
                      "group_size": 64},
           "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                            "sample": f"{Ms} of {cfg['M']} tokens through the 4 FLUX block linears per step",
                            "host_cpu": host_cpu()},
           "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "MLX (the reference's backend) cannot be built here; this is the CPU oracle "
                   "restatement (oracle/qref.c) pinned to the reference fixture"}
    print(json.dumps(out), flush=True)


# ----------------------------------------------------------------------------- GPU arm

def host_cpu():
    """Model name and logical CPU count of the host (from /proc/cpuinfo)."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"model": model, "logical_cpus": os.cpu_count()}


def cpu_baseline_sample(cfg, tokens=(256, 32)):
    """The oracle's fast mode (pthreads, all host threads) on the first `tokens[0]` tokens of
    the FLUX block's four linears; the rate at the other sample sizes shows how flat the CPU
    rate is in M."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    rng = np.random.default_rng(1)
    threads = os.cpu_count() or 1
    lin = []
    for name, N, K, act, _, _ in flux_linears(cfg):
        w = O.to_bf16((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
        lin.append((N, K) + O.quantize(w, cfg["gs"], cfg["bits"]))
    rates = {}
    for Ms in tokens:
        t_total, flops = 0.0, 0.0
        for N, K, wq, s, b in lin:
            x = O.to_bf16(rng.standard_normal((Ms, K)).astype(np.float32))
            O.quantized_matmul_fast(x, wq, s, b, cfg["gs"], cfg["bits"], threads=threads)  # warm
            t0 = time.perf_counter()
            O.quantized_matmul_fast(x, wq, s, b, cfg["gs"], cfg["bits"], threads=threads)
            t_total += time.perf_counter() - t0
            flops += 2.0 * Ms * N * K
        rates[Ms] = flops / t_total / 1e12
    Ms = tokens[0]
    return {"value": rates[Ms], "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{Ms} of {cfg['M']} tokens through the 4 FLUX block linears (oracle fast mode)",
            "rate_by_tokens": {str(k): v for k, v in rates.items()}, "host_cpu": host_cpu()}


def timed_flushed(fn, iters, flush):
    """Mean CUDA-event time (ms) of fn over `iters` calls, with an L2 flush (a write larger
    than the 126 MB L2) before each call, outside the timed events."""
    import torch

    fn()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(iters):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    return tot / iters


def quant_dequant(dev, peaks, iters=10):
    """quantize (bf16 W -> packed Q4 g64) and dequantize (-> bf16) in HBM GB/s, algorithmic
    bytes: quantize N*K*2 + N*K*bits/8 + N*(K/gs)*4, dequantize N*K*bits/8 + N*(K/gs)*4 +
    N*K*2.  W of cfg1 (3072 x 3072) and of the Wan FFN up projection (13824 x 5120); L2
    flushed before every call."""
    import torch
    import qlinear

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(21)
    out = {}
    for name, N, K, bits, gs in (("cfg1_w_q4", 3072, 3072, 4, 64), ("wan_ffn_w_q4", 13824, 5120, 4, 64)):
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        wq, s, b = qlinear.quantize(w, gs, bits)
        deq = torch.empty(N, K, dtype=torch.bfloat16, device=dev)
        qb = N * K * 2 + N * K * bits // 8 + N * (K // gs) * 4
        db = N * K * bits // 8 + N * (K // gs) * 4 + N * K * 2
        from qlinear import _lib, ops
        import ctypes as C

        def q():
            _lib.check(_lib.lib().ql_quantize(ops._ptr(w), _lib.QL_BF16, N, K, gs, bits, ops._ptr(wq), ops._ptr(s),
                                              ops._ptr(b), _lib.QL_BF16, ops._stream(dev)))

        def d():
            _lib.check(_lib.lib().ql_dequantize(ops._ptr(wq), ops._ptr(s), ops._ptr(b), _lib.QL_BF16, N, K, gs, bits,
                                                ops._ptr(deq), _lib.QL_BF16, ops._stream(dev)))

        qms, dms = timed_flushed(q, iters, flush), timed_flushed(d, iters, flush)
        out[name] = {"shape": f"{N}x{K} Q{bits} g{gs}",
                     "quantize": {"value": qb / (qms * 1e-3) / 1e9, "unit": "GB/s", "us": qms * 1e3, "bytes": qb,
                                  "frac_of_hbm": qb / (qms * 1e-3) / 1e9 / peaks["hbm_gbs"]},
                     "dequantize": {"value": db / (dms * 1e-3) / 1e9, "unit": "GB/s", "us": dms * 1e3, "bytes": db,
                                    "frac_of_hbm": db / (dms * 1e-3) / 1e9 / peaks["hbm_gbs"]}}
        del w, wq, s, b, deq
    assert qlinear.device_error() == 0
    return out


def decode_gemv(dev, steps=20, warmup=5, M=1, head=True):
    """Llama-3.2-3B Q4 g64 decode step at M tokens: 28 x (qkv, o, gate/up SwiGLU, down) +
    lm_head; `head` also times the lm_head alone."""
    import torch
    import qlinear

    H, I, V, L, KV = 3072, 8192, 128256, 28, 1024
    g = torch.Generator(device=dev).manual_seed(3)

    def qlin(N, K):
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        return qlinear.quantize(w, 64, 4)

    layers = []
    for _ in range(L):
        layers.append(dict(qkv=qlin(H + 2 * KV, H), o=qlin(H, H), gate=qlin(I, H), up=qlin(I, H), down=qlin(H, I)))
    head = qlin(V, H)
    h = torch.randn(M, H, device=dev, generator=g).to(torch.bfloat16)
    bufs = dict(qkv=torch.empty(M, H + 2 * KV, device=dev, dtype=torch.bfloat16),
                o=torch.empty(M, H, device=dev, dtype=torch.bfloat16),
                g=torch.empty(M, I, device=dev, dtype=torch.bfloat16),
                h=torch.empty(M, H, device=dev, dtype=torch.bfloat16),
                logits=torch.empty(M, V, device=dev, dtype=torch.bfloat16))

    def step():
        x = h
        for ly in layers:
            qlinear.quantized_matmul(x, *ly["qkv"], True, 64, 4, out=bufs["qkv"])
            qlinear.quantized_matmul(x, *ly["o"], True, 64, 4, out=bufs["o"])
            qlinear.quantized_matmul(bufs["o"], *ly["gate"], True, 64, 4, act="swiglu", up=ly["up"], out=bufs["g"])
            qlinear.quantized_matmul(bufs["g"], *ly["down"], True, 64, 4, out=bufs["h"])
            x = bufs["h"]
        qlinear.quantized_matmul(x, *head, True, 64, 4, out=bufs["logits"])

    def nbytes(N, K):
        return N * K * 4 // 8 + N * (K // 64) * 4 + M * (K + N) * 2

    per_layer = nbytes(H + 2 * KV, H) + nbytes(H, H) + 2 * nbytes(I, H) - (H * 2) + nbytes(H, I)
    total_bytes = L * per_layer + nbytes(V, H)
    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        step()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=s):
            step()
    torch.cuda.synchronize()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    res = {"workload": f"llama3.2-3b_q4_g64_decode_M{M}", "value": total_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
           "ms_per_step": ms, "bytes_per_step": total_bytes, "launches_per_step": 4 * L + 1,
           "timing": "CUDA graph of one decode step; 1.8 GB of weights per step (> L2)"}
    if not head:
        return res
    # the lm_head alone (one 197 MB GEMV, the largest single launch of the step)
    def head_only():
        for _ in range(4):
            qlinear.quantized_matmul(h, *head, True, 64, 4, out=bufs["logits"])

    head_only()
    torch.cuda.synchronize()
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        head_only()
        torch.cuda.synchronize()
        with torch.cuda.graph(g2, stream=s):
            head_only()
    torch.cuda.synchronize()
    g2.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(5):
        g2.replay()
    e1.record()
    torch.cuda.synchronize()
    head_ms = e0.elapsed_time(e1) / 20
    res["lm_head_gemv"] = {"value": nbytes(V, H) / (head_ms * 1e-3) / 1e9, "unit": "GB/s", "us": head_ms * 1e3,
                           "shape": f"M={M} N=128256 K=3072 Q4 g64 (197 MB > L2), 20 launches in a graph"}
    return res


def other_configs(dev, iters=5):
    """The other BASELINE configs' GEMM shapes at full size (TFLOP/s, 2*M*N*K per linear,
    LoRA flops not counted): cfg1 (M=4096, 3072x3072 Q4), Z-Image block (M=4608 Q4,
    4 x 3840^2 attention linears and the MLP down with LoRA r=32 fused, the SwiGLU pair
    fused).  The Wan block is timed at every N by run_ours ("wan_block")."""
    import torch
    import qlinear

    g = torch.Generator(device=dev).manual_seed(5)

    def qlin(N, K, bits, gs=64):
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        return qlinear.quantize(w, gs, bits)

    def lora(N, K, r=32):
        a = (torch.randn(K, r, device=dev, generator=g) / r ** 0.5).to(torch.bfloat16)
        b = (torch.randn(r, N, device=dev, generator=g) * 0.01).to(torch.bfloat16)
        return (a, b, 1.0)

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    out = {}
    # cfg1
    M = 4096
    w1 = qlin(3072, 3072, 4)
    x = torch.randn(M, 3072, device=dev, generator=g).to(torch.bfloat16)
    y = torch.empty(M, 3072, device=dev, dtype=torch.bfloat16)
    ms = timed(lambda: qlinear.quantized_matmul(x, *w1, True, 64, 4, out=y))
    fl = 2 * M * 3072 * 3072
    out["cfg1_q4_4096x3072x3072"] = {"value": fl / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": ms}
    del w1, x, y
    # Z-Image block (Q4, LoRA r=32 on the attention linears and the MLP down)
    M, D, F = 4608, 3840, 10240
    att = [(qlin(D, D, 4), lora(D, D)) for _ in range(4)]
    w1, w3 = qlin(F, D, 4), qlin(F, D, 4)
    w2, l2 = qlin(D, F, 4), lora(D, F)
    x = torch.randn(M, D, device=dev, generator=g).to(torch.bfloat16)
    ya = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
    yf = torch.empty(M, F, device=dev, dtype=torch.bfloat16)
    ws = torch.empty(qlinear.workspace_size(M, F, F, 32), dtype=torch.uint8, device=dev)

    def zimage():
        for wq, lo in att:
            qlinear.quantized_matmul(x, *wq, True, 64, 4, lora=lo, workspace=ws, out=ya)
        qlinear.quantized_matmul(x, *w1, True, 64, 4, act="swiglu", up=w3, out=yf)
        qlinear.quantized_matmul(yf, *w2, True, 64, 4, lora=l2, workspace=ws, out=ya)

    ms = timed(zimage)
    fl = 2 * M * (4 * D * D + 2 * F * D + D * F)
    # FLUX.1 block linears with f32 activations (FLUX.2 / Qwen image streams feed f32 x):
    # the tensor-core three-pass split path, f32 output
    M, h, f = 4608, 3072, 12288
    fl_lin = [(qlin(3 * h, h, 8), h, 3 * h, None), (qlin(h, h, 8), h, h, None),
              (qlin(f, h, 8), h, f, "gelu_tanh"), (qlin(h, f, 8), f, h, None)]
    xs32 = {k: torch.randn(M, k, device=dev, generator=g) for k in (h, f)}
    ys32 = {n: torch.empty(M, n, device=dev) for n in (h, 3 * h, f)}
    wsx = torch.empty(max(int(qlinear.ops.lib().ql_matmul_workspace_size_x(M, 1, k, None, 0)) for k in (h, f)),
                      dtype=torch.uint8, device=dev)

    def flux_f32():
        for w_, k, n, a in fl_lin:
            qlinear.quantized_matmul(xs32[k], *w_, True, 64, 8, act=a, out=ys32[n], workspace=wsx)

    ms32 = timed(flux_f32)
    fl32 = sum(2 * M * n * k for _, k, n, _ in fl_lin)
    out["flux_q8_block_f32_activations"] = {"value": fl32 / (ms32 * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": ms32,
                                            "path": "tcgen05 GEMM, three bf16 passes (x and w split hi + lo)"}
    del fl_lin, xs32, ys32, wsx
    # adaLN prologue (FLUX's layer_norm + modulate before the QKV and MLP-up linears) as its
    # own one-pass kernel: its cost against the linears it feeds
    xm = torch.randn(M, h, device=dev, generator=g).to(torch.bfloat16)
    sc = (torch.randn(h, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    sh = (torch.randn(h, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    wqkv, wup = qlin(3 * h, h, 8), qlin(f, h, 8)
    yq = torch.empty(M, 3 * h, device=dev, dtype=torch.bfloat16)
    yu = torch.empty(M, f, device=dev, dtype=torch.bfloat16)
    xn = qlinear.layernorm_modulate(xm, sc, sh)

    def gemms_only():
        qlinear.quantized_matmul(xn, *wqkv, True, 64, 8, out=yq)
        qlinear.quantized_matmul(xn, *wup, True, 64, 8, act="gelu_tanh", out=yu)

    def with_adaln():
        x1 = qlinear.layernorm_modulate(xm, sc, sh)
        qlinear.quantized_matmul(x1, *wqkv, True, 64, 8, out=yq)
        x2 = qlinear.layernorm_modulate(xm, sc, sh)
        qlinear.quantized_matmul(x2, *wup, True, 64, 8, act="gelu_tanh", out=yu)

    t_g, t_a = timed(gemms_only), timed(with_adaln)
    out["adaln_prologue_overhead"] = {"gemms_ms": t_g, "with_two_adaln_passes_ms": t_a,
                                      "overhead_frac": (t_a - t_g) / t_g,
                                      "shape": "FLUX Q8 QKV 3072->9216 and MLP-up 3072->12288 at M=4608, each fed "
                                               "by its own layer_norm + modulate pass over x [4608, 3072] bf16"}
    del xm, yq, yu, xn
    out["zimage_q4_lora32_block"] = {"value": fl / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": ms,
                                     "lora_gflop_not_counted": 2 * M * 32 * (5 * D + 4 * D + F) / 1e9}
    return out


def build_block(cfg, linears, dev, seed, comm, comm_sms, chunks, mode="allreduce"):
    """Seeded synthetic weights (identical on every rank: the same generator seed) and the
    block input, then the product's tensor-parallel block (qlinear.tp.TPBlock) over `comm`.
    Returns (block, unsharded weights, x, external inputs, spec)."""
    import torch
    import qlinear
    from qlinear import tp

    g = torch.Generator(device=dev).manual_seed(seed)
    weights, spec = {}, []
    for name, N, K, act, style, src in linears(cfg):
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        bias = (torch.randn(N, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        weights[name] = (*qlinear.quantize(w, cfg["gs"], cfg["bits"]), bias)
        del w
        spec.append((name, act, style, src))
    x = torch.randn(cfg["M"], cfg["hidden"], device=dev, generator=g).to(torch.bfloat16)
    ext = {}
    for name, N, K, act, style, src in linears(cfg):
        if src == "attn":  # stand-in for the attention output (not part of this path), full width
            ext["attn"] = torch.randn(cfg["M"], K, device=dev, generator=g).to(torch.bfloat16)
    blk = tp.TPBlock(spec, weights, cfg["gs"], cfg["bits"], cfg["M"], comm=comm, chunks=chunks, mode=mode,
                     comm_sms=comm_sms, device=dev)
    torch.cuda.synchronize()
    return blk, weights, x, ext, spec


def tp_parity(blk, weights, spec, cfg, x, ext):
    """The tensor-parallel block output (gathered from the ranks) against the unsharded block
    computed on this GPU with the plain single-GPU quantized_matmul chain, same weights and
    inputs.  Returns {"max_abs", "rel_l2", "ok", ...}; "ok" uses qlinear.tp.parity's bound."""
    import torch
    from qlinear import tp

    blk.forward(x, ext)
    got = blk.gather_output()
    torch.cuda.synchronize()
    ref = tp.reference_forward(spec, weights, cfg["gs"], cfg["bits"], x, ext)["out"]
    torch.cuda.synchronize()
    return tp.parity(got, ref, blk.world)


def time_block(blk, inp, steps, warmup, world, graph=False):
    """Device time per step of `blk` (CUDA events, max over ranks); `graph`: each step is
    one replay of the block captured as a CUDA graph."""
    import torch
    import torch.distributed as dist

    gr = blk.capture(*inp) if graph else None
    fwd = gr.replay if graph else (lambda: blk.forward(*inp))
    for _ in range(warmup):
        fwd()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        fwd()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    if gr is not None:
        gr.reset()  # holds NCCL work: freed before the communicator's teardown
    if world > 1:
        tt = torch.tensor([ms], device=blk.dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    return ms


def breakdown(blk, x, ext, steps, world):
    """Per-step GEMM time (events on the main stream), collective time (events on the
    communication stream) and the exposed remainder (step time not covered by GEMMs), from a
    separate short run with events around every launch (not the timed region)."""
    import torch

    for _ in range(2):
        blk.forward(x, ext)
    torch.cuda.synchronize()
    evs, cevs = [], []
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        blk.forward(x, ext, evs=evs, cevs=cevs)
    t1.record()
    torch.cuda.synchronize()
    step_ms = t0.elapsed_time(t1) / steps
    gemm_ms = sum(a.elapsed_time(b) for _, a, b in evs) / steps
    coll_ms = sum(a.elapsed_time(b) for _, a, b in cevs) / steps
    per = {}
    for name, a, b in evs:
        per[name] = per.get(name, 0.0) + a.elapsed_time(b) / steps
    return {"step_ms": step_ms, "gemm_ms": gemm_ms, "collective_ms": coll_ms,
            "exposed_ms": max(step_ms - gemm_ms, 0.0), "gemm_ms_per_linear": per,
            "note": f"rank {blk.rank}; separate {steps}-step run with events around every GEMM / collective"}


def bind_host_to_gpu(dev):
    """Pin this process to the CPUs NVML reports as closest to `dev` (read-only NVML query),
    so that its pinned host buffers are allocated on the GPU's own NUMA node: with several
    ranks copying at once, buffers on one socket made the host side the bottleneck.
    Returns the number of CPUs bound to, or None when NVML cannot say."""
    try:
        import pynvml
        import torch

        pr = torch.cuda.get_device_properties(dev)
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:"
                                                     f"{pr.pci_device_id:02x}.0".encode())
            nwords = (os.cpu_count() + 63) // 64
            words = pynvml.nvmlDeviceGetCpuAffinity(h, nwords)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (w >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return len(cpus)
    except Exception:  # no NVML or no affinity information: leave the process unbound
        return None


def run_ours(args):
    import torch
    import torch.distributed as dist

    import qlinear
    from qlinear import tp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    json_out = sys.stdout
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    host_cpus = bind_host_to_gpu(dev) if world > 1 else None
    comm = None
    if world > 1:
        # NCCL's log (e.g. its version banner) goes to stderr: stdout carries only the JSON line
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        if args.nccl_channels > 0:  # NCCL's CTAs per collective: the SMs the GEMMs leave free
            os.environ.setdefault("NCCL_MAX_NCHANNELS", str(args.nccl_channels))
        # anything native code prints on fd 1 (NCCL's version banner) goes to stderr too;
        # the JSON line is written to the saved stdout
        sys.stdout.flush()
        json_fd = os.dup(1)
        os.dup2(2, 1)
        json_out = os.fdopen(json_fd, "w")
        comm = tp.Comm.init("nccl", device=dev, timeout_s=120.0)
    cfg = dict(FLUX)
    M, gs, bits = cfg["M"], cfg["gs"], cfg["bits"]

    # weights: generated and quantized identically on every rank, then sharded by qlinear.tp
    blk, weights, x, ext, spec = build_block(cfg, flux_linears, dev, 0, comm, args.comm_sms, chunks=args.flux_chunks)
    # the TP output against the unsharded single-GPU block (before any timing)
    par = tp_parity(blk, weights, spec, cfg, x, ext)
    del weights
    torch.cuda.empty_cache()
    if not par["ok"]:
        raise SystemExit(f"rank {rank}: tensor-parallel block output differs from the unsharded block: {par}")
    # (name, start, end) of the dominant GEMM launch (MLP-up) in the timed region (N = 1):
    # events around every launch would expose each launch's start-up, which back-to-back
    # launches otherwise hide, and slow the very step they time
    evs = []
    ROOF = "up"

    def step(record=False, xin=None, names=(ROOF,)):
        return blk.forward(x if xin is None else xin, ext, evs=evs if record else None, ev_names=set(names))

    # --graph (N > 1): the device-timed step is issued as one CUDA graph replay of the
    # sharded block (TPBlock.capture) instead of a dozen GEMM launches, collectives and
    # stream joins from Python.  Measured equal at N = 2 and within run-to-run spread at
    # N = 4, so eager stays the default.  N = 1 stays eager (its timed region records events
    # around the MLP-up launch for the roofline); so does the e2e loop.
    graphs = {}

    def gstep(xin=None):
        xin = x if xin is None else xin
        key = xin.data_ptr()
        if key not in graphs:
            graphs[key] = blk.capture(xin, ext)
        return graphs[key].replay()

    use_graph = world > 1 and args.graph
    run_step = gstep if use_graph else step

    for _ in range(max(args.warmup, 3)):
        run_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # clocks are sampled from here to the end of the timed region; a ~1 s untimed soak
    # first brings the GPU to its steady (power-capped) clock so the samples describe load
    clocks = ClockSampler(local) if rank == 0 else None
    # ~1 s of untimed soak; the step count is agreed across ranks (every rank must run the
    # same number of collectives)
    t_w = time.perf_counter()
    for _ in range(3):
        run_step()
    torch.cuda.synchronize()
    n_soak = torch.tensor([int(1.0 / max((time.perf_counter() - t_w) / 3, 1e-4))], device=dev)
    if world > 1:
        dist.all_reduce(n_soak, op=dist.ReduceOp.MAX)
    for _ in range(int(n_soak.item())):
        run_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        if use_graph:
            gstep()
        else:
            step(record=(world == 1))
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1) / args.steps
    ck = clocks.stop() if clocks else None
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    total_flops = flux_flops(cfg)
    value = total_flops / (ms * 1e-3) / 1e12
    assert qlinear.device_error() == 0, "a kernel reported a device-side error"
    bd = breakdown(blk, x, ext, 5, world) if world > 1 else None

    result = None
    if rank == 0:
        peaks, src = load_peaks()
        result = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                  "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
                  "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                  "data": "synthetic (seeded; W~N(0,0.02) quantized Q8 g64 on device, x~N(0,1))",
                  "config": {"workload": "flux_q8_block_linears", "M": M, "hidden": cfg["hidden"],
                             "mlp": cfg["mlp"], "bits": bits, "group_size": gs,
                             "flops_per_step": total_flops,
                             "parallelism": f"tp{world}" if world > 1 else "single",
                             "overlap": (f"row-parallel outputs all-reduced in {len(blk.bounds)} M-slices on a second stream, overlapping the next slice's GEMM; the consumer's slice i starts once slice i is reduced" if len(blk.bounds) > 1 else "one all-reduce per row-parallel linear, no slicing") + ("; each step one CUDA graph replay" if use_graph else "") if world > 1 else None,
                             "l2": "no flush: each step touches ~300 MB (> 126 MB L2)"},
                  "gpu_launches": blk.launches * args.steps,
                  "tp_parity": par,
                  "clocks": ck}
        if bd is not None:
            result["breakdown"] = bd
        if world == 1:
            # roofline of the dominant kernel (qgemm_sm100, the MLP-up launch): its algorithmic
            # flops / its CUDA-event time, averaged over the timed region's launches
            up_ms = statistics.mean(e0.elapsed_time(e1) for name, e0, e1 in evs if name == ROOF)
            up_flops = next(2.0 * M * l.N_full * l.K_full for n, l in blk.lin.items() if n == ROOF)
            achieved = up_flops / (up_ms * 1e-3) / 1e12
            peak = peaks["bf16_tflops_sustained"]
            # every launch's time, from a short recorded pass after the timed region (events
            # around each launch: each includes its exposed start-up)
            evs.clear()
            for _ in range(5):
                step(record=True, names=[n for n, _, _, _ in spec])
            torch.cuda.synchronize()
            per = {}
            for name, e0, e1 in evs:
                per.setdefault(name, []).append(e0.elapsed_time(e1))
            result["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                                  "frac": achieved / peak, "peak_kind": f"{src} bf16 sustained",
                                  "frac_of_burst": achieved / peaks["bf16_tflops"],
                                  "traffic": PROFILED_TRAFFIC["bytes"], "traffic_source": PROFILED_TRAFFIC["source"],
                                  "kernel": "qgemm_sm100, MLP-up launch (M=4608, 3072->12288, Q8, bias+GELU): "
                                            f"{up_flops / 1e9:.1f} GFLOP per launch, CUDA events around each of "
                                            f"the {args.steps} in the timed region",
                                  "launch_ms": up_ms,
                                  "per_launch_ms_recorded_pass": {k: statistics.mean(v) for k, v in per.items()}}
    # e2e through the public API with host buffers.  N > 1: every rank moves 1/N of the rows
    # over its own PCIe link -- its slice of x up (then an NCCL all-gather over NVLink gives
    # every rank the whole input) and its slice of the block output down.  Each step's
    # copies are issued on two copy streams (double-buffered device buffers), so step i+1's
    # upload and step i-1's download run on the copy engines under step i's GEMMs; every
    # copy of every step is inside the timed region.  Two different host inputs alternate
    # in pairs of steps (so each device buffer receives a different input than it held
    # before) and the downloads rotate over four pinned host buffers: the last four steps'
    # outputs are each checked against their own input's expected result, which catches a
    # missing or misplaced ordering wait.
    rows = M // world
    g_in = torch.Generator(device=dev).manual_seed(11)
    x_alt = [x, torch.randn(M, cfg["hidden"], device=dev, generator=g_in).to(torch.bfloat16)]
    xh = [xa[rank * rows:(rank + 1) * rows].cpu().pin_memory() for xa in x_alt]
    out_t, out_rows = blk.result_rows()
    comp = blk.main
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    xd2 = [torch.empty_like(x) for _ in range(2)]
    yd2 = [torch.empty(rows, cfg["hidden"], dtype=torch.bfloat16, device=dev) for _ in range(2)]
    yh4 = [torch.empty(rows, cfg["hidden"], dtype=torch.bfloat16).pin_memory() for _ in range(4)]
    in_ready, in_free, out_ready, out_free = ([torch.cuda.Event() for _ in range(2)] for _ in range(4))
    yh_free = [torch.cuda.Event() for _ in range(4)]

    def own_rows(y):
        return y if out_rows < M else y[rank * rows:(rank + 1) * rows]

    y_expect = [own_rows(step(xin=xa)).cpu() for xa in x_alt]  # what the pipeline must deliver
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0.record(comp)
    s_in.wait_stream(comp)
    s_out.wait_stream(comp)
    for i in range(args.steps):
        j, src_i = i % 2, (i // 2) % 2
        xpart = xd2[j][rank * rows:(rank + 1) * rows]
        if i >= 2:
            s_in.wait_event(in_free[j])  # step i-2 has consumed this input buffer
        with torch.cuda.stream(s_in):
            xpart.copy_(xh[src_i], non_blocking=True)
        in_ready[j].record(s_in)
        comp.wait_event(in_ready[j])
        if world > 1:
            comm.all_gather(xd2[j], xpart)
        y = step(xin=xd2[j])
        in_free[j].record(comp)
        if i >= 2:
            comp.wait_event(out_free[j])  # step i-2's download has left this buffer
        yd2[j].copy_(own_rows(y))
        out_ready[j].record(comp)
        s_out.wait_event(out_ready[j])
        with torch.cuda.stream(s_out):
            yh4[i % 4].copy_(yd2[j], non_blocking=True)
        out_free[j].record(s_out)
    comp.wait_stream(s_out)
    t1.record(comp)
    torch.cuda.synchronize()
    # bit-exact on one GPU; across ranks the reductions may legitimately change order
    for i in range(max(0, args.steps - 4), args.steps):
        got, want = yh4[i % 4], y_expect[(i // 2) % 2]
        assert torch.allclose(got.float(), want.float(), rtol=2e-2, atol=2e-2) and \
            (world > 1 or torch.equal(got, want)), f"pipelined e2e delivered a wrong block output at step {i}"
    e2e_ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    for gr in graphs.values():
        gr.reset()  # the graphs hold NCCL work: freed before the communicator's teardown
    graphs.clear()
    # the Wan2.2-shaped block: the multi-GPU scaling workload of the path, timed
    # at every N with the same tensor-parallel scheme
    wan = None
    if not args.no_extras:
        del blk, x, xd2, yd2, x_alt
        torch.cuda.empty_cache()
        wcfg = dict(WAN)
        wblk, wweights, wx, wext, wspec = build_block(wcfg, wan_linears, dev, 4, comm, args.comm_sms, chunks=args.wan_chunks,
                                                      mode="seqpar")
        wpar = tp_parity(wblk, wweights, wspec, wcfg, wx, wext)
        del wweights
        torch.cuda.empty_cache()
        if not wpar["ok"]:
            raise SystemExit(f"rank {rank}: tensor-parallel Wan block differs from the unsharded block: {wpar}")
        wms = time_block(wblk, (wx, wext), steps=5, warmup=2, world=world, graph=world > 1 and args.graph)
        wbd = breakdown(wblk, wx, wext, 3, world) if world > 1 else None
        wan = {"workload": "wan2.2_q4_block_linears", "value": wblk.flops / (wms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": wms, "n_gpus": world, "M": WAN["M"], "flops_per_step": wblk.flops,
               "parallelism": f"tp{world}" if world > 1 else "single",
               "reductions_per_step": 3 if world > 1 else 0, "slices": len(wblk.bounds),
               "tp_mode": "sequence parallel (reduce-scatter + all-gather per slice)" if world > 1 else None,
               "gpu_launches_per_step": wblk.launches, "tp_parity": wpar, "breakdown": wbd}
        assert qlinear.device_error() == 0, "a kernel reported a device-side error"
        del wblk
        torch.cuda.empty_cache()
    if rank == 0:
        if wan is not None:
            result["wan_block"] = wan
        result["e2e"] = {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                         "h2d_bytes_per_step": M * cfg["hidden"] * 2, "d2h_bytes_per_step": M * cfg["hidden"] * 2,
                         "ms_per_step": e2e_ms,
                         "path": "pinned H2D of x and D2H of the block output inside the timed region, "
                                 "double-buffered on two copy streams under the neighbouring steps' GEMMs; "
                                 "two inputs alternate, the last 4 steps' outputs checked"
                                 + ("; each rank copies 1/N of the rows each way, x all-gathered over NCCL"
                                    if world > 1 else ""),
                         "host_cpus_bound": host_cpus}
        if world == 1 and not args.no_extras:
            result["cpu_baseline"] = cpu_baseline_sample(cfg)
            result["decode_gemv"] = decode_gemv(dev)
            peaks, src = load_peaks()
            result["decode_gemv"]["frac_of_hbm"] = result["decode_gemv"]["value"] / peaks["hbm_gbs"]
            lm = result["decode_gemv"]["lm_head_gemv"]
            lm["frac_of_hbm"] = lm["value"] / peaks["hbm_gbs"]
            for m in (4, 8):
                d = decode_gemv(dev, M=m, head=False)
                result["decode_gemv"][f"M{m}"] = {"value": d["value"], "unit": "GB/s", "ms_per_step": d["ms_per_step"],
                                                  "frac_of_hbm": d["value"] / peaks["hbm_gbs"]}
            result["other_configs"] = other_configs(dev)
            ad = result["other_configs"].get("adaln_prologue_overhead")
            if ad:  # the two passes against the whole FLUX block step measured above
                ad["frac_of_block_step"] = (ad["with_two_adaln_passes_ms"] - ad["gemms_ms"]) / result["ms_per_step"]
            result["quant_dequant"] = quant_dequant(dev, peaks)
        print(json.dumps(result), file=json_out, flush=True)
    if comm is not None:
        comm.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--graph", action="store_true", help="N > 1: time the sharded step as CUDA graph replays")
    ap.add_argument("--no-extras", action="store_true", help="skip cpu_baseline and decode_gemv")
    ap.add_argument("--comm-sms", type=int, default=0,
                    help="SMs the GEMMs leave to NCCL when N > 1 (0 measured best at N = 4 and 8)")
    ap.add_argument("--nccl-channels", type=int, default=0,
                    help="NCCL_MAX_NCHANNELS for N > 1 (0: NCCL's choice)")
    ap.add_argument("--flux-chunks", type=int, default=1,
                    help="token-row slices of the FLUX block's reductions (1 measured best at N = 4 and 8)")
    ap.add_argument("--wan-chunks", type=int, default=4, help="token-row slices of the Wan block's reductions")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
