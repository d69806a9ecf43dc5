"""Per-kernel timing of the spar_b200 hot-path kernels at a given size (CUDA events, inputs larger
than L2, warm-up first) with the achieved rate against the B200 peaks.

  python -m spar_b200.microbench all
  python -m spar_b200.microbench gemm --m 8192 --n 4096 --k 4096 [--at] [--bt] [--x3]
  python -m spar_b200.microbench c3        (the C3 Linear table, TF32 and 3xTF32)
  python -m spar_b200.microbench layernorm_bwd|rmsnorm|swiglu|gelu_bwd|softmax_bwd|cross_entropy|adamw|attention

Bandwidth kernels report algorithmic bytes / time (GB/s); GEMMs report 2mnk / time (TFLOP/s).
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from . import ops

ROOT = Path(__file__).resolve().parents[1]


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    d = json.loads(p.read_text()) if p.exists() else {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
    return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0) / 2.0


EAGER = False  # --eager: plain launches, no graph (for per-kernel profilers)


def timed(fn, iters=10, warmup=3):
    """Milliseconds per call: `iters` calls captured in one CUDA graph and replayed, so host-side
    launch and allocation overhead is not timed (eager timing if the call cannot be captured, or
    with --eager)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        if EAGER:
            raise RuntimeError("eager timing requested")
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            fn()
            with torch.cuda.graph(g, stream=s):
                for _ in range(iters):
                    fn()
        g.replay()
        torch.cuda.synchronize()
        a.record()
        g.replay()
        b.record()
    except RuntimeError:
        torch.cuda.synchronize()
        a.record()
        for _ in range(iters):
            fn()
        b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


PEAK_NOTES = {
    "GB/s": "measured HBM copy (MEASURED_PEAKS.json hbm_gbs)",
    "TFLOP/s": "dense TF32 = half the measured bf16 burst GEMM rate (MEASURED_PEAKS.json "
               "bf16_tflops / 2); no TF32 rate is measured directly",
}


def report(name, ms, work, unit, peak):
    rate = work / (ms / 1e3) / (1e9 if unit == "GB/s" else 1e12)
    line = {"kernel": name, "ms": round(ms, 4), "achieved": round(rate, 1), "unit": unit,
            "peak": round(peak, 1), "frac": round(rate / peak, 3), "peak_note": PEAK_NOTES[unit]}
    print(json.dumps(line), flush=True)
    return line


EPILOGUES = {"none": ops.EPI_NONE, "bias": ops.EPI_BIAS, "bias_gelu": ops.EPI_BIAS_GELU,
             "gelu_bwd": ops.EPI_GELU_BWD, "bias_add": ops.EPI_BIAS_ADD}


def run_gemm(m, n, k, at=False, bt=False, x3=False, iters=10, epi="none"):
    dev = torch.device("cuda")
    a = torch.randn((k, m) if at else (m, k), device=dev)
    b = torch.randn((n, k) if bt else (k, n), device=dev) * 0.02
    c = torch.empty(m, n, device=dev)
    bias = torch.randn(n, device=dev) if epi in ("bias", "bias_gelu", "bias_add") else None
    aux = torch.randn(m, n, device=dev) if epi in ("bias_gelu", "gelu_bwd", "bias_add") else None
    prec = ops.TF32X3 if x3 else ops.TF32
    ms = timed(lambda: ops.matmul(a, b, a_t=at, b_t=bt, out=c, precision=prec,
                                  epilogue=EPILOGUES[epi], bias=bias, aux=aux), iters=iters)
    _, tf = peaks()
    return report(f"gemm {m}x{n}x{k} a_t={int(at)} b_t={int(bt)} {'3xtf32' if x3 else 'tf32'} "
                  f"epi={epi}", ms, 2.0 * m * n * k, "TFLOP/s", tf)


def run_c3(iters=10):
    """The isolated Linear forward and backward products of config C3 (X [8192, K] ~ N(0, 1),
    W [K, N] ~ N(0, 0.02), dY [8192, N] ~ N(0, 1)) at W = 4096 x 4096, 4096 x 16384 and
    16384 x 4096, in TF32 and 3xTF32: Y = X W + b (bias epilogue), dX = dY W^T (W read
    transposed in place), dW = X^T dY (X read transposed in place), and db = column sums of dY
    (bandwidth: 4 B per element of dY)."""
    dev = torch.device("cuda")
    hbm, tf = peaks()
    m = 8192
    for k, n in ((4096, 4096), (4096, 16384), (16384, 4096)):
        x = torch.randn(m, k, device=dev)
        w = torch.randn(k, n, device=dev) * 0.02
        dy = torch.randn(m, n, device=dev)
        bias = torch.randn(n, device=dev) * 0.02
        y = torch.empty(m, n, device=dev)
        dx = torch.empty(m, k, device=dev)
        dw = torch.empty(k, n, device=dev)
        for prec, tag in ((ops.TF32, "tf32"), (ops.TF32X3, "3xtf32")):
            fl = 2.0 * m * n * k
            report(f"c3 Y=XW+b {m}x{k}x{n} {tag}", timed(lambda: ops.matmul(
                x, w, out=y, precision=prec, epilogue=ops.EPI_BIAS, bias=bias), iters),
                fl, "TFLOP/s", tf)
            report(f"c3 dX=dY.W^T {m}x{n}x{k} {tag}", timed(lambda: ops.matmul(
                dy, w, b_t=True, out=dx, precision=prec), iters), fl, "TFLOP/s", tf)
            report(f"c3 dW=X^T.dY {k}x{m}x{n} {tag}", timed(lambda: ops.matmul(
                x, dy, a_t=True, out=dw, precision=prec), iters), fl, "TFLOP/s", tf)
        db = torch.empty(n, device=dev)
        report(f"c3 db=sum(dY) {m}x{n}", timed(lambda: ops.column_sum(dy, out=db), iters),
               4.0 * m * n, "GB/s", hbm)
        del x, w, dy, y, dx, dw
        torch.cuda.empty_cache()


def run_attention(b=16, t=1024, h=16, dh=64, iters=10):
    """Fused causal attention at the C5 shape; rate = causal useful FLOPs (QK^T and PV forward,
    five products backward) over time."""
    dev = torch.device("cuda")
    d = h * dh
    qkv = torch.randn(b, t, 3 * d, device=dev)
    do = torch.randn(b, t, d, device=dev)
    ctx, mx, inv = ops.attention_forward(qkv, h)
    _, tf = peaks()
    half = b * h * t * (t + 1) / 2 * dh * 2.0  # one causal [t, t] x dh product
    report(f"attention_fwd {b}x{h}x{t}x{dh}", timed(lambda: ops.attention_forward(qkv, h), iters),
           2 * half, "TFLOP/s", tf)
    return report(f"attention_bwd {b}x{h}x{t}x{dh}",
                  timed(lambda: ops.attention_backward(do, qkv, ctx, mx, inv, h), iters),
                  5 * half, "TFLOP/s", tf)


ADAMW_PARAMS = 350_000_000  # --adamw-params: C2's AdamW size (smaller for profiler captures)


def run_bandwidth(name, iters=10):
    dev = torch.device("cuda")
    hbm, _ = peaks()
    if name == "layernorm_bwd":
        x = torch.randn(16384, 1024, device=dev)
        dy = torch.randn_like(x)
        g = torch.ones(1024, device=dev)
        _, mean, rstd = ops.layer_norm_forward(x, g, torch.zeros_like(g))
        report("layernorm_fwd 16384x1024", timed(lambda: ops.layer_norm_forward(x, g, g), iters),
               8 * x.numel(), "GB/s", hbm)
        # As in the training step: dx accumulates into the residual-stream gradient (read + write).
        dx = torch.zeros_like(x)
        dg, db = torch.empty_like(g), torch.empty_like(g)
        return report("layernorm_bwd 16384x1024",
                      timed(lambda: ops.layer_norm_backward(dy, x, g, mean, rstd, dg, db, dx,
                                                            accumulate_dx=True), iters),
                      16 * x.numel(), "GB/s", hbm)
    if name == "rmsnorm":
        x = torch.randn(65536, 1024, device=dev)  # 256 MB: larger than L2
        dy = torch.randn_like(x)
        w = torch.ones(1024, device=dev)
        _, rstd = ops.rms_norm_forward(x, w)
        report("rmsnorm_fwd 65536x1024", timed(lambda: ops.rms_norm_forward(x, w), iters),
               8 * x.numel(), "GB/s", hbm)
        dx = torch.zeros_like(x)
        dw = torch.empty_like(w)
        return report("rmsnorm_bwd 65536x1024",
                      timed(lambda: ops.rms_norm_backward(dy, x, w, rstd, dw, dx,
                                                          accumulate_dx=True), iters),
                      16 * x.numel(), "GB/s", hbm)
    if name == "swiglu":
        # gate | value as the two halves of one fused [16384, 2 x 4096] projection output
        gv = torch.randn(16384, 8192, device=dev)
        gate, value = gv[:, :4096], gv[:, 4096:]
        h = torch.empty(16384, 4096, device=dev)
        dh = torch.randn_like(h)
        dgv = torch.empty_like(gv)
        report("swiglu_fwd 16384x4096", timed(lambda: ops.swiglu_forward(gate, value, out=h), iters),
               12 * h.numel(), "GB/s", hbm)
        return report("swiglu_bwd 16384x4096",
                      timed(lambda: ops.swiglu_backward(dh, gate, value, dgv[:, :4096],
                                                        dgv[:, 4096:]), iters),
                      20 * h.numel(), "GB/s", hbm)
    if name == "gelu_bwd":
        x = torch.randn(16384, 4096, device=dev)
        dy = torch.randn_like(x)
        return report("gelu_bwd 16384x4096", timed(lambda: ops.gelu_backward(dy, x), iters),
                      12 * x.numel(), "GB/s", hbm)
    if name == "softmax_bwd":
        t = 1024
        s = torch.randn(96, t, t, device=dev)
        p = ops.causal_softmax_forward(s, 0.125)
        dp = torch.randn_like(s)
        ds = torch.empty_like(s)
        causal = 96 * (2 * t * (t + 1) // 2 + t * t) * 4
        return report("causal_softmax_bwd 96x1024x1024", timed(lambda: ops.causal_softmax_backward(dp, p, 0.125, out=ds), iters),
                      causal, "GB/s", hbm)
    if name == "cross_entropy":
        z = 2 * torch.randn(8192, 32768, device=dev)
        tg = torch.randint(0, 32768, (8192,), dtype=torch.int32, device=dev)
        return report("cross_entropy 8192x32768", timed(lambda: ops.cross_entropy_forward_backward(z, tg, in_place=True), iters),
                      8 * z.numel(), "GB/s", hbm)
    if name == "adamw":
        n = ADAMW_PARAMS
        p = torch.randn(n, device=dev) * 0.02
        g = torch.randn(n, device=dev) * 1e-3
        m = torch.zeros_like(p)
        v = torch.zeros_like(p)
        st = ops.grad_norm_squared([g])
        ms = timed(lambda: ops.adamw_clipped([p], [g], [m], [v], st, lr=3e-4, beta1=0.9, beta2=0.95,
                                             weight_decay=0.1, step=1, max_norm=1.0), min(iters, 5))
        report(f"adamw {n / 1e6:.0f}M", ms, 28 * n, "GB/s", hbm)
        return report(f"grad_norm {n / 1e6:.0f}M", timed(lambda: ops.grad_norm_squared([g], st), min(iters, 5)),
                      4 * n, "GB/s", hbm)
    raise SystemExit(f"unknown kernel {name}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel")
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--at", action="store_true")
    ap.add_argument("--bt", action="store_true")
    ap.add_argument("--x3", action="store_true")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--epi", default="none", choices=sorted(EPILOGUES))
    ap.add_argument("--batch", type=int, default=16, help="attention: sequences (C5: 16)")
    ap.add_argument("--eager", action="store_true", help="time plain launches (no CUDA graph)")
    ap.add_argument("--adamw-params", type=int, default=350_000_000)
    a = ap.parse_args()
    global EAGER, ADAMW_PARAMS
    EAGER = a.eager
    ADAMW_PARAMS = a.adamw_params
    if a.kernel == "gemm":
        run_gemm(a.m, a.n, a.k, a.at, a.bt, a.x3, a.iters, a.epi)
    elif a.kernel == "all":
        for (m, n, k, at, bt) in [(8192, 4096, 4096, 0, 0), (8192, 4096, 4096, 0, 1),
                                  (4096, 4096, 8192, 1, 0), (16384, 3072, 1024, 0, 0),
                                  (16384, 1024, 4096, 0, 0), (1024, 4096, 16384, 1, 0),
                                  (16384, 32768, 1024, 0, 1)]:
            run_gemm(m, n, k, bool(at), bool(bt), False, a.iters)
        run_attention(iters=a.iters)
        for name in ("layernorm_bwd", "rmsnorm", "swiglu", "gelu_bwd", "softmax_bwd",
                     "cross_entropy", "adamw"):
            run_bandwidth(name, a.iters)
    elif a.kernel == "c3":
        run_c3(a.iters)
    elif a.kernel == "attention":
        run_attention(b=a.batch, iters=a.iters)
    else:
        run_bandwidth(a.kernel, a.iters)


if __name__ == "__main__":
    _ = math
    main()
