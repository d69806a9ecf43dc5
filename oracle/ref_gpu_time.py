#!/usr/bin/env python
"""Times the reference's own GPU path (TEST INFRASTRUCTURE; reported beside the product's
numbers, never a parity check).

Two builds of the reference's sources (oracle/make_ref.py) run the same Spar code on cuda:0:
  stock  Spar's own CUDA backend (src/backend/cuda_kernels.cu, synchronous SIMT kernels) and its
         cuBLAS SGEMM seam (src/backend/cuda_blas.cppm:122-194) - the GPU bar;
  b200   the same Spar code with libspar_b200.so as its backend (spar_cuda_* and the tcgen05
         matmul seam), i.e. what a Spar user gets from the drop-in alone, without the fused
         training runtime.
Workloads: the C1 tiny LN/GELU decoder step (batch 8 x 64), the C4
GPT-2-small-shaped step (12 x d768, vocabulary 50257, batch 8 x 1024), each a full step
(forward, LM loss, backward, clip, AdamW) built from Spar ops; and the C3 forward products
X [8192, K] x W [K, N] through Spar's matmul. One JSON line per measurement.

Usage: python oracle/ref_gpu_time.py [--variant stock|b200 ...] [--skip-c4]
"""
from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main() -> int:
    from oracle import cpu_ref
    from spar_b200.lm import C1, C4

    ap = argparse.ArgumentParser()
    ap.add_argument("--variant", action="append", choices=["stock", "b200"])
    ap.add_argument("--skip-c4", action="store_true")
    a = ap.parse_args()
    for variant in a.variant or ["stock", "b200"]:
        if not cpu_ref.available(variant):
            print(json.dumps({"variant": variant, "unavailable": "not built"}))
            continue
        for name, cfg, warm, iters in (("c1", C1, 2, 10), ("c4", C4, 1, 2)):
            if name == "c4" and a.skip_c4:
                continue
            s = cpu_ref.lm_step_seconds(cfg, cfg.micro_batch, warm, iters, 0, variant)
            tokens = cfg.micro_batch * cfg.seq
            print(json.dumps({"variant": variant, "workload": f"{name} train step (Spar ops)",
                              "s_per_step": round(s, 4), "tokens_per_s": round(tokens / s, 1),
                              "model_tflops": round(tokens * cfg.flops_per_token() / s / 1e12, 2)}),
                  flush=True)
        for k, n in ((4096, 4096), (4096, 16384), (16384, 4096)):
            s = cpu_ref.matmul_seconds(8192, k, n, 5, 0, variant)
            print(json.dumps({"variant": variant, "workload": f"c3 matmul 8192x{k}x{n}",
                              "ms": round(s * 1e3, 3),
                              "tflops": round(2.0 * 8192 * k * n / s / 1e12, 1)}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
