#!/usr/bin/env python
"""Generates the golden fixtures in tests/golden/ by running the reference implementation itself
(bzzling/spar compiled from its own sources: oracle/_ref/libspar_ref.so, built by
oracle/make_ref.py). The reference ships no tests or golden vectors, so these fixtures are how the
CPU oracle and the CUDA path are pinned to the reference's behaviour.

Inputs are regenerated from seeds (SplitMix64 streams of oracle/spar_oracle.py, which the tests
also use); each .npz stores the inputs it needs and the reference outputs.

Usage: python tests/golden/make_golden.py [name ...]   (all fixtures take a few minutes: the
reference is slow; names restrict the writes, e.g. `rmsnorm swiglu`)
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

import cpu_ref as R  # noqa: E402
from oracle import spar_oracle as O  # noqa: E402


def normal(seed, shape, std=1.0):
    return O.Random(seed).normal(int(np.prod(shape)), std).reshape(shape)


def save(name, **arrays):
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(name, {k: v.shape for k, v in arrays.items()})


def main(only=()):
    """Writes every fixture, or only those named in `only` (the .npz stems)."""
    global save
    if only:
        write = save

        def save(name, **arrays):  # noqa: F811 - restrict the writes to the names asked for
            if name in only:
                write(name, **arrays)
    # LayerNorm (composed from Spar ops), incl. a wide-range row
    x = normal(1, (24, 64))
    x[3] *= 100.0
    g = 1.0 + normal(2, (64,), 0.1)
    b = normal(3, (64,), 0.1)
    dy = normal(4, (24, 64))
    y, dx, dg, db = R.layernorm(x, g, b, dy, 1e-5)
    save("layernorm", x=x, gamma=g, beta=b, dy=dy, y=y, dx=dx, dgamma=dg, dbeta=db)

    # RMSNorm (nn::RMSNorm), incl. a wide-range row and a zero row
    x = normal(30, (24, 96))
    x[5] *= 100.0
    x[9] = 0.0
    w = 1.0 + normal(31, (96,), 0.1)
    dy = normal(32, (24, 96))
    y, dx, dw = R.rmsnorm(x, w, dy, 1e-5)
    save("rmsnorm", x=x, weight=w, dy=dy, y=y, dx=dx, dweight=dw)

    # SwiGLU (nn::swiglu), incl. large |gate| and zero
    gt = np.concatenate([normal(33, (500,), 3.0),
                         np.array([0.0, -30.0, 30.0, 1e-6, -1e-6, -90.0, 90.0], np.float32)])
    vl = normal(34, gt.shape)
    dh = normal(35, gt.shape)
    h, dgt, dvl = R.swiglu(gt, vl, dh)
    save("swiglu", gate=gt, value=vl, dh=dh, h=h, dgate=dgt, dvalue=dvl)

    # Grouped-query causal attention (4 query heads sharing 2 key/value heads), head_dim 32
    qa = normal(36, (1, 4, 40, 32))
    ka = normal(37, (1, 2, 40, 32))
    va = normal(38, (1, 2, 40, 32))
    doa = normal(39, (1, 4, 40, 32))
    oa, dqa, dka, dva = R.attention(qa, ka, va, doa)
    save("attention_gqa", q=qa, k=ka, v=va, d_out=doa, out=oa, dq=dqa, dk=dka, dv=dva)

    # GELU through Spar's sigmoid, incl. large |x| and zero
    x = np.concatenate([normal(5, (500,), 3.0), np.array([0.0, -30.0, 30.0, 1e-6, -1e-6, 15.0],
                                                          np.float32)])
    dy = normal(6, x.shape)
    y, dx = R.gelu(x, dy)
    save("gelu", x=x, dy=dy, y=y, dx=dx)

    # causal softmax (scale + causal mask + softmax) and its backward
    s = normal(7, (3, 20, 20))
    dp = normal(8, (3, 20, 20))
    p, ds = R.causal_softmax(s, dp, 0.125)
    save("causal_softmax", s=s, dp=dp, scale=np.float64(0.125), p=p, ds=ds)

    # cross-entropy, plain and language-model (shifted targets)
    z = normal(9, (12, 37), 2.0)
    t = O.Random(10).bounded(12, 37).astype(np.int32)
    loss, dz = R.cross_entropy(z, t)
    zl = normal(11, (24, 29), 2.0)
    ids = O.Random(12).bounded(24, 29).astype(np.int32)
    lm_loss, dzl = R.cross_entropy(zl, ids, seq=8)
    save("cross_entropy", logits=z, targets=t, loss=np.float32(loss), dlogits=dz,
         lm_logits=zl, lm_ids=ids, lm_seq=np.int64(8), lm_loss=np.float32(lm_loss), lm_dlogits=dzl)

    # matmul forward/backward (sequential-k fp32 CPU path)
    a = normal(13, (9, 13))
    bm = normal(14, (13, 7), 0.02)
    dc = normal(15, (9, 7))
    c, da, dbm = R.matmul(a, bm, dc)
    save("matmul", a=a, b=bm, dc=dc, c=c, da=da, db=dbm)

    # clip_grad_norm + AdamW, three steps with a fixed gradient
    p0 = normal(16, (257,), 0.02)
    gr = normal(17, (257,), 0.5)
    p3, m3, v3, norm = R.adamw(p0, gr, 3, 3e-4, 0.9, 0.95, 1e-8, 0.1, 1.0)
    save("adamw", p0=p0, g=gr, steps=np.int64(3), p=p3, m=m3, v=v3, norm=np.float64(norm))

    # warmup-cosine schedule
    steps = np.array([0, 1, 50, 99, 100, 101, 450, 998, 999, 1000, 5000], np.uint64)
    lrs = np.array([R.warmup_cosine(3e-4, 3e-5, 100, 900, int(s)) for s in steps])
    save("schedule", steps=steps, lr=lrs)

    # RoPE forward/backward
    xr = normal(18, (2, 8, 16))
    dyr = normal(19, (2, 8, 16))
    out, dxr = R.rope(xr, dyr)
    save("rope", x=xr, dy=dyr, out=out, dx=dxr)

    # A tiny decoder step, full gradients (two micro-batches)
    tiny = {"vocab": 32, "dim": 32, "hidden": 64, "layers": 2, "heads": 2}
    opt = {"beta1": 0.9, "beta2": 0.95, "eps": 1e-8, "weight_decay": 0.1, "max_grad_norm": 1.0}
    names = O.parameter_names(tiny["layers"])
    params = O.init_parameters(tiny, 0x5EED0101)
    ids = O.Random(0x5EED1101).bounded(2 * 2 * 8, 32).reshape(2, 2, 8).astype(np.int32)
    loss, norm, grads, new = R.lm_step(params, names, ids, tiny, 3e-4, opt)
    save("lm_tiny", ids=ids, loss=np.float32(loss), norm=np.float64(norm),
         **{"grad/" + n: grads[n] for n in names}, **{"new/" + n: new[n] for n in names})

    # BASELINE config 1 (2 blocks, d 128, 4 heads, d_ff 512, T 64, V 256, batch 8): loss, norm,
    # per-tensor gradient norms and 64 sampled entries per gradient / updated parameter.
    c1 = {"vocab": 256, "dim": 128, "hidden": 512, "layers": 2, "heads": 4}
    names = O.parameter_names(2)
    params = O.init_parameters(c1, 0x5EED0001)
    ids = O.Random(0x5EED1001).bounded(8 * 64, 256).reshape(1, 8, 64).astype(np.int32)
    loss, norm, grads, new = R.lm_step(params, names, ids, c1, 3e-4, opt)
    samp = {}
    rng = np.random.default_rng(0)
    for n in names:
        idx = rng.choice(grads[n].size, size=min(64, grads[n].size), replace=False)
        samp["idx/" + n] = idx
        samp["grad/" + n] = grads[n].ravel()[idx]
        samp["new/" + n] = new[n].ravel()[idx]
        samp["gnorm/" + n] = np.float64(np.linalg.norm(grads[n].astype(np.float64)))
    save("lm_c1", ids=ids, loss=np.float32(loss), norm=np.float64(norm), **samp)

    save("lm_spar", **spar_family_fixture())


def spar_family_fixture():
    """Spar's own nn::DecoderLM (RMSNorm, grouped-query attention with q/k norms, SwiGLU, no
    biases): one optimiser step of two micro-batches; loss, norm, per-tensor gradient norms and 64
    sampled entries of every gradient / updated parameter."""
    cfg = {"vocab": 64, "dim": 128, "hidden": 256, "layers": 2, "heads": 4, "kv_heads": 2,
           "qk_norm": 1}
    opt = {"beta1": 0.9, "beta2": 0.95, "eps": 1e-8, "weight_decay": 0.1, "max_grad_norm": 1.0}
    names = [n for n, _ in R.spar_param_info(cfg)]
    assert names == list(O.spar_family_shapes(cfg)), names
    params = O.spar_family_parameters(cfg, 0x5EED0301)
    ids = O.Random(0x5EED1301).bounded(2 * 2 * 32, 64).reshape(2, 2, 32).astype(np.int32)
    loss, norm, grads, new = R.spar_lm_step(params, names, ids, cfg, 3e-4, opt)
    samp = {}
    rng = np.random.default_rng(1)
    for n in names:
        idx = rng.choice(grads[n].size, size=min(64, grads[n].size), replace=False)
        samp["idx/" + n] = idx
        samp["grad/" + n] = grads[n].ravel()[idx]
        samp["new/" + n] = new[n].ravel()[idx]
        samp["gnorm/" + n] = np.float64(np.linalg.norm(grads[n].astype(np.float64)))
    return dict(ids=ids, loss=np.float32(loss), norm=np.float64(norm), **samp)


if __name__ == "__main__":
    main(tuple(sys.argv[1:]))
