"""ctypes access to the reference implementation compiled from its own sources
(oracle/_ref/libspar_ref.so, built by oracle/make_ref.py). TEST INFRASTRUCTURE ONLY: used by the
golden-fixture generator, the oracle tests and bench.py's CPU baseline / reference arm.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int64, c_uint64, c_void_p
from pathlib import Path

import numpy as np

REF = Path(__file__).resolve().parent / "_ref"
LIB = REF / "libspar_ref.so"
# Builds of the same reference sources (oracle/make_ref.py): "cpu" the CPU path; "b200" Spar with
# its CUDA backend on libspar_b200.so (the drop-in); "stock" Spar's own CUDA backend + cuBLAS.
VARIANT_LIBS = {"cpu": LIB, "b200": REF / "libspar_ref_b200.so", "stock": REF / "libspar_ref_stock.so"}
_libs: dict = {}

F = POINTER(c_float)
I32 = POINTER(ctypes.c_int32)


def available(variant: str = "cpu") -> bool:
    return VARIANT_LIBS[variant].exists()


def load(variant: str = "cpu"):
    if variant not in _libs:
        path = VARIANT_LIBS[variant]
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (python oracle/make_ref.py)")
        if variant == "b200":  # its spar_cuda_* / spar_b200_* come from the in-tree product build
            import spar_b200._lib as product

            product.load()
        lib = ctypes.CDLL(str(path))
        lib.ref_last_error.restype = c_char_p
        sig = {
            "ref_layernorm": [F, F, F, F, c_int64, c_int64, c_double, F, F, F, F],
            "ref_gelu": [F, F, c_int64, F, F],
            "ref_rmsnorm": [F, F, F, c_int64, c_int64, c_double, F, F, F],
            "ref_swiglu": [F, F, F, c_int64, F, F, F],
            "ref_attention": [F, F, F, F] + [c_int64] * 5 + [F, F, F, F],
            "ref_split_documents": [c_int64, c_int64, c_uint64, POINTER(c_int64)],
            "ref_batches": [c_char_p, POINTER(c_int64), c_int64, c_int64, c_int64, c_int64,
                            c_int64, c_uint64, c_int64, c_int64, I32, POINTER(c_int64), I32,
                            POINTER(c_int64), POINTER(c_int64)],
            "ref_spar_param_info": [c_int64] * 8 + [c_char_p, c_int64, POINTER(c_int64)],
            "ref_spar_ckpt_save": [c_char_p] + [c_int64] * 7 + [c_double] * 3 +
                                  [POINTER(F)] * 3 + [c_uint64] * 4 + [c_double] * 5,
            "ref_spar_ckpt_load": [c_char_p] + [POINTER(F)] * 3 + [POINTER(c_uint64)] * 4 +
                                  [POINTER(c_double)],
            "ref_spar_lm_step": [c_int64] * 10 + [c_double, c_double, POINTER(F), I32, c_double,
                                                  c_double, c_double, c_double, c_double,
                                                  c_double, F, POINTER(c_double), POINTER(F),
                                                  POINTER(F), c_int64],
            "ref_causal_softmax": [F, F, c_int64, c_int64, c_double, F, F],
            "ref_cross_entropy": [F, I32, c_int64, c_int64, c_int64, F, F],
            "ref_matmul": [F, F, F, c_int64, c_int64, c_int64, F, F, F],
            "ref_adamw": [F, F, F, F, c_int64, c_int64, c_double, c_double, c_double, c_double,
                          c_double, c_double, POINTER(c_double)],
            "ref_rope": [F, F, c_int64, c_int64, c_int64, c_double, F, F],
            "ref_lm_step": [c_int64] * 8 + [c_double, c_double, POINTER(F), I32, c_double,
                                            c_double, c_double, c_double, c_double, c_double, F,
                                            POINTER(c_double), POINTER(F), POINTER(F), c_int64],
        }
        for name, args in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = c_int
        lib.ref_warmup_cosine.argtypes = [c_double, c_double, c_uint64, c_uint64, c_uint64]
        lib.ref_warmup_cosine.restype = c_double
        if hasattr(lib, "ref_lm_step_fused"):  # the drop-in build only
            lib.ref_lm_step_fused.argtypes = (
                [c_int64] * 8 + [c_double, c_double, POINTER(F), I32, c_double, c_double, c_double,
                                 c_double, c_double, c_double, F, POINTER(c_double), POINTER(F),
                                 POINTER(F), c_int64, POINTER(c_int64), POINTER(c_double),
                                 POINTER(c_int64)])
            lib.ref_lm_step_fused.restype = c_int
        lib.ref_train_sample_seconds.argtypes = [c_int64] * 6
        lib.ref_train_sample_seconds.restype = c_double
        lib.ref_lm_step_seconds.argtypes = [c_int64] * 10
        lib.ref_lm_step_seconds.restype = c_double
        lib.ref_matmul_seconds.argtypes = [c_int64] * 5
        lib.ref_matmul_seconds.restype = c_double
        _libs[variant] = lib
    return _libs[variant]


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return a.ctypes.data_as(F)


def _check(rc, lib=None):
    if rc != 0:
        raise RuntimeError("reference: " + (lib or load()).ref_last_error().decode())


def layernorm(x, gamma, beta, dy, eps=1e-5):
    x, gamma, beta, dy = map(_f, (x, gamma, beta, dy))
    rows, cols = x.shape
    y, dx = np.empty_like(x), np.empty_like(x)
    dg, db = np.empty(cols, np.float32), np.empty(cols, np.float32)
    _check(load().ref_layernorm(_p(x), _p(gamma), _p(beta), _p(dy), rows, cols, eps, _p(y), _p(dx),
                                _p(dg), _p(db)))
    return y, dx, dg, db


def rmsnorm(x, weight, dy, eps=1e-5):
    x, weight, dy = map(_f, (x, weight, dy))
    rows, cols = x.shape
    y, dx, dw = np.empty_like(x), np.empty_like(x), np.empty(cols, np.float32)
    _check(load().ref_rmsnorm(_p(x), _p(weight), _p(dy), rows, cols, eps, _p(y), _p(dx), _p(dw)))
    return y, dx, dw


def swiglu(gate, value, dh):
    gate, value, dh = map(_f, (gate, value, dh))
    h, dg, dv = np.empty_like(gate), np.empty_like(gate), np.empty_like(gate)
    _check(load().ref_swiglu(_p(gate), _p(value), _p(dh), gate.size, _p(h), _p(dg), _p(dv)))
    return h, dg, dv


def attention(q, k, v, d_out):
    """Causal scaled_dot_product_attention; q [b, h, t, dh], k / v [b, kvh, t, dh]."""
    q, k, v, d_out = map(_f, (q, k, v, d_out))
    b, h, t, dh = q.shape
    kvh = k.shape[1]
    out, dq = np.empty_like(q), np.empty_like(q)
    dk, dv = np.empty_like(k), np.empty_like(v)
    _check(load().ref_attention(_p(q), _p(k), _p(v), _p(d_out), b, h, kvh, t, dh, _p(out), _p(dq),
                                _p(dk), _p(dv)))
    return out, dq, dk, dv


def gelu(x, dy):
    x, dy = _f(x).ravel(), _f(dy).ravel()
    y, dx = np.empty_like(x), np.empty_like(x)
    _check(load().ref_gelu(_p(x), _p(dy), x.size, _p(y), _p(dx)))
    return y, dx


def causal_softmax(s, dp, scale):
    s, dp = _f(s), _f(dp)
    b, t, _ = s.shape
    p, ds = np.empty_like(s), np.empty_like(s)
    _check(load().ref_causal_softmax(_p(s), _p(dp), b, t, scale, _p(p), _p(ds)))
    return p, ds


def cross_entropy(logits, targets, seq=0):
    z = _f(logits)
    rows, classes = z.shape
    tg = np.ascontiguousarray(targets, dtype=np.int32)
    loss = np.zeros(1, np.float32)
    dz = np.empty_like(z)
    _check(load().ref_cross_entropy(_p(z), tg.ctypes.data_as(I32), rows, classes, seq, _p(loss), _p(dz)))
    return float(loss[0]), dz


def matmul(a, b, dc):
    a, b, dc = map(_f, (a, b, dc))
    m, k = a.shape
    n = b.shape[1]
    c, da, db = np.empty((m, n), np.float32), np.empty_like(a), np.empty_like(b)
    _check(load().ref_matmul(_p(a), _p(b), _p(dc), m, k, n, _p(c), _p(da), _p(db)))
    return c, da, db


def adamw(p, g, steps, lr, beta1, beta2, eps, wd, max_norm):
    p, g = _f(p).copy(), _f(g)
    m, v = np.empty_like(p), np.empty_like(p)
    norm = c_double(0.0)
    _check(load().ref_adamw(_p(p), _p(g), _p(m), _p(v), p.size, steps, lr, beta1, beta2, eps, wd,
                            max_norm, ctypes.byref(norm)))
    return p, m, v, norm.value


def warmup_cosine(peak, minimum, warmup, decay, step):
    return load().ref_warmup_cosine(peak, minimum, warmup, decay, step)


def rope(x, dy, theta=10000.0):
    x, dy = _f(x), _f(dy)
    outer, t, d = x.shape
    out, dx = np.empty_like(x), np.empty_like(x)
    _check(load().ref_rope(_p(x), _p(dy), outer, t, d, theta, _p(out), _p(dx)))
    return out, dx


def lm_step(params: dict, names, ids, cfg: dict, lr, opt: dict, device: int = -1,
            variant: str = "cpu"):
    """One reference training step; ids [micro, batch, t]. Returns (loss, norm, grads, new).
    device >= 0 runs it on that CUDA device (variants "b200" / "stock")."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    micro, batch, t = ids.shape
    ps = [_f(params[n]) for n in names]
    gs = [np.empty_like(p) for p in ps]
    outs = [np.empty_like(p) for p in ps]
    arr = lambda lst: (F * len(lst))(*[_p(a) for a in lst])
    loss = np.zeros(1, np.float32)
    norm = c_double(0.0)
    lib = load(variant)
    _check(lib.ref_lm_step(cfg["vocab"], cfg["dim"], cfg["hidden"], cfg["layers"], cfg["heads"],
                           batch, t, micro, cfg.get("eps", 1e-5), cfg.get("rope_theta", 1e4),
                           arr(ps), ids.ctypes.data_as(I32), lr, opt["beta1"], opt["beta2"],
                           opt["eps"], opt["weight_decay"], opt["max_grad_norm"], _p(loss),
                           ctypes.byref(norm), arr(gs), arr(outs), device), lib)
    return float(loss[0]), norm.value, dict(zip(names, gs)), dict(zip(names, outs))


def lm_step_fused(params: dict, names, ids, cfg: dict, lr, opt: dict, device: int = 0):
    """ref_lm_step with the product's fused operations recorded on Spar's tape (drop-in build):
    (loss, norm, grads, new, hook_calls, hook_norms, hook_order) for the grad_ready slots (per
    block: ln1 gain, ln2 gain, up-projection weight)."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    micro, batch, t = ids.shape
    ps = [_f(params[n]) for n in names]
    gs = [np.empty_like(p) for p in ps]
    outs = [np.empty_like(p) for p in ps]
    arr = lambda lst: (F * len(lst))(*[_p(a) for a in lst])
    loss = np.zeros(1, np.float32)
    norm = c_double(0.0)
    slots = 3 * cfg["layers"]
    calls = np.zeros(slots, np.int64)
    norms = np.zeros(slots, np.float64)
    order = np.full(slots * micro, -1, np.int64)
    lib = load("b200")
    _check(lib.ref_lm_step_fused(cfg["vocab"], cfg["dim"], cfg["hidden"], cfg["layers"],
                                 cfg["heads"], batch, t, micro, cfg.get("eps", 1e-5),
                                 cfg.get("rope_theta", 1e4), arr(ps), ids.ctypes.data_as(I32), lr,
                                 opt["beta1"], opt["beta2"], opt["eps"], opt["weight_decay"],
                                 opt["max_grad_norm"], _p(loss), ctypes.byref(norm), arr(gs),
                                 arr(outs), device, calls.ctypes.data_as(POINTER(c_int64)),
                                 norms.ctypes.data_as(POINTER(c_double)),
                                 order.ctypes.data_as(POINTER(c_int64))), lib)
    return (float(loss[0]), norm.value, dict(zip(names, gs)), dict(zip(names, outs)), calls, norms,
            order)


def _spar_dims(cfg):
    return (cfg["vocab"], cfg["dim"], cfg["hidden"], cfg["layers"], cfg["heads"],
            cfg.get("kv_heads", cfg["heads"]), int(cfg.get("qk_norm", 0)))


def spar_param_info(cfg: dict):
    """[(name, numel)] of nn::DecoderLM's named_parameters for cfg (the reference's own order)."""
    lib = load()
    n = c_int64(0)
    buf = ctypes.create_string_buffer(256)
    _check(lib.ref_spar_param_info(*_spar_dims(cfg), -1, buf, 256, ctypes.byref(n)))
    out = []
    for i in range(n.value):
        k = c_int64(0)
        _check(lib.ref_spar_param_info(*_spar_dims(cfg), i, buf, 256, ctypes.byref(k)))
        out.append((buf.value.decode(), k.value))
    return out


def spar_lm_step(params: dict, names, ids, cfg: dict, lr, opt: dict, device: int = -1,
                 variant: str = "cpu"):
    """One training step of the reference's nn::DecoderLM; ids [micro, batch, t].
    Returns (loss, norm, grads, new) keyed by the reference's parameter names. device >= 0 runs
    it on that CUDA device (variants "b200" / "stock")."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    micro, batch, t = ids.shape
    ps = [_f(params[n]) for n in names]
    gs = [np.empty_like(p) for p in ps]
    outs = [np.empty_like(p) for p in ps]
    arr = lambda lst: (F * len(lst))(*[_p(a) for a in lst])
    loss = np.zeros(1, np.float32)
    norm = c_double(0.0)
    lib = load(variant)
    _check(lib.ref_spar_lm_step(*_spar_dims(cfg), batch, t, micro, cfg.get("eps", 1e-5),
                                cfg.get("rope_theta", 1e4), arr(ps), ids.ctypes.data_as(I32),
                                lr, opt["beta1"], opt["beta2"], opt["eps"],
                                opt["weight_decay"], opt["max_grad_norm"], _p(loss),
                                ctypes.byref(norm), arr(gs), arr(outs), device), lib)
    return float(loss[0]), norm.value, dict(zip(names, gs)), dict(zip(names, outs))


def spar_ckpt_save(path, cfg: dict, params: list, m: list, v: list, adam_step: int,
                   global_step: int, tokens: int, rng_state: int, lr: float, opt: dict):
    """checkpoint::save_training_checkpoint of the reference's nn::DecoderLM (params / m / v in
    named-parameter order)."""
    arr = lambda lst: (F * len(lst))(*[_p(_f(a)) for a in lst])
    keep = [_f(a) for a in params + m + v]  # noqa: F841 - alive during the call
    _check(load().ref_spar_ckpt_save(str(path).encode(), *_spar_dims(cfg), cfg.get("eps", 1e-5),
                                     cfg.get("rope_theta", 1e4), cfg.get("qk_eps", 1e-6),
                                     arr(params), arr(m), arr(v), adam_step, global_step, tokens,
                                     rng_state, lr, opt["beta1"], opt["beta2"], opt["eps"],
                                     opt["weight_decay"]))


def spar_ckpt_load(path, cfg: dict):
    """checkpoint::load_training_checkpoint: (params, m, v, adam_step, global_step, tokens,
    rng_state, lr) with arrays in named-parameter order."""
    sizes = [k for _, k in spar_param_info(cfg)]
    ps = [np.empty(k, np.float32) for k in sizes]
    ms = [np.empty(k, np.float32) for k in sizes]
    vs = [np.empty(k, np.float32) for k in sizes]
    arr = lambda lst: (F * len(lst))(*[_p(a) for a in lst])
    u = [c_uint64() for _ in range(4)]
    lr = c_double()
    _check(load().ref_spar_ckpt_load(str(path).encode(), arr(ps), arr(ms), arr(vs),
                                     *[ctypes.byref(x) for x in u], ctypes.byref(lr)))
    return ps, ms, vs, u[0].value, u[1].value, u[2].value, u[3].value, lr.value


def split_documents(count: int, validation: int, seed: int):
    """The reference's data::split_documents: (train indices, validation indices)."""
    out = np.empty(max(count, 1), np.int64)
    _check(load().ref_split_documents(count, validation, seed,
                                      out.ctypes.data_as(POINTER(c_int64))))
    return out[validation:count], out[:validation]


def batches(documents: list, seq: int, stride: int, batch: int, shuffle: bool, seed: int,
            drop_last: bool, epochs: int):
    """The reference's LMBatchIterator over its byte-level TokenizedCorpus of `documents`
    (bytes): (corpus tokens int32, [batch arrays [rows, seq] int32 in order])."""
    blob = b"".join(documents)
    lens = (c_int64 * len(documents))(*[len(d) for d in documents])
    ntok = len(blob) + len(documents)
    windows = max(0, 1 + (ntok - seq) // stride) if ntok >= seq else 0
    toks = np.empty(ntok, np.int32)
    out = np.empty((max(1, windows * epochs), seq), np.int32)
    rows = np.empty(max(1, windows * epochs), np.int64)
    tc, nb = c_int64(), c_int64()
    _check(load().ref_batches(blob, lens, len(documents), seq, stride, batch, int(shuffle), seed,
                              int(drop_last), epochs, toks.ctypes.data_as(I32), ctypes.byref(tc),
                              out.ctypes.data_as(I32), rows.ctypes.data_as(POINTER(c_int64)),
                              ctypes.byref(nb)))
    res, r0 = [], 0
    for k in range(nb.value):
        res.append(out[r0:r0 + rows[k]].copy())
        r0 += rows[k]
    return toks[:tc.value], res


def _sample_worker(args):
    vocab, d, f, heads, t, iters = args
    return load().ref_train_sample_seconds(vocab, d, f, heads, t, iters)


def lm_step_seconds(cfg, batch: int, warmup: int, iters: int, device: int = 0,
                    variant: str = "stock") -> float:
    """Seconds per full training step of the LN/GELU decoder `cfg` (an LMConfig) on [batch, seq]
    ids through the given build's backend (default: the reference's own CUDA path)."""
    v = load(variant).ref_lm_step_seconds(cfg.vocab, cfg.dim, cfg.hidden, cfg.layers, cfg.heads,
                                          batch, cfg.seq, warmup, iters, device)
    if v <= 0:
        _check(1, load(variant))
    return v


def matmul_seconds(m: int, k: int, n: int, iters: int, device: int = 0,
                   variant: str = "stock") -> float:
    """Seconds per Spar matmul [m, k] x [k, n] (fp32) through the given build's cuda_blas seam."""
    v = load(variant).ref_matmul_seconds(m, k, n, iters, device)
    if v <= 0:
        _check(1, load(variant))
    return v


def default_processes() -> int:
    """All host cores, capped so the concurrent samples (~1.5 GB each at config 5) fit in RAM."""
    n = os.cpu_count() or 1
    try:
        import psutil

        n = min(n, max(1, int(psutil.virtual_memory().available / 1.5e9)))
    except ImportError:
        pass
    return max(1, n)


def run_reference_sample(cfg, seconds_budget: float = 20.0, processes: int = 1, t: int = 2):
    """Times the reference CPU training step on a bounded sample of `cfg`'s workload: one block
    with cfg's d_model / heads / d_ff / vocab on a short sequence (forward, LM loss, backward,
    clip, AdamW), in `processes` concurrent single-threaded processes (the reference has no
    threading). Its FLOP rate is converted to tokens/s of the full configuration with the per-token
    FLOPs (6 x matmul params + 12 L d T attention). t=2 tokens keeps one sample near 15 s at
    config 5's dimensions."""
    per_token_sample = 6.0 * (4 * cfg.dim ** 2 + 2 * cfg.dim * cfg.hidden + cfg.vocab * cfg.dim) \
        + 12.0 * cfg.dim * t
    args = (cfg.vocab, cfg.dim, cfg.hidden, cfg.heads, t, 1)
    if processes <= 1:
        secs = [_sample_worker(args)]
    else:
        import multiprocessing as mp

        with mp.get_context("spawn").Pool(processes) as pool:
            secs = pool.map(_sample_worker, [args] * processes)
    if min(secs) <= 0:
        raise RuntimeError("reference sample failed")
    rate = sum(per_token_sample * t / s for s in secs)  # FLOP/s over all processes
    tokens_per_s = rate / cfg.flops_per_token()
    return {"tokens_per_s": tokens_per_s, "cores": processes, "kind": "reference",
            "sample": (f"{processes}x one training step (fwd+loss+bwd+clip+AdamW) of a 1-block "
                       f"decoder d={cfg.dim} H={cfg.heads} F={cfg.hidden} V={cfg.vocab} on 1x{t} "
                       f"tokens, {max(secs):.1f} s; FLOP rate extrapolated to the full step by "
                       f"{cfg.flops_per_token() / 1e9:.3f} GFLOP/token"),
            "seconds": secs}


_ = (c_void_p, os)
