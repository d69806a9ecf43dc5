"""Host-side handle for the decoder training runtime in libspar_b200.so.

Mirrors the reference's model/optimiser surface for this path: parameters are addressed by Spar's
named_parameters names (src/nn/parameters.cpp:51-132), weights are [in, out] as in nn::Linear
(src/nn/linear.cpp:33-35), and a training step is forward -> LM cross-entropy -> backward ->
clip_grad_norm -> AdamW (src/training/gradients.cpp:176-190, src/optim/adamw.cpp:83-170) with the
learning rate from warmup_cosine_learning_rate (src/training/schedule.cpp:9-38). Errors raise
SparError with the reference's status codes.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import SparB200LMConfig, SparError, check

WHICH = {"param": 0, "grad": 1, "m": 2, "v": 3}


@dataclass
class LMConfig:
    vocab: int
    dim: int
    hidden: int
    layers: int
    heads: int
    seq: int
    micro_batch: int
    eps: float = 1e-5
    rope_theta: float = 10000.0
    use_rope: bool = True
    precision: int = 0  # 0 TF32, 1 3xTF32
    beta1: float = 0.9
    beta2: float = 0.95
    adam_eps: float = 1e-8
    weight_decay: float = 0.1
    max_grad_norm: float = 1.0
    family: int = 0  # 0: LayerNorm / GELU benchmark decoder, 1: Spar's nn::DecoderLM
    kv_heads: int = 0  # family 1: key/value heads (0 = heads)
    qk_norm: bool = False  # family 1
    qk_eps: float = 1e-6  # family 1

    def oracle_dict(self):
        return {"vocab": self.vocab, "dim": self.dim, "hidden": self.hidden, "layers": self.layers,
                "heads": self.heads, "eps": self.eps, "rope_theta": self.rope_theta}

    def opt_dict(self):
        return {"beta1": self.beta1, "beta2": self.beta2, "eps": self.adam_eps,
                "weight_decay": self.weight_decay, "max_grad_norm": self.max_grad_norm}

    def flops_per_token(self) -> float:
        """6 * matmul params + attention (12 * L * d * T, half of it under the causal mask is
        skipped by the kernels but counted here as the standard estimate)."""
        if self.family == 1:  # q | k | v with kv_heads, out, gate | up | down
            kvh = self.kv_heads or self.heads
            qkv = self.dim * (self.dim + 2 * kvh * (self.dim // self.heads))
            per_layer = qkv + self.dim * self.dim + 3 * self.dim * self.hidden
        else:
            per_layer = 4 * self.dim * self.dim + 2 * self.dim * self.hidden
        n_mm = self.layers * per_layer + self.vocab * self.dim
        return 6.0 * n_mm + 12.0 * self.layers * self.dim * self.seq


def native_config(cfg: LMConfig) -> SparB200LMConfig:
    """The C-ABI config struct of a model config."""
    return SparB200LMConfig(cfg.vocab, cfg.dim, cfg.hidden, cfg.layers, cfg.heads, cfg.seq,
                            cfg.micro_batch, cfg.eps, cfg.rope_theta, int(cfg.use_rope),
                            cfg.precision, cfg.beta1, cfg.beta2, cfg.adam_eps, cfg.weight_decay,
                            cfg.max_grad_norm, cfg.family, int(cfg.qk_norm), cfg.kv_heads,
                            cfg.qk_eps)


class DecoderLM:
    """One decoder + optimiser state resident on one GPU."""

    def __init__(self, cfg: LMConfig, device: int = 0):
        self.cfg = cfg
        self.device = device
        self.lib = _lib.load()
        c = native_config(cfg)
        h = ctypes.c_void_p()
        check("spar_b200_lm_create", self.lib.spar_b200_lm_create(ctypes.byref(c), device,
                                                                  ctypes.byref(h)))
        self.handle = h
        self.names = []
        self.shapes = {}
        buf = ctypes.create_string_buffer(256)
        for i in range(self.lib.spar_b200_lm_parameter_count(h)):
            r, col = ctypes.c_uint64(), ctypes.c_uint64()
            check("spar_b200_lm_parameter_info",
                  self.lib.spar_b200_lm_parameter_info(h, i, buf, 256, ctypes.byref(r), ctypes.byref(col)))
            name = buf.value.decode()
            self.names.append(name)
            self.shapes[name] = (r.value, col.value) if col.value else (r.value,)
        self.index = {n: i for i, n in enumerate(self.names)}
        self.step_count = 0

    def close(self):
        if self.handle:
            self.lib.spar_b200_lm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------ parameters
    def set(self, name: str, value, which: str = "param"):
        a = np.ascontiguousarray(value, dtype=np.float32)
        if a.shape != self.shapes[name]:
            raise ValueError(f"{name}: shape {a.shape} != {self.shapes[name]}")
        check("spar_b200_lm_parameter_copy",
              self.lib.spar_b200_lm_parameter_copy(self.handle, self.index[name], WHICH[which], 1,
                                                   a.ctypes.data))

    def get(self, name: str, which: str = "param") -> np.ndarray:
        a = np.empty(self.shapes[name], dtype=np.float32)
        check("spar_b200_lm_parameter_copy",
              self.lib.spar_b200_lm_parameter_copy(self.handle, self.index[name], WHICH[which], 0,
                                                   a.ctypes.data))
        return a

    def load_state_dict(self, params: dict):
        """nn::load_state_dict equivalent (src/nn/state.cpp:22-54): every name must be present."""
        missing = set(self.names) - set(params)
        if missing:
            raise KeyError(f"missing parameters: {sorted(missing)[:5]}")
        for n in self.names:
            self.set(n, params[n])

    def state_dict(self, which: str = "param") -> dict:
        return {n: self.get(n, which) for n in self.names}

    def init_normal(self, seed: int, std: float = 0.02, stream: int = 0):
        check("spar_b200_lm_init_normal", self.lib.spar_b200_lm_init_normal(self.handle, seed, std, stream))

    def flat_size(self) -> int:
        return self.lib.spar_b200_lm_flat_size(self.handle)

    def flat_buffer(self, which: str = "grad") -> int:
        return self.lib.spar_b200_lm_flat_buffer(self.handle, WHICH[which])

    def profile(self, enable: bool):
        check("spar_b200_lm_profile", self.lib.spar_b200_lm_profile(self.handle, int(enable)))

    def profile_read(self):
        """(gemm_ms, gemm_flops, gemm_launches, kernel_launches) since profiling was enabled."""
        ms, fl = ctypes.c_double(), ctypes.c_double()
        gl, kl = ctypes.c_uint64(), ctypes.c_uint64()
        check("spar_b200_lm_profile_read",
              self.lib.spar_b200_lm_profile_read(self.handle, ctypes.byref(ms), ctypes.byref(fl),
                                                 ctypes.byref(gl), ctypes.byref(kl)))
        return ms.value, fl.value, gl.value, kl.value

    # ------------------------------------------------------------------ training
    def attach_comm(self, comm, world_size: int):
        check("spar_b200_lm_set_comm", self.lib.spar_b200_lm_set_comm(self.handle, comm, world_size))

    def save_checkpoint(self, path, global_step: int, tokens_seen: int, rng_state: int,
                        learning_rate: float, adam_step: int):
        """SPARCKPT v1 training checkpoint (Spar-family models; collective with a sharded
        optimiser: every rank calls it, path None on ranks that only take part in the gather)."""
        meta = _lib.SparB200Checkpoint(global_step, tokens_seen, rng_state, learning_rate, adam_step)
        check("spar_b200_lm_save_checkpoint", self.lib.spar_b200_lm_save_checkpoint(
            self.handle, None if path is None else str(path).encode(), ctypes.byref(meta)))

    def load_checkpoint(self, path) -> dict:
        """Loads parameters and AdamW moments; returns the progress fields (adam_step: the
        next train_step is step adam_step + 1)."""
        meta = _lib.SparB200Checkpoint()
        check("spar_b200_lm_load_checkpoint", self.lib.spar_b200_lm_load_checkpoint(
            self.handle, str(path).encode(), ctypes.byref(meta)))
        return {k: getattr(meta, k) for k, _ in meta._fields_}

    def gather(self, which: str = "param", stream: int = 0):
        """Sharded optimiser: all-gathers one arena's pieces from every rank so that it can be read
        (get / state_dict). Collective: every rank calls it, in the same order."""
        check("spar_b200_lm_gather", self.lib.spar_b200_lm_gather(self.handle, WHICH[which], stream))

    def train_step(self, ids, lr: float, step: int | None = None, stream: int = 0):
        """ids: int32 array [micro_steps, micro_batch, seq] in host memory (numpy or pinned
        torch tensor), or a CUDA int32 tensor of that shape. Returns (loss, grad_norm, flags)."""
        if step is None:
            step = self.step_count + 1
        on_host = 1
        if hasattr(ids, "is_cuda"):
            on_host = 0 if ids.is_cuda else 1
            ptr = ids.data_ptr()
            micro = ids.shape[0]
            if ids.dtype.__repr__() != "torch.int32":
                raise ValueError("ids must be int32")
        else:
            ids = np.ascontiguousarray(ids, dtype=np.int32)
            ptr = ids.ctypes.data
            micro = ids.shape[0]
        loss = ctypes.c_float()
        norm = ctypes.c_double()
        flags = (ctypes.c_int32 * 2)()
        check("spar_b200_lm_train_step",
              self.lib.spar_b200_lm_train_step(self.handle, ptr, on_host, micro, lr, step,
                                               ctypes.byref(loss), ctypes.byref(norm), flags, stream))
        self.step_count = step
        return loss.value, norm.value, (flags[0], flags[1])


def write_checkpoint(path, cfg: LMConfig, values: list, first_moments: list | None,
                     second_moments: list | None, global_step: int = 0, tokens_seen: int = 0,
                     rng_state: int = 0, learning_rate: float = 0.0, adam_step: int = 0):
    """SPARCKPT v1 from host arrays (one per named tensor, layout order), no GPU needed."""
    lib = _lib.load()
    c = native_config(cfg)
    meta = _lib.SparB200Checkpoint(global_step, tokens_seen, rng_state, learning_rate, adam_step)
    keep = [np.ascontiguousarray(a, np.float32) for a in values]
    arr = lambda lst: (ctypes.c_void_p * len(lst))(*[a.ctypes.data for a in lst])  # noqa: E731
    km = [np.ascontiguousarray(a, np.float32) for a in (first_moments or [])]
    kv = [np.ascontiguousarray(a, np.float32) for a in (second_moments or [])]
    check("spar_b200_checkpoint_write",
          lib.spar_b200_checkpoint_write(str(path).encode(), ctypes.byref(c), ctypes.byref(meta),
                                         arr(keep), arr(km) if km else None,
                                         arr(kv) if kv else None))


def read_checkpoint(path, cfg: LMConfig, sizes: list):
    """(values, first moments, second moments, meta dict) of a SPARCKPT v1 file for cfg;
    sizes: element counts of the named tensors in layout order."""
    lib = _lib.load()
    c = native_config(cfg)
    meta = _lib.SparB200Checkpoint()
    vals, ms, vs = ([np.empty(k, np.float32) for k in sizes] for _ in range(3))
    arr = lambda lst: (ctypes.c_void_p * len(lst))(*[a.ctypes.data for a in lst])  # noqa: E731
    check("spar_b200_checkpoint_read",
          lib.spar_b200_checkpoint_read(str(path).encode(), ctypes.byref(c), ctypes.byref(meta),
                                        arr(vals), arr(ms), arr(vs)))
    return vals, ms, vs, {k: getattr(meta, k) for k, _ in meta._fields_}


def warmup_cosine(peak: float, minimum: float, warmup: int, decay: int, step: int) -> float:
    v = _lib.load().spar_b200_warmup_cosine(peak, minimum, warmup, decay, step)
    if v != v:
        raise ValueError("invalid warmup-cosine configuration")
    return v


C1 = LMConfig(vocab=256, dim=128, hidden=512, layers=2, heads=4, seq=64, micro_batch=8)
C4 = LMConfig(vocab=50257, dim=768, hidden=3072, layers=12, heads=12, seq=1024, micro_batch=8)
C5 = LMConfig(vocab=32768, dim=1024, hidden=4096, layers=24, heads=16, seq=1024, micro_batch=16)


def smoke_step(device) -> None:
    """One tiny training step on `device` (the flagship path end to end); raises on failure."""
    import torch

    cfg = LMConfig(vocab=256, dim=128, hidden=256, layers=1, heads=4, seq=32, micro_batch=2)
    lm = DecoderLM(cfg, device.index or 0)
    lm.init_normal(1234)
    rng = np.random.default_rng(0)
    ids = rng.integers(0, cfg.vocab, (1, cfg.micro_batch, cfg.seq)).astype(np.int32)
    loss, norm, flags = lm.train_step(ids, 3e-4)
    torch.cuda.synchronize()
    if not (np.isfinite(loss) and np.isfinite(norm)) or flags != (0, 0):
        raise SparError("smoke", _lib.SparCudaStatus(2, 0))
    lm.close()


def _measure(cfg: "LMConfig", micro: int, steps: int, warmup: int, precision: int) -> None:
    """Tokens/s of `steps` graph-replayed training steps of `cfg` (after `warmup` steps), timed
    with CUDA events on the step's stream; one JSON line."""
    import json
    from dataclasses import replace

    import torch

    cfg = replace(cfg, precision=precision)
    lm = DecoderLM(cfg, 0)
    lm.init_normal(0x5EED0000 + cfg.dim, 0.02)
    rng = np.random.default_rng(cfg.vocab)
    ids = torch.from_numpy(rng.integers(0, cfg.vocab, (micro, cfg.micro_batch, cfg.seq))
                           .astype(np.int32)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for s in range(warmup):
        lm.train_step(ids, 3e-4, step=s + 1, stream=stream)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for s in range(steps):
        _, _, flags = lm.train_step(ids, 3e-4, step=warmup + s + 1, stream=stream)
    b.record()
    torch.cuda.synchronize()
    lm.close()
    ms = a.elapsed_time(b) / steps
    tokens = micro * cfg.micro_batch * cfg.seq
    print(json.dumps({"config": {"vocab": cfg.vocab, "dim": cfg.dim, "layers": cfg.layers,
                                 "heads": cfg.heads, "seq": cfg.seq, "micro_batch": cfg.micro_batch,
                                 "micro_steps": micro},
                      "precision": "tf32x3" if precision else "tf32", "ms_per_step": round(ms, 3),
                      "tokens_per_s": round(tokens / ms * 1e3, 1),
                      "model_tflops": round(tokens * cfg.flops_per_token() / ms / 1e9, 1),
                      "flags": list(flags)}), flush=True)


def _main() -> None:
    """`python -m spar_b200.lm --micro-batch MB --steps S [--family spar --kv-heads K --qk-norm]`:
    S training steps of the C5 decoder (or, with --family spar, Spar's own nn::DecoderLM at the C5
    dimensions: RMSNorm, K key/value heads, SwiGLU with the same hidden size) on one GPU, with
    rank 0's share of the 64-sequence global batch for 16 / MB ranks (4 accumulation micro-steps
    of MB sequences), synthetic weights and ids; prints the loss and step time.

    `python -m spar_b200.lm --config c1|c4 [--precision tf32x3] [--steps S]`: the step rate of the
    C1 tiny model (batch 8 x 64 tokens) or the C4 GPT-2-small-shaped model (batch 8 x 1024 tokens,
    vocabulary 50257), one micro-step per optimiser step, timed on the device."""
    import argparse
    import time
    from dataclasses import replace

    import torch

    from .data import rank_share

    ap = argparse.ArgumentParser()
    ap.add_argument("--micro-batch", type=int, default=16, choices=[1, 2, 4, 8, 16])
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--family", default="ln", choices=["ln", "spar"])
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--qk-norm", action="store_true")
    ap.add_argument("--config", default="c5", choices=["c1", "c4", "c5"])
    ap.add_argument("--precision", default="tf32", choices=["tf32", "tf32x3"])
    a = ap.parse_args()
    if a.config != "c5":
        _measure(C1 if a.config == "c1" else C4, 1, max(a.steps, 5), 3,
                 1 if a.precision == "tf32x3" else 0)
        return
    cfg = replace(C5, micro_batch=a.micro_batch)
    if a.family == "spar":
        cfg = replace(cfg, family=1, kv_heads=a.kv_heads, qk_norm=a.qk_norm)
    if a.precision == "tf32x3":
        cfg = replace(cfg, precision=1)
    lm = DecoderLM(cfg, 0)
    lm.init_normal(0x5EED0005, 0.02)
    ids = torch.from_numpy(rank_share(0x5EED1005, 64, 4, cfg.seq, cfg.vocab, 0,
                                      16 // a.micro_batch)).cuda()
    tokens = ids.numel()
    for s in range(a.steps):
        t0 = time.perf_counter()
        loss, norm, flags = lm.train_step(ids, 3e-4, step=s + 1)
        torch.cuda.synchronize()
        ms = (time.perf_counter() - t0) * 1e3
        print(f"step {s + 1}: loss {loss:.4f} grad-norm {norm:.4f} flags {flags} {ms:.1f} ms "
              f"({tokens / ms * 1e3:.0f} tokens/s)", flush=True)
    lm.close()


if __name__ == "__main__":
    _main()
