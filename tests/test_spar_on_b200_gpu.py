"""Spar's own code running on Device::cuda through libspar_b200.

oracle/make_ref.py (variant "b200") builds the reference's sources as a Spar build that adopts the
drop-in would: SPAR_ENABLE_CUDA=1, src/backend/cuda_kernels.cu left out and libspar_b200.so
linked in its place (its spar_cuda_* entry points serve src/backend/cuda_ops.cppm unchanged), and
spar_b200/spar/cuda_blas.cppm compiled in place of src/backend/cuda_blas.cppm (every matmul on the
tcgen05 GEMM). A training step of the reference's own nn::DecoderLM (src/nn/decoder.cpp:73-90:
RMSNorm, grouped-query attention with q/k norms, RoPE, SwiGLU, tied logits), and of the LN/GELU
decoder composed from Spar ops, then runs on cuda:0 through Spar's autograd, loss, clip and
AdamW, and is compared with the same library's CPU step on the same weights and ids.

Bars: matmuls in 3xTF32 (the seam's default): loss, norm and every gradient within 1e-5 relative
L2 of the CPU step; in TF32 (SPAR_B200_MATMUL_PRECISION=tf32): 3e-3 overall and 1e-2 per tensor
(the grouped-query bars of the runtime's own Spar-family tests). The update is compared where the
CPU gradient is well conditioned (|g| >= 5 % of the tensor's RMS; at step 1 AdamW's update is
lr * sign(g) elsewhere, which only tests the sign of near-zero gradients).
"""
import ctypes

import numpy as np
import pytest

from _util import rel_l2
from oracle import spar_oracle as O

pytestmark = pytest.mark.gpu

OPT = {"beta1": 0.9, "beta2": 0.95, "eps": 1e-8, "weight_decay": 0.1, "max_grad_norm": 1.0}


@pytest.fixture(scope="module")
def ref(cuda):
    from oracle import cpu_ref

    if not cpu_ref.available("b200"):
        pytest.skip("Spar drop-in build absent (python oracle/make_ref.py --variant b200)")
    return cpu_ref


def _flat(d, names):
    return np.concatenate([np.asarray(d[n], np.float64).ravel() for n in names])


def _compare(cpu, gpu, params, names, tol_all, tol_each):
    (l0, n0, g0, p0), (l1, n1, g1, p1) = cpu, gpu
    assert abs(l1 - l0) <= tol_all * abs(l0)
    assert abs(n1 - n0) <= tol_all * n0
    assert rel_l2(_flat(g1, names), _flat(g0, names)) <= tol_all
    for n in names:
        assert rel_l2(g1[n], g0[n]) <= tol_each, (n, rel_l2(g1[n], g0[n]))
        g = np.asarray(g0[n], np.float64)
        mask = np.abs(g) >= 0.05 * np.sqrt(np.mean(g * g))
        d0 = p0[n].astype(np.float64) - params[n]
        d1 = p1[n].astype(np.float64) - params[n]
        assert rel_l2(d1[mask], d0[mask]) <= tol_each, n


def test_backend_symbols_come_from_libspar_b200(ref):
    """The drop-in build defines no spar_cuda_* itself: each resolves into libspar_b200.so."""
    lib = ref.load("b200")

    class DlInfo(ctypes.Structure):
        _fields_ = [("dli_fname", ctypes.c_char_p), ("dli_fbase", ctypes.c_void_p),
                    ("dli_sname", ctypes.c_char_p), ("dli_saddr", ctypes.c_void_p)]

    libc = ctypes.CDLL(None)
    for name in ("spar_cuda_launch_binary", "spar_cuda_launch_adamw", "spar_b200_matmul"):
        info = DlInfo()
        addr = ctypes.cast(getattr(lib, name), ctypes.c_void_p)
        assert libc.dladdr(addr, ctypes.byref(info)) != 0
        assert info.dli_fname.decode().endswith("spar_b200/libspar_b200.so"), name


@pytest.mark.parametrize("precision,tol_all,tol_each", [("tf32x3", 1e-5, 1e-5),
                                                        ("tf32", 3e-3, 1e-2)])
def test_spar_decoder_step_on_cuda_matches_cpu(ref, monkeypatch, precision, tol_all, tol_each):
    monkeypatch.setenv("SPAR_B200_MATMUL_PRECISION", precision)
    cfg = dict(vocab=96, dim=128, hidden=256, layers=2, heads=4, kv_heads=2, qk_norm=1)
    params = O.spar_family_parameters(cfg, 0x5EED0701)
    names = [n for n, _ in ref.spar_param_info(cfg)]
    shaped = {n: params[n] for n in names}
    ids = O.Random(0x5EED1701).bounded(2 * 2 * 48, 96).reshape(2, 2, 48).astype(np.int32)
    cpu = ref.spar_lm_step(shaped, names, ids, cfg, 3e-4, OPT, device=-1, variant="b200")
    gpu = ref.spar_lm_step(shaped, names, ids, cfg, 3e-4, OPT, device=0, variant="b200")
    _compare(cpu, gpu, shaped, names, tol_all, tol_each)


@pytest.mark.parametrize("precision,tol_all,tol_each", [("tf32x3", 1e-5, 1e-5),
                                                        ("tf32", 2e-3, 1e-2)])
def test_ln_gelu_decoder_step_on_cuda_matches_cpu(ref, monkeypatch, precision, tol_all, tol_each):
    """The LN/GELU decoder composed from Spar ops (LayerNorm from mean / subtract / square /
    add_scalar / sqrt / divide / multiply / add; GELU through sigmoid), Spar's SelfAttention with
    biases and RoPE, Linear, Embedding, LM cross-entropy, clip and AdamW."""
    monkeypatch.setenv("SPAR_B200_MATMUL_PRECISION", precision)
    cfg = {"vocab": 256, "dim": 128, "hidden": 512, "layers": 2, "heads": 4, "eps": 1e-5,
           "rope_theta": 1e4}
    params = O.init_parameters(cfg, 0x5EED0801)
    r = np.random.default_rng(8)
    for n, v in params.items():  # non-trivial biases and LayerNorm parameters
        if v.ndim == 1:
            params[n] = ((1.0 if n.endswith("norm.weight") else 0.0)
                         + 0.05 * r.standard_normal(v.shape)).astype(np.float32)
    names = O.parameter_names(cfg["layers"])
    ids = O.Random(0x5EED1801).bounded(2 * 4 * 64, 256).reshape(2, 4, 64).astype(np.int32)
    cpu = ref.lm_step(params, names, ids, cfg, 3e-4, OPT, device=-1, variant="b200")
    gpu = ref.lm_step(params, names, ids, cfg, 3e-4, OPT, device=0, variant="b200")
    _compare(cpu, gpu, params, names, tol_all, tol_each)


def test_fused_ops_on_spar_tape_match_composed_cpu_step(ref, monkeypatch):
    """The product's differentiable fused operations (spar_b200/spar/fused.cppm, module spar.b200:
    layer_norm, linear_gelu, language_model_cross_entropy, grad_ready) recorded on Spar's own
    autograd tape through detail::record_operation, in the LN/GELU decoder on cuda:0, against the
    CPU step built from Spar's composed ops: the same 1e-5 bars (3xTF32 products). grad_ready's
    hooks fire once per backward pass per parameter, blocks in reverse order, each with the
    parameter's whole gradient (one micro-step: the gradient it ends with)."""
    monkeypatch.setenv("SPAR_B200_MATMUL_PRECISION", "tf32x3")
    lib = ref.load("b200")
    if not hasattr(lib, "ref_lm_step_fused"):
        pytest.skip("drop-in build without the fused module")
    cfg = {"vocab": 256, "dim": 128, "hidden": 512, "layers": 2, "heads": 4, "eps": 1e-5,
           "rope_theta": 1e4}
    params = O.init_parameters(cfg, 0x5EED0901)
    r = np.random.default_rng(9)
    for n, v in params.items():
        if v.ndim == 1:
            params[n] = ((1.0 if n.endswith("norm.weight") else 0.0)
                         + 0.05 * r.standard_normal(v.shape)).astype(np.float32)
    names = O.parameter_names(cfg["layers"])
    ids = O.Random(0x5EED1901).bounded(1 * 4 * 64, 256).reshape(1, 4, 64).astype(np.int32)
    cpu = ref.lm_step(params, names, ids, cfg, 3e-4, OPT, device=-1, variant="b200")
    loss, norm, grads, new, calls, norms, order = ref.lm_step_fused(params, names, ids, cfg, 3e-4,
                                                                    OPT, device=0)
    _compare(cpu, (loss, norm, grads, new), params, names, 1e-5, 1e-5)
    assert list(calls) == [1] * 6
    # slots (block, kind): block 1's three fire before block 0's (reverse layer order)
    assert sorted(order[:3]) == [3, 4, 5] and sorted(order[3:]) == [0, 1, 2]
    hooked = [f"blocks.{b}.{k}" for b in range(2)
              for k in ("attention_norm.weight", "mlp_norm.weight", "mlp.up_proj.weight")]
    for slot, n in enumerate(hooked):
        want = np.linalg.norm(grads[n].astype(np.float64))
        assert abs(norms[slot] - want) <= 1e-6 * want, n
