"""CPU checks of the oracle itself: known answers of the RNG, finite-difference gradients of
every restated backward (float64), and schedule/optimiser properties. The reference-pinned
golden fixtures are checked in tests/test_golden.py."""
import math

import numpy as np
import pytest

from oracle import spar_oracle as O


def test_splitmix64_known_answers():
    # SplitMix64 reference outputs for seed 0 (the generator Spar's Random implements,
    # src/core/random.cpp:22-28).
    r = O.Random(0)
    got = [int(v) for v in r.next_u64(3)]
    assert got == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]
    # The counter form used by the device initialiser gives the same stream.
    r2 = O.Random(0)
    assert [int(v) for v in r2.next_u64(1)] + [int(v) for v in r2.next_u64(2)] == got


def test_uniform_and_normal_moments():
    r = O.Random(123)
    u = r.uniform_double(200000)
    assert 0.0 <= u.min() and u.max() < 1.0 and abs(u.mean() - 0.5) < 5e-3
    z = O.Random(7).normal(200000, 0.02)
    assert z.dtype == np.float32
    assert abs(z.mean()) < 3e-4 and abs(z.std() - 0.02) < 3e-4


def test_bounded_index_rejection():
    r = O.Random(5)
    v = r.bounded(1000, 50257)
    assert v.min() >= 0 and v.max() < 50257
    v2 = O.Random(5).bounded(1000, 256)
    assert v2.max() < 256


def _fd(f, x, eps=1e-6, n=25, seed=0):
    """Central differences of scalar f along random coordinates of x."""
    r = np.random.default_rng(seed)
    idx = r.choice(x.size, size=min(n, x.size), replace=False)
    out = []
    for i in idx:
        xp = x.copy().ravel()
        xm = x.copy().ravel()
        xp[i] += eps
        xm[i] -= eps
        out.append((f(xp.reshape(x.shape)) - f(xm.reshape(x.shape))) / (2 * eps))
    return idx, np.array(out)


def test_layer_norm_backward_fd():
    r = np.random.default_rng(1)
    x = r.standard_normal((5, 12))
    g = 1 + 0.1 * r.standard_normal(12)
    b = 0.1 * r.standard_normal(12)
    w = r.standard_normal((5, 12))
    loss = lambda xx: float((O.layer_norm_forward(xx, g, b, 1e-5, np.float64)[0] * w).sum())
    dx, dg, db = O.layer_norm_backward(w, x, g, 1e-5)
    idx, num = _fd(loss, x)
    np.testing.assert_allclose(dx.ravel()[idx], num, rtol=1e-6, atol=1e-8)
    idx, num = _fd(lambda gg: float((O.layer_norm_forward(x, gg, b, 1e-5, np.float64)[0] * w).sum()), g)
    np.testing.assert_allclose(dg.ravel()[idx], num, rtol=1e-6, atol=1e-8)
    np.testing.assert_allclose(db, w.sum(0), rtol=1e-12)


def test_gelu_derivative_fd():
    x = np.linspace(-8, 8, 101)
    num = (O.gelu_forward(x + 1e-6, np.float64) - O.gelu_forward(x - 1e-6, np.float64)) / 2e-6
    np.testing.assert_allclose(O.gelu_derivative(x), num, rtol=1e-6, atol=1e-8)
    # tanh form identity: x * sigmoid(2u) == 0.5 x (1 + tanh(u))
    u = 0.7978845608028654 * (x + 0.044715 * x ** 3)
    np.testing.assert_allclose(O.gelu_forward(x, np.float64), 0.5 * x * (1 + np.tanh(u)), rtol=1e-12, atol=1e-15)


def test_causal_softmax_backward_fd():
    r = np.random.default_rng(2)
    s = r.standard_normal((2, 6, 6))
    w = r.standard_normal((2, 6, 6))
    scale = 0.3
    p = O.causal_softmax_forward(s, scale, np.float64)
    assert np.allclose(p.sum(-1), 1) and np.all(np.triu(p[0], 1) == 0)
    ds = O.causal_softmax_backward(w, p, scale)
    idx, num = _fd(lambda ss: float((O.causal_softmax_forward(ss, scale, np.float64) * w).sum()), s)
    np.testing.assert_allclose(ds.ravel()[idx], num, rtol=1e-6, atol=1e-9)


def test_cross_entropy_gradient_fd():
    r = np.random.default_rng(3)
    z = 2 * r.standard_normal((7, 11))
    t = r.integers(0, 11, 5)
    rows = np.array([0, 1, 3, 4, 6])
    loss, _, d = O.cross_entropy_forward_backward(z, t, rows)
    idx, num = _fd(lambda zz: float(O.cross_entropy_forward_backward(zz, t, rows)[0]), z)
    np.testing.assert_allclose(d.ravel()[idx], num, rtol=1e-6, atol=1e-9)
    assert np.all(d[[2, 5]] == 0)


def test_lm_backward_fd():
    cfg = {"vocab": 16, "dim": 8, "hidden": 12, "layers": 2, "heads": 2}
    params = O.init_parameters(cfg, 9, std=0.3)
    r = np.random.default_rng(4)
    for n in params:  # non-trivial LayerNorm parameters and biases
        if params[n].ndim == 1:
            params[n] = params[n] + 0.1 * r.standard_normal(params[n].shape).astype(np.float32)
    ids = r.integers(0, 16, (2, 6))
    P64 = {k: v.astype(np.float64) for k, v in params.items()}
    _, grads = O.lm_forward_backward(P64, ids, cfg)
    for name in ["token_embedding.weight", "blocks.0.attention.q_proj.weight",
                 "blocks.1.attention.k_proj.bias", "blocks.0.mlp.up_proj.weight",
                 "blocks.1.mlp_norm.weight", "final_norm.bias", "blocks.0.attention_norm.bias"]:
        def f(w, name=name):
            q = dict(P64)
            q[name] = w
            return O.lm_forward_backward(q, ids, cfg)[0]
        idx, num = _fd(f, P64[name], eps=1e-6, n=12)
        np.testing.assert_allclose(grads[name].ravel()[idx], num, rtol=2e-5, atol=1e-9, err_msg=name)


def test_warmup_cosine_schedule():
    assert O.warmup_cosine(1.0, 0.0, 10, 100, 0) == pytest.approx(0.1)
    assert O.warmup_cosine(1.0, 0.0, 10, 100, 9) == pytest.approx(1.0)
    assert O.warmup_cosine(1.0, 0.0, 10, 100, 10) == pytest.approx(1.0)
    assert O.warmup_cosine(1.0, 0.1, 10, 100, 109) == pytest.approx(0.1)
    assert O.warmup_cosine(1.0, 0.1, 10, 100, 500) == 0.1
    mid = O.warmup_cosine(1.0, 0.0, 0, 101, 50)
    assert mid == pytest.approx(0.5)


def test_adamw_first_step_is_sign_update():
    p = np.array([0.5, -0.5, 0.1], np.float32)
    g = np.array([1e-3, -2.0, 0.0], np.float32)
    z = np.zeros(3, np.float32)
    p2, m, v = O.adamw_update(p, g, z, z, 1, 0.01, 0.9, 0.95, 1e-8, 0.1)
    expect = p.astype(np.float64) * (1 - 0.001) - 0.01 * np.sign(g)
    np.testing.assert_allclose(p2, expect, rtol=1e-5, atol=1e-9)
    assert math.isnan(O.global_grad_norm([np.array([np.nan], np.float32)]))
    with pytest.raises(RuntimeError):
        O.clip_factor(float("inf"), 1.0)


def test_product_token_stream_matches_oracle_sampler():
    """spar_b200.data draws the same ids as the oracle's bounded_index restatement."""
    from spar_b200.data import token_ids

    for vocab in (256, 32768, 50257, 1000003):
        np.testing.assert_array_equal(token_ids(77, 3000, vocab), O.Random(77).bounded(3000, vocab))
