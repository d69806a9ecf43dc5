"""Parity of the bandwidth-bound kernels (through the C ABI) against the CPU oracle.

Tolerance: per-op max relative error (max|ours - oracle| / max|oracle|) <= 1e-5 against the
float64 restatement, the bar stated for the non-GEMM kernels.
"""
import math

import numpy as np
import pytest

from _util import rel_err
from oracle import spar_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _rng(seed):
    return np.random.default_rng(seed)


@pytest.mark.parametrize("rows,cols", [(64, 128), (257, 768), (512, 1024), (33, 2048), (7, 4)])
def test_layernorm_forward_backward(cuda, rows, cols):
    import torch
    from spar_b200 import ops

    r = _rng(rows * cols)
    x = r.standard_normal((rows, cols)).astype(np.float32)
    gamma = (1 + 0.1 * r.standard_normal(cols)).astype(np.float32)
    beta = (0.1 * r.standard_normal(cols)).astype(np.float32)
    dy = r.standard_normal((rows, cols)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)
    y, mean, rstd = ops.layer_norm_forward(t(x), t(gamma), t(beta), 1e-5)
    dx, dg, db = ops.layer_norm_backward(t(dy), t(x), t(gamma), mean, rstd)
    torch.cuda.synchronize()
    y64, _, _ = O.layer_norm_forward(x, gamma, beta, 1e-5, np.float64)
    dx64, dg64, db64 = O.layer_norm_backward(dy, x, gamma, 1e-5)
    assert rel_err(y.cpu().numpy(), y64) <= TOL
    assert rel_err(dx.cpu().numpy(), dx64) <= TOL
    assert rel_err(dg.cpu().numpy(), dg64) <= TOL
    assert rel_err(db.cpu().numpy(), db64) <= TOL


def test_layernorm_backward_accumulate_and_deterministic(cuda):
    import torch
    from spar_b200 import ops

    r = _rng(5)
    x = torch.from_numpy(r.standard_normal((1000, 1024)).astype(np.float32)).to(cuda)
    dy = torch.from_numpy(r.standard_normal((1000, 1024)).astype(np.float32)).to(cuda)
    g = torch.ones(1024, device=cuda)
    b = torch.zeros(1024, device=cuda)
    _, mean, rstd = ops.layer_norm_forward(x, g, b)
    dx1, dg1, db1 = ops.layer_norm_backward(dy, x, g, mean, rstd)
    dx2, dg2, db2 = ops.layer_norm_backward(dy, x, g, mean, rstd)
    assert torch.equal(dg1, dg2) and torch.equal(db1, db2) and torch.equal(dx1, dx2)
    dg3, db3 = dg1.clone(), db1.clone()
    ops.layer_norm_backward(dy, x, g, mean, rstd, dgamma=dg3, dbeta=db3, accumulate_params=True)
    torch.cuda.synchronize()
    assert torch.allclose(dg3, 2 * dg1, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("rows,cols", [(64, 128), (257, 768), (2048, 1024), (33, 2048), (7, 4)])
def test_rmsnorm_forward_backward(cuda, rows, cols):
    import torch
    from spar_b200 import ops

    r = _rng(rows * cols + 1)
    x = r.standard_normal((rows, cols)).astype(np.float32)
    x[0] *= 50.0
    w = (1 + 0.1 * r.standard_normal(cols)).astype(np.float32)
    dy = r.standard_normal((rows, cols)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda)
    y, rstd = ops.rms_norm_forward(t(x), t(w), 1e-5)
    dx, dw = ops.rms_norm_backward(t(dy), t(x), t(w), rstd)
    torch.cuda.synchronize()
    y64, rstd64 = O.rms_norm_forward(x, w, 1e-5, np.float64)
    dx64, dw64 = O.rms_norm_backward(dy, x, w, 1e-5)
    assert rel_err(y.cpu().numpy(), y64) <= TOL and rel_err(rstd.cpu().numpy(), rstd64) <= TOL
    assert rel_err(dx.cpu().numpy(), dx64) <= TOL
    assert rel_err(dw.cpu().numpy(), dw64) <= TOL


def test_rmsnorm_backward_accumulate_deterministic_and_empty(cuda):
    import torch
    from spar_b200 import ops

    r = _rng(6)
    x = torch.from_numpy(r.standard_normal((1000, 1024)).astype(np.float32)).to(cuda)
    dy = torch.from_numpy(r.standard_normal((1000, 1024)).astype(np.float32)).to(cuda)
    w = torch.ones(1024, device=cuda)
    _, rstd = ops.rms_norm_forward(x, w)
    dx1, dw1 = ops.rms_norm_backward(dy, x, w, rstd)
    dx2, dw2 = ops.rms_norm_backward(dy, x, w, rstd)
    assert torch.equal(dw1, dw2) and torch.equal(dx1, dx2)
    dw3, dx3 = dw1.clone(), dx1.clone()
    ops.rms_norm_backward(dy, x, w, rstd, dweight=dw3, dx=dx3, accumulate_params=True,
                          accumulate_dx=True)
    torch.cuda.synchronize()
    assert torch.allclose(dw3, 2 * dw1, rtol=1e-6, atol=1e-6)
    assert torch.allclose(dx3, 2 * dx1, rtol=1e-6, atol=1e-6)
    # No rows: the weight gradient is zero (or left alone when accumulating).
    e = torch.empty(0, 1024, device=cuda)
    dwz = torch.full((1024,), 5.0, device=cuda)
    ops.rms_norm_backward(e, e, w, torch.empty(0, device=cuda), dweight=dwz)
    torch.cuda.synchronize()
    assert torch.count_nonzero(dwz).item() == 0


@pytest.mark.parametrize("tokens,heads,head_dim", [(2048, 16, 64), (37, 4, 32), (5, 3, 128)])
def test_head_rmsnorm_qk_norm(cuda, tokens, heads, head_dim):
    """qk-norm on the q and k parts of a packed [tokens, 3d] projection, in place, against the
    oracle RMSNorm over each head's features; the v part is untouched."""
    import torch
    from spar_b200 import ops

    d = heads * head_dim
    r = _rng(tokens * heads + head_dim)
    qkv = (2 * r.standard_normal((tokens, 3 * d))).astype(np.float32)
    w = (1 + 0.1 * r.standard_normal(head_dim)).astype(np.float32)
    dy = r.standard_normal((tokens, 3 * d)).astype(np.float32)
    t = torch.from_numpy(qkv.copy()).to(cuda)
    wt = torch.from_numpy(w).to(cuda)
    dyt = torch.from_numpy(dy).to(cuda)
    q, k = t[:, :d], t[:, d:2 * d]
    saved = t.clone()  # the inputs, with the packed row stride
    x_q, x_k = saved[:, :d], saved[:, d:2 * d]
    _, rq = ops.head_rms_norm_forward(q, heads, head_dim, wt, out=q)
    yk, rk = ops.head_rms_norm_forward(k, heads, head_dim, wt)
    dxq, dwq = ops.head_rms_norm_backward(dyt[:, :d], x_q, heads, head_dim, wt, rq)
    dxk, dwk = ops.head_rms_norm_backward(dyt[:, d:2 * d], x_k, heads, head_dim, wt, rk)
    torch.cuda.synchronize()
    out = t.cpu().numpy()
    assert np.array_equal(out[:, 2 * d:], qkv[:, 2 * d:]) and np.array_equal(out[:, d:2 * d], qkv[:, d:2 * d])
    for part, y, dx, dw in ((0, out[:, :d], dxq, dwq), (1, yk.cpu().numpy(), dxk, dwk)):
        xs = qkv[:, part * d:(part + 1) * d].reshape(tokens * heads, head_dim)
        dys = dy[:, part * d:(part + 1) * d].reshape(tokens * heads, head_dim)
        y64, _ = O.rms_norm_forward(xs, w, 1e-5, np.float64)
        dx64, dw64 = O.rms_norm_backward(dys, xs, w, 1e-5)
        assert rel_err(np.asarray(y).reshape(tokens * heads, head_dim), y64) <= TOL
        assert rel_err(dx.cpu().numpy().reshape(tokens * heads, head_dim), dx64) <= TOL
        assert rel_err(dw.cpu().numpy(), dw64) <= TOL


@pytest.mark.parametrize("rows,cols,fused", [(2048, 4096, True), (2048, 4096, False), (3, 7, True),
                                             (1, 1, False), (513, 1028, True)])
def test_swiglu(cuda, rows, cols, fused):
    """gate / value as the two column halves of one [rows, 2 cols] projection (row stride 2 cols)
    or as separate tensors; odd widths take the scalar path."""
    import torch
    from spar_b200 import ops

    r = _rng(rows * cols + int(fused))
    gv = (3 * r.standard_normal((rows, 2 * cols))).astype(np.float32)
    gv[0, :4 if cols >= 4 else 1] = [0.0, -40.0, 40.0, 1e-6][:4 if cols >= 4 else 1]
    dh = r.standard_normal((rows, cols)).astype(np.float32)
    t = torch.from_numpy(gv).to(cuda)
    if fused:
        gate, value = t[:, :cols], t[:, cols:]
    else:
        gate, value = t[:, :cols].contiguous(), t[:, cols:].contiguous()
    h = ops.swiglu_forward(gate, value)
    dg, dv = ops.swiglu_backward(torch.from_numpy(dh).to(cuda), gate, value)
    torch.cuda.synchronize()
    g64, v64 = gv[:, :cols], gv[:, cols:]
    assert rel_err(h.cpu().numpy(), O.swiglu_forward(g64, v64, np.float64)) <= TOL
    odg, odv = O.swiglu_backward(dh, g64, v64)
    assert rel_err(dg.cpu().numpy(), odg) <= TOL and rel_err(dv.cpu().numpy(), odv) <= TOL


@pytest.mark.parametrize("n", [1, 7, 4096, 1 << 20])
def test_gelu(cuda, n):
    import torch
    from spar_b200 import ops

    r = _rng(n)
    x = (3 * r.standard_normal(n)).astype(np.float32)
    x[:min(n, 4)] = [0.0, -20.0, 20.0, 1e-3][:min(n, 4)]
    dy = r.standard_normal(n).astype(np.float32)
    xt = torch.from_numpy(x).to(cuda)
    y = ops.gelu_forward(xt)
    dx = ops.gelu_backward(torch.from_numpy(dy).to(cuda), xt)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), O.gelu_forward(x, np.float64)) <= TOL
    assert rel_err(dx.cpu().numpy(), dy * O.gelu_derivative(x)) <= TOL


@pytest.mark.parametrize("batch,t", [(4, 64), (3, 256), (2, 1024), (1, 12), (1, 2048)])
def test_causal_softmax(cuda, batch, t):
    import torch
    from spar_b200 import ops

    r = _rng(batch * t)
    s = r.standard_normal((batch, t, t)).astype(np.float32)
    dp = r.standard_normal((batch, t, t)).astype(np.float32)
    scale = 1.0 / math.sqrt(64)
    st = torch.from_numpy(s).to(cuda)
    # Entries above the diagonal must never be read: poison them.
    st.masked_fill_(torch.triu(torch.ones(t, t, dtype=torch.bool, device=cuda), 1), float("nan"))
    p = ops.causal_softmax_forward(st, scale)
    ds = ops.causal_softmax_backward(torch.from_numpy(dp).to(cuda), p, scale)
    torch.cuda.synchronize()
    p64 = O.causal_softmax_forward(s, scale, np.float64)
    assert rel_err(p.cpu().numpy(), p64) <= TOL
    assert rel_err(ds.cpu().numpy(), O.causal_softmax_backward(dp, p64, scale)) <= TOL


def test_causal_softmax_zero_fill_block(cuda):
    import torch
    from spar_b200 import ops

    t = 512
    s = torch.randn(2, t, t, device=cuda)
    out = torch.full_like(s, 7.0)
    ops.causal_softmax_forward(s, 0.125, zero_fill_block=128, out=out)
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    for i in (0, 5, 127, 128, 300, 511):
        end = min(t, (i // 128 + 1) * 128)
        assert np.all(o[:, i, i + 1:end] == 0.0)
        assert np.all(o[:, i, end:] == 7.0)


@pytest.mark.parametrize("rows,classes,seq", [(512, 256, 64), (64, 32768, 0), (96, 50257, 0),
                                              (128, 4096, 16), (17, 8, 0)])
def test_cross_entropy(cuda, rows, classes, seq):
    import torch
    from spar_b200 import ops

    r = _rng(rows + classes)
    z = (2 * r.standard_normal((rows, classes))).astype(np.float32)
    tg = r.integers(0, classes, rows).astype(np.int32)
    loss, dz, invalid = ops.cross_entropy_forward_backward(
        torch.from_numpy(z).to(cuda), torch.from_numpy(tg).to(cuda), sequence_length=seq)
    torch.cuda.synchronize()
    if seq:
        sel = np.arange(rows).reshape(-1, seq)[:, :-1].reshape(-1)
        targets = tg.reshape(-1, seq)[:, 1:].reshape(-1)
    else:
        sel, targets = np.arange(rows), tg
    mean, row_loss, d = O.cross_entropy_forward_backward(z, targets, sel)
    assert invalid.item() == 0
    assert rel_err(loss.cpu().numpy(), row_loss) <= TOL
    assert rel_err(dz.cpu().numpy(), d) <= TOL
    got_mean = loss.cpu().numpy().astype(np.float64).sum() / len(sel)
    assert abs(got_mean - mean) <= TOL * abs(mean)


def test_cross_entropy_invalid_target_flag(cuda):
    import torch
    from spar_b200 import ops

    z = torch.randn(4, 64, device=cuda)
    tg = torch.tensor([1, 64, 3, -1], dtype=torch.int32, device=cuda)
    loss, dz, invalid = ops.cross_entropy_forward_backward(z, tg)
    torch.cuda.synchronize()
    assert invalid.item() == 1
    l = loss.cpu().numpy()
    assert np.isnan(l[1]) and np.isnan(l[3]) and np.isfinite(l[0]) and np.isfinite(l[2])
    assert torch.count_nonzero(dz[1]).item() == 0


def test_cross_entropy_in_place(cuda):
    import torch
    from spar_b200 import ops

    z = torch.randn(64, 32768, device=cuda)
    tg = torch.randint(0, 32768, (64,), dtype=torch.int32, device=cuda)
    l1, d1, _ = ops.cross_entropy_forward_backward(z.clone(), tg)
    zz = z.clone()
    l2, d2, _ = ops.cross_entropy_forward_backward(zz, tg, in_place=True)
    torch.cuda.synchronize()
    assert d2.data_ptr() == zz.data_ptr()
    assert torch.equal(d1, d2) and torch.equal(l1, l2)


@pytest.mark.parametrize("clip", [1.0, 1e9, -1.0])
def test_grad_norm_and_adamw(cuda, clip):
    import torch
    from spar_b200 import ops

    r = _rng(11)
    sizes = [1000, 4096, 3, 65536]
    ps = [(0.02 * r.standard_normal(s)).astype(np.float32) for s in sizes]
    gs = [(1e-1 * r.standard_normal(s)).astype(np.float32) for s in sizes]
    ms = [(1e-2 * r.standard_normal(s)).astype(np.float32) for s in sizes]
    vs = [(1e-3 * np.abs(r.standard_normal(s))).astype(np.float32) for s in sizes]
    T = lambda l: [torch.from_numpy(a.copy()).to(cuda) for a in l]
    tp, tg, tm, tv = T(ps), T(gs), T(ms), T(vs)
    state = ops.grad_norm_squared(tg)
    flag = ops.adamw_clipped(tp, tg, tm, tv, state, lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8,
                             weight_decay=0.1, step=3, max_norm=clip)
    torch.cuda.synchronize()
    norm = O.global_grad_norm(gs)
    assert abs(math.sqrt(state[0].item()) - norm) <= 1e-12 * norm
    assert flag.item() == 0
    factor = O.clip_factor(norm, clip) if clip >= 0 else 1.0
    for j in range(len(sizes)):
        p2, m2, v2 = O.adamw_update(ps[j], gs[j], ms[j], vs[j], 3, 3e-4, 0.9, 0.95, 1e-8, 0.1,
                                    factor)
        # The oracle mirrors the reference's double math: expect (near) bit equality.
        assert rel_err(tp[j].cpu().numpy(), p2) <= 1e-6
        assert rel_err(tm[j].cpu().numpy(), m2) <= 1e-6
        assert rel_err(tv[j].cpu().numpy(), v2) <= 1e-6


def test_adamw_nonfinite_norm_leaves_state(cuda):
    import torch
    from spar_b200 import ops

    p = torch.randn(4096, device=cuda)
    g = torch.randn(4096, device=cuda)
    g[17] = float("inf")
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    p0 = p.clone()
    state = ops.grad_norm_squared([g])
    flag = ops.adamw_clipped([p], [g], [m], [v], state, lr=1e-3, step=1, max_norm=1.0)
    torch.cuda.synchronize()
    assert flag.item() == 1
    assert torch.equal(p, p0) and torch.count_nonzero(m).item() == 0


@pytest.mark.parametrize("vocab,dim,count", [(256, 128, 512), (32768, 1024, 4096),
                                             (50257, 768, 1000), (8, 4, 3000)])
def test_embedding(cuda, vocab, dim, count):
    import torch
    from spar_b200 import ops

    r = _rng(vocab + count)
    w = r.standard_normal((vocab, dim)).astype(np.float32)
    ids = r.integers(0, vocab, count).astype(np.int32)
    go = r.standard_normal((count, dim)).astype(np.float32)
    base = r.standard_normal((vocab, dim)).astype(np.float32)
    wt = torch.from_numpy(w).to(cuda)
    it = torch.from_numpy(ids).to(cuda)
    out, invalid = ops.embedding_forward(wt, it)
    gw = torch.from_numpy(base.copy()).to(cuda)
    ops.embedding_backward(gw, torch.from_numpy(go).to(cuda), it)
    gw2 = torch.from_numpy(base.copy()).to(cuda)
    ops.embedding_backward(gw2, torch.from_numpy(go).to(cuda), it)
    torch.cuda.synchronize()
    assert invalid.item() == 0
    assert np.array_equal(out.cpu().numpy(), w[ids])
    ref = base.astype(np.float64).copy()
    np.add.at(ref, ids, go.astype(np.float64))
    assert rel_err(gw.cpu().numpy(), ref) <= TOL
    assert torch.equal(gw, gw2)  # deterministic


def test_embedding_invalid_ids(cuda):
    import torch
    from spar_b200 import ops

    w = torch.randn(16, 8, device=cuda)
    ids = torch.tensor([0, 16, -3, 5], dtype=torch.int32, device=cuda)
    out, invalid = ops.embedding_forward(w, ids)
    gw = torch.zeros_like(w)
    ops.embedding_backward(gw, torch.ones(4, 8, device=cuda), ids)
    torch.cuda.synchronize()
    assert invalid.item() == 1
    assert torch.count_nonzero(out[1]).item() == 0
    assert gw[0].sum().item() == 8 and gw[5].sum().item() == 8 and gw.sum().item() == 16


@pytest.mark.parametrize("rows,cols", [(16384, 1024), (100, 3072), (5, 4)])
def test_column_sum(cuda, rows, cols):
    import torch
    from spar_b200 import ops

    x = np.random.default_rng(rows).standard_normal((rows, cols)).astype(np.float32)
    out = ops.column_sum(torch.from_numpy(x).to(cuda))
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), x.astype(np.float64).sum(0)) <= TOL


def test_rope_roundtrip_and_values(cuda):
    import torch
    from spar_b200 import ops

    b, t, h, d = 2, 64, 4, 32
    ld = 3 * h * d  # q block of a fused qkv row
    r = _rng(3)
    qkv = r.standard_normal((b * t, ld)).astype(np.float32)
    xt = torch.from_numpy(qkv.copy()).to(cuda)
    table = ops.rope_table(t, d, 10000.0, device=cuda)
    ops.rope_apply_(xt, table, b, t, h, d, ld)
    torch.cuda.synchronize()
    cos, sin = O.rope_table(t, d)
    q = qkv[:, : h * d].reshape(b, t, h, d).transpose(0, 2, 1, 3)
    ref = O.rope_apply(q.astype(np.float64), cos, sin).transpose(0, 2, 1, 3).reshape(b * t, h * d)
    got = xt.cpu().numpy()
    assert rel_err(got[:, : h * d], ref) <= TOL
    assert np.array_equal(got[:, h * d:], qkv[:, h * d:])
    ops.rope_apply_(xt, table, b, t, h, d, ld, inverse=True)
    torch.cuda.synchronize()
    assert rel_err(xt.cpu().numpy(), qkv) <= 1e-6
