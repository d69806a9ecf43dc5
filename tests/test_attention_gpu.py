"""Fused causal attention (forward, and the query / key backward kernels) through the C ABI
against the float64 oracle restatement of the reference's attention chain.

Tolerance: relative L2 error <= 2e-3 for ctx and every third of dqkv (TF32 products: 10 explicit
mantissa bits in Q K^T, P V, dS K, ...), the bar stated for TF32 mode. The tensor cores read fp32
operands by dropping their low 13 mantissa bits, so inputs are handed over rounded to nearest
TF32 (as the training runtime stores them); the oracle sees the unrounded values.
"""
import numpy as np
import pytest

from _util import rel_l2
from oracle import spar_oracle as O

pytestmark = pytest.mark.gpu


def rn_tf32(x):
    """Round fp32 to the nearest TF32-representable value (10 explicit mantissa bits)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return (((b + 0x1000) & 0xFFFFE000).astype(np.uint32)).view(np.float32)


def _run(cuda, b, t, h, dh, seed):
    import torch
    from spar_b200 import ops

    r = np.random.default_rng(seed)
    d = h * dh
    qkv = r.standard_normal((b, t, 3 * d)).astype(np.float32)
    dctx = r.standard_normal((b, t, d)).astype(np.float32)
    q = torch.from_numpy(rn_tf32(qkv)).to(cuda)
    ctx, row_max, row_inv = ops.attention_forward(q, h)
    dqkv = ops.attention_backward(torch.from_numpy(rn_tf32(dctx)).to(cuda), q, ctx, row_max,
                                  row_inv, h)
    torch.cuda.synchronize()
    assert ops.attention_error(0) == 0
    ref_ctx, ref_dqkv = O.attention_forward_backward(qkv, h, dctx)
    return ctx.cpu().numpy(), dqkv.cpu().numpy(), ref_ctx, ref_dqkv, d


@pytest.mark.parametrize("b,t,h,dh", [
    (2, 256, 4, 64),    # whole 128-row tiles
    (1, 1024, 2, 64),   # the C4/C5 sequence length
    (2, 64, 4, 32),     # C1 shape: one partial tile, head_dim 32
    (1, 200, 3, 64),    # ragged sequence (partial query and key tiles)
    (3, 130, 2, 32),    # one row past a tile boundary
])
def test_attention_matches_oracle(cuda, b, t, h, dh):
    ctx, dqkv, ref_ctx, ref_dqkv, d = _run(cuda, b, t, h, dh, seed=b * 1000 + t + h + dh)
    assert rel_l2(ctx, ref_ctx) <= 2e-3
    for part, name in enumerate(("dq", "dk", "dv")):
        got = dqkv[..., part * d:(part + 1) * d]
        ref = ref_dqkv[..., part * d:(part + 1) * d]
        assert rel_l2(got, ref) <= 2e-3, name


def test_attention_adjacent_tile_pairs_match_oracle(cuda):
    """Enough work items (four or more per SM) switch the forward to adjacent query-tile pairs,
    heaviest first; an odd tile count leaves one unpaired tile per head."""
    b, t, h, dh = 24, 384, 16, 64
    ctx, dqkv, ref_ctx, ref_dqkv, d = _run(cuda, b, t, h, dh, seed=4242)
    assert rel_l2(ctx, ref_ctx) <= 2e-3
    for part, name in enumerate(("dq", "dk", "dv")):
        got = dqkv[..., part * d:(part + 1) * d]
        ref = ref_dqkv[..., part * d:(part + 1) * d]
        assert rel_l2(got, ref) <= 2e-3, name


def test_attention_is_deterministic(cuda):
    import torch
    from spar_b200 import ops

    r = np.random.default_rng(5)
    q = torch.from_numpy(r.standard_normal((2, 512, 3 * 256)).astype(np.float32)).to(cuda)
    do = torch.from_numpy(r.standard_normal((2, 512, 256)).astype(np.float32)).to(cuda)
    outs = []
    for _ in range(2):
        ctx, mx, inv = ops.attention_forward(q, 4)
        outs.append((ctx.cpu().numpy(), ops.attention_backward(do, q, ctx, mx, inv, 4).cpu().numpy()))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])


def test_attention_statistics(cuda):
    """The saved statistics reproduce the softmax: exp(scaled score - row_max * ln 2) * row_inv sums
    to 1 over the causal keys, and row_max (a running maximum that only moves when a key tile
    exceeds it by more than 8 in log2 units) lies within [max - 8 ln 2, max] of the scaled scores."""
    import torch
    from spar_b200 import ops

    b, t, h, dh = 1, 300, 2, 32
    r = np.random.default_rng(9)
    qkv = r.standard_normal((b, t, 3 * h * dh)).astype(np.float32)
    qkv[..., h * dh:2 * h * dh] *= (1.0 + np.arange(t) / 40.0)[None, :, None]  # later keys larger
    qkv = rn_tf32(qkv)  # exact TF32 operands, so the scores below are the kernel's to fp32 rounding
    ctx, row_max, row_inv = ops.attention_forward(torch.from_numpy(qkv).to(cuda), h)
    d = h * dh
    q = qkv[..., :d].reshape(b, t, h, dh).transpose(0, 2, 1, 3).astype(np.float64)
    k = qkv[..., d:2 * d].reshape(b, t, h, dh).transpose(0, 2, 1, 3).astype(np.float64)
    s = np.where(np.triu(np.ones((t, t), bool), 1), -np.inf, q @ k.transpose(0, 1, 3, 2) / np.sqrt(dh))
    m = s.max(-1)
    used = row_max.cpu().numpy().astype(np.float64) * np.log(2.0)
    assert np.all(used <= m + 1e-3 * np.abs(m) + 1e-4)
    assert np.all(used >= m - 8 * np.log(2.0) - 1e-3 * np.abs(m) - 1e-4)
    total = (np.exp(s - used[..., None]).sum(-1)) * row_inv.cpu().numpy()
    np.testing.assert_allclose(total, 1.0, rtol=1e-4)


def test_attention_running_max_rescale(cuda):
    """Keys that grow along the sequence make later key tiles exceed the running maximum, so the
    forward rescales O and the row sums mid-row; results still match the oracle."""
    import torch
    from spar_b200 import ops

    b, t, h, dh = 2, 512, 2, 64
    d = h * dh
    r = np.random.default_rng(77)
    qkv = r.standard_normal((b, t, 3 * d)).astype(np.float32)
    qkv[..., d:2 * d] *= (1.0 + np.arange(t) / 48.0)[None, :, None]
    qkv = rn_tf32(qkv)
    dctx = rn_tf32(r.standard_normal((b, t, d)).astype(np.float32))
    q = torch.from_numpy(qkv).to(cuda)
    ctx, row_max, row_inv = ops.attention_forward(q, h)
    dqkv = ops.attention_backward(torch.from_numpy(dctx).to(cuda), q, ctx, row_max, row_inv, h)
    torch.cuda.synchronize()
    assert ops.attention_error(0) == 0
    ref_ctx, ref_dqkv = O.attention_forward_backward(qkv, h, dctx)
    assert rel_l2(ctx.cpu().numpy(), ref_ctx) <= 2e-3
    got = dqkv.cpu().numpy()
    for part, name in enumerate(("dq", "dk", "dv")):
        assert rel_l2(got[..., part * d:(part + 1) * d], ref_dqkv[..., part * d:(part + 1) * d]) <= 2e-3, name


def test_attention_invalid_arguments(cuda):
    import torch
    from spar_b200 import _lib, ops

    q = torch.zeros(1, 64, 3 * 4 * 48, device=cuda)
    with pytest.raises(_lib.SparError):
        ops.attention_forward(q, 4)  # head_dim 48 is not supported


def test_attention_backward_inverse_rope(cuda):
    """With a RoPE table the backward returns dq, dk rotated back: the same as rotating the
    plain result with the standalone inverse rotation."""
    import torch
    from spar_b200 import ops

    b, t, h, dh = 2, 160, 2, 64
    d = h * dh
    r = np.random.default_rng(31)
    q = torch.from_numpy(rn_tf32(r.standard_normal((b, t, 3 * d)).astype(np.float32))).to(cuda)
    do = torch.from_numpy(rn_tf32(r.standard_normal((b, t, d)).astype(np.float32))).to(cuda)
    tab = ops.rope_table(t, dh, 10000.0, device=cuda)
    ctx, mx, inv = ops.attention_forward(q, h)
    rot = ops.attention_backward(do, q, ctx, mx, inv, h, rope_table=tab)
    plain = ops.attention_backward(do, q, ctx, mx, inv, h)
    ops.rope_apply_(plain, tab, b, t, 2 * h, dh, 3 * d, inverse=True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(rot.cpu().numpy(), plain.cpu().numpy(), rtol=1e-5, atol=1e-6)


def test_attention_c5_shape_repeated_without_timeouts(cuda):
    """The training shape (16 x 1024 tokens, 16 heads of 64, RoPE in the backward) run back to
    back: every CTA walks many work items, so the producer / MMA / softmax pipelines wrap many
    times; no bounded wait may expire and every output stays finite."""
    import torch
    from spar_b200 import ops

    b, t, h, dh = 16, 1024, 16, 64
    g = torch.Generator(device=cuda).manual_seed(3)
    qkv = torch.randn(b, t, 3 * h * dh, device=cuda, generator=g)
    do = torch.randn(b, t, h * dh, device=cuda, generator=g)
    tab = ops.rope_table(t, dh, 10000.0, device=cuda)
    for _ in range(6):
        ctx, mx, inv = ops.attention_forward(qkv, h)
        dqkv = ops.attention_backward(do, qkv, ctx, mx, inv, h, rope_table=tab)
    torch.cuda.synchronize()
    assert ops.attention_error(0) == 0
    assert torch.isfinite(ctx).all() and torch.isfinite(dqkv).all()


@pytest.mark.parametrize("b,t,h,kvh,dh", [(2, 384, 8, 2, 64), (1, 200, 4, 1, 32), (3, 256, 6, 3, 64),
                                          (2, 1024, 16, 4, 64)])
def test_gqa_matches_oracle(cuda, b, t, h, kvh, dh):
    """Grouped-query attention: query head i reads key/value head i // (h / kvh); the backward's
    dK / dV are summed over each group. Against the float64 oracle (repeat_kv_heads + the MHA
    chain) at the TF32 tolerance of the other attention tests."""
    import torch
    from spar_b200 import ops

    r = np.random.default_rng(b * t + h * 10 + kvh)
    w = (h + 2 * kvh) * dh
    qkv = r.standard_normal((b, t, w)).astype(np.float32)
    do = r.standard_normal((b, t, h * dh)).astype(np.float32)
    qt = torch.from_numpy(rn_tf32(qkv)).to(cuda)
    ctx, mx, inv = ops.attention_forward(qt, h, kv_heads=kvh)
    dqkv = ops.attention_backward(torch.from_numpy(rn_tf32(do)).to(cuda), qt, ctx, mx, inv, h,
                                  kv_heads=kvh)
    torch.cuda.synchronize()
    assert ops.attention_error(0) == 0
    o_ctx, o_d = O.attention_forward_backward(qkv, h, do, kv_heads=kvh)
    assert rel_l2(ctx.cpu().numpy(), o_ctx) <= 2e-3
    got = dqkv.cpu().numpy()
    d, dkv = h * dh, kvh * dh
    for lo, hi in ((0, d), (d, d + dkv), (d + dkv, w)):
        assert rel_l2(got[..., lo:hi], o_d[..., lo:hi]) <= 2e-3, (lo, hi)


def test_gqa_with_one_group_is_the_mha_call(cuda):
    """kv_heads == heads through the grouped entry points is bitwise the plain entry points."""
    import torch
    from spar_b200 import _lib, ops

    r = np.random.default_rng(5)
    b, t, h, dh = 2, 256, 4, 64
    qkv = torch.from_numpy(r.standard_normal((b, t, 3 * h * dh)).astype(np.float32)).to(cuda)
    do = torch.from_numpy(r.standard_normal((b, t, h * dh)).astype(np.float32)).to(cuda)
    ctx, mx, inv = ops.attention_forward(qkv, h, kv_heads=h)
    d1 = ops.attention_backward(do, qkv, ctx, mx, inv, h, kv_heads=h)
    lib = _lib.load()
    ctx2 = torch.empty_like(ctx)
    mx2, inv2 = torch.empty_like(mx), torch.empty_like(inv)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check("spar_b200_attention_forward",
               lib.spar_b200_attention_forward(qkv.data_ptr(), ctx2.data_ptr(), mx2.data_ptr(),
                                               inv2.data_ptr(), b, t, h, dh, 0, stream))
    d2 = torch.empty_like(qkv)
    delta = torch.empty_like(mx)
    _lib.check("spar_b200_attention_backward",
               lib.spar_b200_attention_backward(qkv.data_ptr(), ctx2.data_ptr(), do.data_ptr(),
                                                mx2.data_ptr(), inv2.data_ptr(), delta.data_ptr(),
                                                d2.data_ptr(), b, t, h, dh, None, 0, stream))
    torch.cuda.synchronize()
    assert torch.equal(ctx, ctx2) and torch.equal(d1, d2)
