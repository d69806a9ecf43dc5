"""Parity of the tcgen05 GEMM (through the C ABI) against a float64 matmul.

Tolerances: TF32 mode rel-L2 <= 2e-3 (TF32 keeps 10 mantissa bits), 3xTF32 mode rel-L2 <= 1e-5
and max relative error <= 1e-5 (fp32-faithful), the bars stated for the GEMMs.
"""
import numpy as np
import pytest

from _util import rel_err, rel_l2

pytestmark = pytest.mark.gpu


def _mats(m, n, k, a_t, b_t, seed=0):
    r = np.random.default_rng(seed)
    a = r.standard_normal((k, m) if a_t else (m, k)).astype(np.float32)
    b = (0.02 * r.standard_normal((n, k) if b_t else (k, n))).astype(np.float32)
    a64 = a.astype(np.float64).T if a_t else a.astype(np.float64)
    b64 = b.astype(np.float64).T if b_t else b.astype(np.float64)
    return a, b, a64 @ b64


SHAPES = [
    (128, 256, 64),
    (256, 512, 1024),
    (200, 300, 96),     # ragged M/N, K multiple of 32
    (1000, 768, 3072),
    (64, 64, 64),
    (384, 100, 40),     # ragged K
    (2048, 1024, 4096),
]


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_tf32_layouts(cuda, shape, a_t, b_t):
    import torch
    from spar_b200 import ops

    m, n, k = shape
    if (a_t and m % 4) or (not b_t and n % 4) or (not a_t and k % 4) or (b_t and k % 4):
        pytest.skip("leading dimension must be a multiple of 4")
    a, b, ref = _mats(m, n, k, a_t, b_t, seed=m + n + k)
    c = ops.matmul(torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda), a_t=a_t, b_t=b_t)
    torch.cuda.synchronize()
    assert ops.gemm_error(0) == 0
    assert rel_l2(c.cpu().numpy(), ref) <= 2e-3


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False)])
@pytest.mark.parametrize("shape", [(256, 512, 1024), (200, 300, 96), (1024, 1024, 2048),
                                   (512, 768, 24576), (128, 96, 24576)])
def test_gemm_3xtf32(cuda, shape, a_t, b_t):
    """The last two shapes have a long K: on SM pairs the accumulator is drained into fp32
    registers every 256 concatenated K elements, on single SMs K is split into parts."""
    import torch
    from spar_b200 import ops

    m, n, k = shape
    a, b, ref = _mats(m, n, k, a_t, b_t, seed=7)
    c = ops.matmul(torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda), a_t=a_t, b_t=b_t,
                   precision=ops.TF32X3)
    torch.cuda.synchronize()
    assert ops.gemm_error(0) == 0
    got = c.cpu().numpy()
    assert rel_l2(got, ref) <= 1e-5
    assert rel_err(got, ref) <= 1e-5


def test_gemm_epilogues(cuda):
    import torch
    from spar_b200 import ops
    from oracle import spar_oracle as O

    m, n, k = 256, 512, 256
    a, b, ref = _mats(m, n, k, False, False, seed=3)
    bias = np.random.default_rng(4).standard_normal(n).astype(np.float32)
    at, bt = torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)
    biast = torch.from_numpy(bias).to(cuda)
    prec = ops.TF32X3
    c = ops.matmul(at, bt, epilogue=ops.EPI_BIAS, bias=biast, precision=prec, alpha=0.5)
    pre = torch.empty(m, n, device=cuda)
    g = ops.matmul(at, bt, epilogue=ops.EPI_BIAS_GELU, bias=biast, aux=pre, precision=prec)
    dpre = ops.matmul(at, bt, epilogue=ops.EPI_GELU_BWD, aux=pre, precision=prec)
    acc = torch.ones(m, n, device=cuda)
    ops.matmul(at, bt, out=acc, accumulate=True, precision=prec)
    resid = torch.randn(m, n, device=cuda)
    radd = ops.matmul(at, bt, epilogue=ops.EPI_BIAS_ADD, bias=biast, aux=resid, precision=prec)
    radd_nb = ops.matmul(at, bt, epilogue=ops.EPI_BIAS_ADD, aux=resid, precision=prec)
    torch.cuda.synchronize()
    pre_ref = ref + bias
    assert rel_err(c.cpu().numpy(), 0.5 * ref + bias) <= 1e-5
    assert rel_err(pre.cpu().numpy(), pre_ref) <= 1e-5
    assert rel_err(g.cpu().numpy(), O.gelu_forward(pre_ref, np.float64)) <= 1e-5
    pre32 = pre.cpu().numpy()
    assert rel_err(dpre.cpu().numpy(), ref * O.gelu_derivative(pre32)) <= 1e-5
    assert rel_err(acc.cpu().numpy(), ref + 1.0) <= 1e-5
    r = resid.cpu().numpy().astype(np.float64)
    assert rel_err(radd.cpu().numpy(), ref + bias + r) <= 1e-5
    assert rel_err(radd_nb.cpu().numpy(), ref + r) <= 1e-5


@pytest.mark.parametrize("m,n,k", [(1024, 1024, 16384), (1024, 3072, 8192), (768, 768, 4096),
                                   (300, 196, 8192), (200, 100, 6144)])
def test_gemm_split_k_weight_gradient(cuda, m, n, k):
    """Weight-gradient shapes (A transposed, K = tokens) take the split-K path: partial tiles
    summed in split order, so accumulate + alpha hold and repeated runs are bitwise equal.
    Ragged shapes cover clipped rows/columns on the paired and the single-SM kernels."""
    import torch
    from spar_b200 import ops

    a, b, ref = _mats(m, n, k, True, False, seed=11)
    at, bt = torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)
    base = torch.from_numpy(np.random.default_rng(12).standard_normal((m, n)).astype(np.float32))
    outs = []
    for _ in range(2):
        c = base.to(cuda)
        ops.matmul(at, bt, a_t=True, out=c, accumulate=True, alpha=0.5)
        outs.append(c.cpu().numpy())
    torch.cuda.synchronize()
    assert ops.gemm_error(0) == 0
    assert np.array_equal(outs[0], outs[1])
    expect = 0.5 * ref + base.numpy().astype(np.float64)
    assert rel_l2(outs[0], expect) <= 2e-3


def _attention_views(cuda, b, h, t, dh, seed=0):
    import torch

    d = h * dh
    r = np.random.default_rng(seed)
    qkv = r.standard_normal((b * t, 3 * d)).astype(np.float32)
    return qkv, torch.from_numpy(qkv).to(cuda)


@pytest.mark.parametrize("b,h,t,dh", [(2, 4, 256, 64), (1, 2, 512, 64), (2, 3, 64, 32)])
def test_gemm_attention_batched_causal(cuda, b, h, t, dh):
    """The six attention products on head-strided views of a fused [B*T, 3d] QKV buffer."""
    import torch
    from spar_b200 import ops

    d = h * dh
    qkv, qkvt = _attention_views(cuda, b, h, t, dh, seed=t)
    ld = 3 * d
    base = qkvt.data_ptr()
    q_ptr, k_ptr, v_ptr = base, base + 4 * d, base + 8 * d
    bs = (t * ld, dh)  # (batch, head) strides in elements
    dev, stream = 0, torch.cuda.current_stream().cuda_stream
    prec = ops.TF32X3
    S = torch.empty(b, h, t, t, device=cuda)
    s_bs = (h * t * t, t * t)
    # S = Q K^T (lower tiles only)
    ops.gemm_run(ops.gemm_desc(t, t, dh, q_ptr, ld, k_ptr, ld, S.data_ptr(), t, b_t=True,
                               batch=(b, h), a_bs=bs, b_bs=bs, c_bs=s_bs, precision=prec,
                               causal=ops.CAUSAL_LOWER), dev, stream)
    P = ops.causal_softmax_forward(S, 1.0 / np.sqrt(dh), zero_fill_block=128)
    # O = P V  (k <= row)
    ctx = torch.empty(b * t, d, device=cuda)
    ops.gemm_run(ops.gemm_desc(t, dh, t, P.data_ptr(), t, v_ptr, ld, ctx.data_ptr(), d,
                               batch=(b, h), a_bs=s_bs, b_bs=bs, c_bs=(t * d, dh),
                               precision=prec, causal=ops.CAUSAL_K_UPTO), dev, stream)
    dO = torch.randn(b * t, d, device=cuda)
    # dV = P^T dO (k >= row)
    dV = torch.empty(b * t, d, device=cuda)
    ops.gemm_run(ops.gemm_desc(t, dh, t, P.data_ptr(), t, dO.data_ptr(), d, dV.data_ptr(), d,
                               a_t=True, batch=(b, h), a_bs=s_bs, b_bs=(t * d, dh),
                               c_bs=(t * d, dh), precision=prec, causal=ops.CAUSAL_K_FROM),
                 dev, stream)
    # dP = dO V^T (lower tiles)
    dP = torch.empty_like(S)
    ops.gemm_run(ops.gemm_desc(t, t, dh, dO.data_ptr(), d, v_ptr, ld, dP.data_ptr(), t,
                               b_t=True, batch=(b, h), a_bs=(t * d, dh), b_bs=bs, c_bs=s_bs,
                               precision=prec, causal=ops.CAUSAL_LOWER), dev, stream)
    dS = ops.causal_softmax_backward(dP, P, 1.0 / np.sqrt(dh), zero_fill_block=128)
    # dQ = dS K (k <= row), dK = dS^T Q (k >= row)
    dQ = torch.empty(b * t, d, device=cuda)
    dK = torch.empty(b * t, d, device=cuda)
    ops.gemm_run(ops.gemm_desc(t, dh, t, dS.data_ptr(), t, k_ptr, ld, dQ.data_ptr(), d,
                               batch=(b, h), a_bs=s_bs, b_bs=bs, c_bs=(t * d, dh),
                               precision=prec, causal=ops.CAUSAL_K_UPTO), dev, stream)
    ops.gemm_run(ops.gemm_desc(t, dh, t, dS.data_ptr(), t, q_ptr, ld, dK.data_ptr(), d,
                               a_t=True, batch=(b, h), a_bs=s_bs, b_bs=bs, c_bs=(t * d, dh),
                               precision=prec, causal=ops.CAUSAL_K_FROM), dev, stream)
    torch.cuda.synchronize()
    assert ops.gemm_error(0) == 0

    def heads(x):
        return x.reshape(b, t, h, dh).transpose(0, 2, 1, 3).astype(np.float64)

    q = heads(qkv[:, :d])
    k = heads(qkv[:, d:2 * d])
    v = heads(qkv[:, 2 * d:])
    mask = np.triu(np.ones((t, t), bool), 1)
    s = np.where(mask, -np.inf, q @ k.transpose(0, 1, 3, 2) / np.sqrt(dh))
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    o = p @ v
    do = heads(dO.cpu().numpy())
    dv = p.transpose(0, 1, 3, 2) @ do
    dp = do @ v.transpose(0, 1, 3, 2)
    ds = p * (dp - (dp * p).sum(-1, keepdims=True)) / np.sqrt(dh)
    dq = ds @ k
    dk = ds.transpose(0, 1, 3, 2) @ q
    merge = lambda x: x.transpose(0, 2, 1, 3).reshape(b * t, d)
    lower = ~mask
    assert rel_err(np.where(lower, S.cpu().numpy(), 0), np.where(lower, q @ k.transpose(0, 1, 3, 2), 0)) <= 1e-5
    assert rel_err(ctx.cpu().numpy(), merge(o)) <= 1e-5
    assert rel_err(dV.cpu().numpy(), merge(dv)) <= 1e-5
    assert rel_err(dQ.cpu().numpy(), merge(dq)) <= 1e-5
    assert rel_err(dK.cpu().numpy(), merge(dk)) <= 1e-5


def test_gemm_invalid_arguments(cuda):
    import torch
    from spar_b200 import ops
    from spar_b200._lib import SparError

    a = torch.randn(64, 64, device=cuda)
    with pytest.raises(SparError) as e:
        ops.gemm_run(ops.gemm_desc(64, 64, 0, a.data_ptr(), 64, a.data_ptr(), 64, a.data_ptr(), 64),
                     0, 0)
    assert e.value.code == 1
    with pytest.raises(SparError):  # unaligned leading dimension
        ops.gemm_run(ops.gemm_desc(64, 64, 62, a.data_ptr(), 62, a.data_ptr(), 64, a.data_ptr(), 64),
                     0, 0)


def test_gemm_rope_epilogue(cuda):
    """RoPE in the epilogue (fused QKV projection: q and k thirds rotated, v not) equals the
    GEMM followed by the standalone rotation kernel."""
    import torch
    from spar_b200 import ops

    b, t, h, dh = 2, 96, 4, 32
    d = h * dh
    r = np.random.default_rng(21)
    x = torch.from_numpy(r.standard_normal((b * t, d)).astype(np.float32)).to(cuda)
    w = torch.from_numpy((0.05 * r.standard_normal((d, 3 * d))).astype(np.float32)).to(cuda)
    bias = torch.from_numpy(r.standard_normal(3 * d).astype(np.float32)).to(cuda)
    tab = ops.rope_table(t, dh, 10000.0, device=cuda)
    for prec in (ops.TF32, ops.TF32X3):
        fused = ops.matmul(x, w, epilogue=ops.EPI_BIAS, bias=bias, precision=prec,
                           rope=(tab, t, dh, 2 * d))
        plain = ops.matmul(x, w, epilogue=ops.EPI_BIAS, bias=bias, precision=prec)
        ops.rope_apply_(plain, tab, b, t, 2 * h, dh, 3 * d)
        torch.cuda.synchronize()
        assert ops.gemm_error(0) == 0
        np.testing.assert_allclose(fused.cpu().numpy(), plain.cpu().numpy(), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("shape", [(4096, 3072, 288), (16384, 1024, 288), (6144, 1000, 160)])
@pytest.mark.parametrize("epi", ["none", "bias_gelu", "bias_add"])
def test_gemm_many_tiles_per_sm_pair(cuda, epi, shape):
    """More paired tiles (256 x 256, or 256 x 128 for the narrower outputs) than SM pairs, so every
    persistent CTA pair runs several tiles and cycles both TMEM accumulators and the operand-stage
    ring (plain and eight-warp epilogues; a ragged N on the last shape)."""
    import torch
    from spar_b200 import ops
    from oracle import spar_oracle as O

    m, n, k = shape
    a, b, ref = _mats(m, n, k, False, False, seed=23)
    at, bt = torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)
    r = np.random.default_rng(24)
    bias = r.standard_normal(n).astype(np.float32)
    aux = r.standard_normal((m, n)).astype(np.float32)
    biast, auxt = torch.from_numpy(bias).to(cuda), torch.from_numpy(aux).to(cuda)
    if epi == "none":
        c = ops.matmul(at, bt)
        expect = ref
    elif epi == "bias_gelu":
        c = ops.matmul(at, bt, epilogue=ops.EPI_BIAS_GELU, bias=biast, aux=auxt)
        expect = O.gelu_forward(ref + bias, np.float64)
    else:
        c = ops.matmul(at, bt, epilogue=ops.EPI_BIAS_ADD, bias=biast, aux=auxt)
        expect = ref + bias + aux
    torch.cuda.synchronize()
    assert ops.gemm_error(0) == 0
    assert rel_l2(c.cpu().numpy(), expect) <= 2e-3


@pytest.mark.parametrize("epi", ["bias", "bias_gelu", "gelu_bwd", "bias_add", "rope_round", "accumulate"])
def test_gemm_split_k_with_epilogues(cuda, epi):
    """Few output tiles and a long K: the product is split along K and the reduction kernel
    applies the epilogue. Same results as the unsplit definition (fp64 reference)."""
    import torch
    from spar_b200 import ops
    from oracle import spar_oracle as O

    m, n, k = 512, 512, 8192
    a, b, ref = _mats(m, n, k, False, False, seed=31)
    at, bt = torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)
    r = np.random.default_rng(32)
    bias = r.standard_normal(n).astype(np.float32)
    aux = r.standard_normal((m, n)).astype(np.float32)
    biast, auxt = torch.from_numpy(bias).to(cuda), torch.from_numpy(aux).to(cuda)
    tol = 2e-3
    if epi == "bias":
        got = ops.matmul(at, bt, epilogue=ops.EPI_BIAS, bias=biast)
        expect = ref + bias
    elif epi == "bias_gelu":
        pre = torch.empty(m, n, device=cuda)
        got = ops.matmul(at, bt, epilogue=ops.EPI_BIAS_GELU, bias=biast, aux=pre)
        torch.cuda.synchronize()
        assert rel_l2(pre.cpu().numpy(), ref + bias) <= tol
        expect = O.gelu_forward(ref + bias, np.float64)
    elif epi == "gelu_bwd":
        got = ops.matmul(at, bt, epilogue=ops.EPI_GELU_BWD, aux=auxt)
        expect = ref * O.gelu_derivative(aux)
    elif epi == "bias_add":
        got = ops.matmul(at, bt, epilogue=ops.EPI_BIAS_ADD, bias=biast, aux=auxt)
        expect = ref + bias + aux
    elif epi == "rope_round":
        t, dh = 128, 64
        tab = ops.rope_table(t, dh, 10000.0, device=cuda)
        got = ops.matmul(at, bt, epilogue=ops.EPI_BIAS, bias=biast, round_output=True,
                         rope=(tab, t, dh, 256))
        plain = ops.matmul(at, bt, epilogue=ops.EPI_BIAS, bias=biast)
        ops.rope_apply_(plain, tab, m // t, t, 4, dh, n)
        torch.cuda.synchronize()
        g = got.cpu().numpy()
        assert np.array_equal(g.view(np.uint32) & 0x1FFF, np.zeros_like(g.view(np.uint32)))
        expect = plain.cpu().numpy().astype(np.float64)
    else:
        got = auxt.clone()
        ops.matmul(at, bt, out=got, accumulate=True, alpha=0.25)
        expect = 0.25 * ref + aux
    torch.cuda.synchronize()
    assert ops.gemm_error(0) == 0
    assert rel_l2(got.cpu().numpy(), expect) <= tol


@pytest.mark.parametrize("dtype", [0, 1])  # SPAR_CUDA_FLOAT32, SPAR_CUDA_FLOAT64
@pytest.mark.parametrize("shape", [(3, 128, 64, 96), (2, 5, 7, 3), (4, 33, 17, 9), (1, 300, 1, 1),
                                   (6, 64, 64, 64), (2, 1, 130, 3)])
def test_contiguous_matmul_any_shape(cuda, shape, dtype):
    """spar_b200_matmul, the body behind Spar's cuda_blas seam: batched contiguous products of any
    shape (k or n not a multiple of 4 go through zero-padded staging), float32 in both precisions
    against float64, float64 (SIMT kernel) to double rounding."""
    import torch
    from spar_b200 import _lib

    lib = _lib.load()
    batch, m, k, n = shape
    r = np.random.default_rng(sum(shape) + dtype)
    npt = np.float32 if dtype == 0 else np.float64
    a = r.standard_normal((batch, m, k)).astype(npt)
    b = r.standard_normal((batch, k, n)).astype(npt)
    ref = np.einsum("bmk,bkn->bmn", a.astype(np.float64), b.astype(np.float64))
    ga, gb = torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)
    for precision, tol in ((0, 2e-3), (1, 1e-5)) if dtype == 0 else ((0, 1e-13),):
        gc = torch.full((batch, m, n), float("nan"), dtype=ga.dtype, device=cuda)
        st = lib.spar_b200_matmul(ga.data_ptr(), gb.data_ptr(), gc.data_ptr(), batch, m, k, n,
                                  dtype, precision, 0, None)
        assert st.code == 0
        torch.cuda.synchronize()
        assert rel_l2(gc.cpu().numpy(), ref) <= tol, (precision, rel_l2(gc.cpu().numpy(), ref))
    # k == 0: zeros, as the reference seam returns
    gc = torch.full((batch, m, n), 5.0, dtype=ga.dtype, device=cuda)
    assert lib.spar_b200_matmul(ga.data_ptr(), gb.data_ptr(), gc.data_ptr(), batch, m, 0, n, dtype,
                                1, 0, None).code == 0
    torch.cuda.synchronize()
    assert not gc.cpu().numpy().any()


@pytest.mark.parametrize("precision", [0, 1])
@pytest.mark.parametrize("epi", ["gelu_bwd", "bias", "none"])
@pytest.mark.parametrize("shape", [(2048, 4096, 1024), (300, 200, 96), (16384, 3072, 256),
                                   (256, 300, 8192)])
def test_gemm_column_partials(cuda, shape, epi, precision):
    """The epilogue's per-32-row column sums (the bias gradient of a product without re-reading
    its output): their row sums equal the column sums of C (float64 reference) to fp32
    summation error, whatever tile kernel and epilogue the plan picks. With a K split (3xTF32
    past 512 concatenated K elements; the last shape in either precision) the reduction kernel
    writes them."""
    import torch
    from spar_b200 import ops

    m, n, k = shape
    r = np.random.default_rng(m + n + k)
    a = torch.from_numpy(r.standard_normal((m, k)).astype(np.float32)).to(cuda)
    b = torch.from_numpy((0.02 * r.standard_normal((k, n))).astype(np.float32)).to(cuda)
    bias = torch.from_numpy(r.standard_normal(n).astype(np.float32)).to(cuda)
    aux = torch.from_numpy(r.standard_normal((m, n)).astype(np.float32)).to(cuda)
    e = {"gelu_bwd": ops.EPI_GELU_BWD, "bias": ops.EPI_BIAS, "none": ops.EPI_NONE}[epi]
    parts = torch.full(((m + 31) // 32, n), float("nan"), device=cuda)
    c = ops.matmul(a, b, epilogue=e, bias=bias if epi == "bias" else None,
                   aux=aux if epi == "gelu_bwd" else None, precision=precision,
                   column_partials=parts)
    torch.cuda.synchronize()
    assert ops.gemm_error(0) == 0
    got = parts.cpu().numpy().astype(np.float64).sum(0)
    want = c.cpu().numpy().astype(np.float64).sum(0)
    scale = np.abs(c.cpu().numpy()).astype(np.float64).sum(0)
    assert np.all(np.abs(got - want) <= 1e-5 * scale + 1e-30)


@pytest.mark.parametrize("precision,accumulate", [(0, False), (1, False), (1, True)])
def test_gemm_split_k_ragged_columns(cuda, precision, accumulate):
    """A product whose column count is not a multiple of 4, stored with a padded row stride (the
    tied LM head: logits [tokens, vocab] in rows of the padded vocabulary), K split in 3xTF32.
    Every column up to n is written, the bias included; the padding past the 16-byte chunk that
    holds column n - 1 is untouched (tile stores write whole 16-byte chunks)."""
    import torch
    from spar_b200 import ops

    m, n, k, ldc = 256, 301, 8192, 320
    a, b, ref = _mats(m, n, k, False, True, seed=41)
    bias = np.random.default_rng(42).standard_normal(n).astype(np.float32)
    prev = np.random.default_rng(43).standard_normal((m, n)).astype(np.float32)
    at, bt = torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)
    biast = torch.from_numpy(bias).to(cuda)
    c = torch.full((m, ldc), float("nan"), device=cuda)
    if accumulate:
        c[:, :n] = torch.from_numpy(prev).to(cuda)
    desc = ops.gemm_desc(m, n, k, at.data_ptr(), k, bt.data_ptr(), k, c.data_ptr(), ldc, b_t=True,
                         accumulate=accumulate, epilogue=ops.EPI_BIAS, bias=biast.data_ptr(),
                         precision=precision)
    ops.gemm_run(desc, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert ops.gemm_error(0) == 0
    got = c.cpu().numpy()
    assert np.isnan(got[:, (n + 3) // 4 * 4:]).all()  # padding untouched
    expect = ref + bias + (prev if accumulate else 0.0)
    assert not np.isnan(got[:, :n]).any()
    assert rel_l2(got[:, :n], expect) <= (1e-5 if precision else 2e-3)
