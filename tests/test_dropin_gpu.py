"""The drop-in backend ABI (include/spar_cuda_kernels.h) on the GPU, against the reference's own
CUDA backend.

Every spar_cuda_* entry point of libspar_b200.so (spar_b200/csrc/compat.cu) is called on the same
device buffers as the same entry point of the reference's unchanged backend
(src/backend/cuda_kernels.cu, compiled from its sources into oracle/_ref/libspar_ref_stock.so by
oracle/make_ref.py, the checker here), for float32 and float64, int32 and int64 indices, and the
special cases the reference defines: NaN, all -inf and +inf slices of softmax / log-softmax
(cuda_kernels.cu:529-617), out-of-range embedding indices and class targets (the invalid flags,
:313-324, :619-630), non-finite gradient norms (:367-433). Results must be bitwise equal where
both sides do the same IEEE operations in the same order, and within a few units in the last
place where the order of a reduction or an atomic scatter differs (stated per test).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32, F64, I32, I64 = 0, 1, 2, 3
DT = {F32: np.float32, F64: np.float64}


@pytest.fixture(scope="module")
def libs(cuda):
    from oracle import cpu_ref
    from spar_b200 import _lib

    if not cpu_ref.available("stock"):
        pytest.skip("reference GPU build absent (python oracle/make_ref.py --variant stock)")
    prod = _lib.load()
    ref = ctypes.CDLL(str(cpu_ref.VARIANT_LIBS["stock"]))
    # Both libraries get the same ctypes signatures (pointers as 64-bit, sizes as uint64): a call
    # without them would pass pointers as 32-bit C ints.
    table = {**_lib.SIGNATURES, **_lib.EXTRA_SIGNATURES}
    names = [n for n in table if n.startswith("spar_cuda_")]
    assert len(names) == 23
    for name in names:
        fn = getattr(ref, name)
        fn.restype, fn.argtypes = table[name]
        assert getattr(prod, name).argtypes is not None
    return prod, ref


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _both(libs, name, make_args, outs):
    """Runs `name` in both libraries. make_args(out_tensors) -> argument tuple; `outs` are host
    arrays giving each output's initial contents. Returns ([ours], [reference]) host arrays."""
    results = []
    for lib in libs:
        fn = getattr(lib, name)
        assert fn.argtypes is not None and fn.restype is not None, name
        dev = [_dev(o.copy()) for o in outs]
        st = fn(*make_args(dev))
        assert (st.code, st.cuda_error) == (0, 0), (name, st.code, st.cuda_error)
        results.append([d.cpu().numpy() for d in dev])
    return results


def _ptr(t):
    return t.data_ptr()


def _same(a, b):
    np.testing.assert_array_equal(a, b)


def _close(a, b, rtol):
    a64, b64 = np.asarray(a, np.float64), np.asarray(b, np.float64)
    assert np.array_equal(np.isnan(a64), np.isnan(b64))
    fin = np.isfinite(b64)
    assert np.array_equal(a64[~fin & ~np.isnan(b64)], b64[~fin & ~np.isnan(b64)])
    scale = max(np.abs(b64[fin]).max(initial=0.0), 1e-300)
    assert np.abs(a64[fin] - b64[fin]).max(initial=0.0) <= rtol * scale


RTOL = {F32: 2e-6, F64: 1e-14}


@pytest.mark.parametrize("dtype", [F32, F64])
def test_binary_scalar_unary(libs, dtype):
    r = np.random.default_rng(1 + dtype)
    n = (1 << 18) + 13
    x = r.standard_normal(n).astype(DT[dtype])
    y = r.standard_normal(n).astype(DT[dtype])
    y[::97] = 0.0  # division by zero -> +-inf / NaN on both sides
    gx, gy = _dev(x), _dev(y)
    for op in range(4):
        ours, ref = _both(libs, "spar_cuda_launch_binary",
                          lambda o: (_ptr(o[0]), _ptr(gx), _ptr(gy), n, dtype, op, 0),
                          [np.zeros(n, DT[dtype])])
        _same(ours[0], ref[0])
        ours, ref = _both(libs, "spar_cuda_launch_scalar",
                          lambda o: (_ptr(o[0]), _ptr(gx), n, dtype, op, 0.3700000001, 0),
                          [np.zeros(n, DT[dtype])])
        _same(ours[0], ref[0])
    z = x * 30.0  # exp overflow / sigmoid tails; log / sqrt of negatives and zero -> NaN / -inf
    z[::101] = 0.0
    gz = _dev(z)
    for op in range(8):
        ours, ref = _both(libs, "spar_cuda_launch_unary",
                          lambda o: (_ptr(o[0]), _ptr(gz), n, dtype, op, 0),
                          [np.zeros(n, DT[dtype])])
        _close(ours[0], ref[0], RTOL[dtype])


@pytest.mark.parametrize("dtype", [F32, F64])
def test_reductions(libs, dtype):
    r = np.random.default_rng(3 + dtype)
    n = 1_000_003
    x = r.standard_normal(n).astype(DT[dtype])
    gx = _dev(x)
    for op in range(3):
        ours, ref = _both(libs, "spar_cuda_launch_reduction",
                          lambda o: (_ptr(o[0]), _ptr(gx), n, dtype, op, 0), [np.zeros(1, DT[dtype])])
        if op == 2:
            _same(ours[0], ref[0])
        else:  # summation order differs: relative to the sum of magnitudes
            bound = (1e-6 if dtype == F32 else 1e-14) * np.abs(x).sum() / (n if op == 1 else 1)
            assert abs(float(ours[0][0]) - float(ref[0][0])) <= bound
    x[12345] = np.nan  # max propagates NaN
    gx = _dev(x)
    ours, ref = _both(libs, "spar_cuda_launch_reduction",
                      lambda o: (_ptr(o[0]), _ptr(gx), n, dtype, 2, 0), [np.zeros(1, DT[dtype])])
    assert np.isnan(ours[0][0]) and np.isnan(ref[0][0])
    rows, cols = 3001, 777
    m = r.standard_normal((rows, cols)).astype(DT[dtype])
    gm = _dev(m)
    for op in (0, 1):
        ours, ref = _both(libs, "spar_cuda_launch_row_reduction",
                          lambda o: (_ptr(o[0]), _ptr(gm), rows, cols, dtype, op, 0),
                          [np.zeros(rows, DT[dtype])])
        _close(ours[0], ref[0], 5 * RTOL[dtype])


@pytest.mark.parametrize("dtype", [F32, F64])
@pytest.mark.parametrize("logarithmic", [0, 1])
def test_probability_forward_backward_special_slices(libs, dtype, logarithmic):
    """softmax / log_softmax along the middle axis of (outer, axis, inner), with a NaN slice, an
    all -inf slice and slices holding one and two +inf entries (reference special cases)."""
    r = np.random.default_rng(5 + dtype + 2 * logarithmic)
    outer, axis, inner = 37, 300, 5
    x = (3 * r.standard_normal((outer, axis, inner))).astype(DT[dtype])
    x[0, 17, 0] = np.nan
    x[1, :, 1] = -np.inf
    x[2, 5, 2] = np.inf
    x[3, 5, 3] = np.inf
    x[3, 250, 3] = np.inf
    x[4, :100, 4] = -np.inf  # partially masked slice stays ordinary
    gx = _dev(x)
    slices = outer * inner
    ours, ref = _both(libs, "spar_cuda_launch_probability_forward",
                      lambda o: (_ptr(o[0]), _ptr(o[1]), _ptr(gx), outer, axis, inner, dtype,
                                 logarithmic, 0),
                      [np.zeros_like(x), np.zeros(slices, np.int32)])
    _same(ours[1], ref[1])
    _close(ours[0], ref[0], 4 * RTOL[dtype])
    y, undefined = _dev(ref[0]), _dev(ref[1])
    g = _dev(r.standard_normal(x.shape).astype(DT[dtype]))
    ours, ref = _both(libs, "spar_cuda_launch_probability_backward",
                      lambda o: (_ptr(o[0]), _ptr(g), _ptr(y), _ptr(undefined), outer, axis, inner,
                                 dtype, logarithmic, 0),
                      [np.zeros_like(x)])
    _close(ours[0], ref[0], 8 * RTOL[dtype])


@pytest.mark.parametrize("index_dtype", [I32, I64])
@pytest.mark.parametrize("dtype", [F32, F64])
def test_embedding_and_targets(libs, dtype, index_dtype):
    r = np.random.default_rng(7 + dtype + 2 * index_dtype)
    vocab, dim, count = 1000, 96, 4096
    idx_np = np.int32 if index_dtype == I32 else np.int64
    ids = r.integers(0, vocab, count).astype(idx_np)
    w = r.standard_normal((vocab, dim)).astype(DT[dtype])
    gw, gi = _dev(w), _dev(ids)
    ours, ref = _both(libs, "spar_cuda_launch_validate_embedding_indices",
                      lambda o: (_ptr(o[0]), _ptr(gi), count, vocab, index_dtype, 0),
                      [np.zeros(1, np.int32)])
    assert ours[0][0] == ref[0][0] == 0
    ours, ref = _both(libs, "spar_cuda_launch_embedding_forward",
                      lambda o: (_ptr(o[0]), _ptr(o[1]), _ptr(gw), _ptr(gi), count, vocab, dim,
                                 dtype, index_dtype, 0),
                      [np.zeros((count, dim), DT[dtype]), np.zeros(1, np.int32)])
    _same(ours[0], ref[0])
    _same(ours[1], ref[1])
    grad = _dev(r.standard_normal((count, dim)).astype(DT[dtype]))
    ours, ref = _both(libs, "spar_cuda_launch_embedding_backward",
                      lambda o: (_ptr(o[0]), _ptr(grad), _ptr(gi), count, dim, dtype, index_dtype,
                                 0),
                      [np.zeros((vocab, dim), DT[dtype])])
    _close(ours[0], ref[0], 20 * RTOL[dtype])  # atomic scatter order differs
    bad = ids.copy()
    bad[77] = vocab + 5
    bad[99] = -1
    gb = _dev(bad)
    ours, ref = _both(libs, "spar_cuda_launch_validate_embedding_indices",
                      lambda o: (_ptr(o[0]), _ptr(gb), count, vocab, index_dtype, 0),
                      [np.zeros(1, np.int32)])
    assert ours[0][0] == ref[0][0] == 1
    # validate_targets reports through a HOST int32 (the reference copies its flag back).
    for ids_dev, want in ((gi, 0), (gb, 1)):
        for lib in libs:
            flag = ctypes.c_int32(7)
            st = lib.spar_cuda_validate_targets(ctypes.byref(flag), _ptr(ids_dev), count, vocab,
                                                index_dtype, 0)
            assert (st.code, flag.value) == (0, want)


@pytest.mark.parametrize("language_model", [0, 1])
@pytest.mark.parametrize("index_dtype", [I32, I64])
@pytest.mark.parametrize("dtype", [F32, F64])
def test_nll_forward_backward(libs, dtype, index_dtype, language_model):
    r = np.random.default_rng(11 + dtype + 2 * index_dtype + 4 * language_model)
    classes, batch, seq = 513, 6, 33
    rows = batch * seq
    logp = r.standard_normal((rows, classes)).astype(DT[dtype])
    targets = r.integers(0, classes, rows).astype(np.int32 if index_dtype == I32 else np.int64)
    out_count = batch * (seq - 1) if language_model else rows
    gl, gt = _dev(logp), _dev(targets)
    ours, ref = _both(libs, "spar_cuda_launch_nll_forward",
                      lambda o: (_ptr(o[0]), _ptr(gl), _ptr(gt), out_count, classes,
                                 seq if language_model else 0, dtype, index_dtype, language_model, 0),
                      [np.zeros(out_count, DT[dtype])])
    _same(ours[0], ref[0])
    g = _dev(r.standard_normal(out_count).astype(DT[dtype]))
    ours, ref = _both(libs, "spar_cuda_launch_nll_backward",
                      lambda o: (_ptr(o[0]), _ptr(g), _ptr(gt), out_count, classes,
                                 seq if language_model else 0, dtype, index_dtype, language_model, 0),
                      [np.zeros((rows, classes), DT[dtype])])
    _same(ours[0], ref[0])


@pytest.mark.parametrize("dtype", [F32, F64])
def test_rope_mask_fill_copy(libs, dtype):
    r = np.random.default_rng(13 + dtype)
    b, t, d = 3, 129, 64
    x = r.standard_normal((b, t, d)).astype(DT[dtype])
    gx = _dev(x)
    for inverse in (0, 1):
        ours, ref = _both(libs, "spar_cuda_launch_rope",
                          lambda o: (_ptr(o[0]), _ptr(gx), b * t * d // 2, t, d, 7, 10000.0, dtype,
                                     inverse, 0),
                          [np.zeros_like(x)])
        _close(ours[0], ref[0], 4 * RTOL[dtype])
    ours, ref = _both(libs, "spar_cuda_launch_causal_mask", lambda o: (_ptr(o[0]), 77, dtype, 0),
                      [np.zeros((77, 77), DT[dtype])])
    _same(ours[0], ref[0])
    scalar = _dev(np.array([1.75], DT[dtype]))
    ours, ref = _both(libs, "spar_cuda_launch_fill_from_scalar",
                      lambda o: (_ptr(o[0]), _ptr(scalar), 5003, dtype, 0.125, 0),
                      [np.zeros(5003, DT[dtype])])
    _same(ours[0], ref[0])
    src = _dev(r.standard_normal(5003).astype(DT[dtype]))
    start = r.standard_normal(5003).astype(DT[dtype])
    ours, ref = _both(libs, "spar_cuda_launch_add_in_place",
                      lambda o: (_ptr(o[0]), _ptr(src), 5003, dtype, 0), [start])
    _same(ours[0], ref[0])
    ours, ref = _both(libs, "spar_cuda_launch_scale_in_place",
                      lambda o: (_ptr(o[0]), 5003, dtype, 0.3, 0), [start])
    _same(ours[0], ref[0])


@pytest.mark.parametrize("element_size", [4, 8])
def test_strided_copy_and_broadcast_reduce(libs, element_size):
    """strided_copy of a permuted, offset view (rank 4); broadcast_reduce of a [4, 5, 6, 7]
    gradient onto [5, 1, 7] (leading dimension dropped, one dimension broadcast)."""
    r = np.random.default_rng(17 + element_size)
    dtype = F32 if element_size == 4 else F64
    base = r.standard_normal(4 * 5 * 6 * 7 + 11).astype(DT[dtype])
    gb = _dev(base)
    ext = (ctypes.c_uint64 * 4)(7, 6, 5, 4)  # a permuted view of a [4, 5, 6, 7] tensor at offset 11
    strides = (ctypes.c_uint64 * 4)(1, 7, 42, 210)
    count = 4 * 5 * 6 * 7
    ours, ref = _both(libs, "spar_cuda_launch_strided_copy",
                      lambda o: (_ptr(o[0]), _ptr(gb), 4, ext, strides, 11, count, element_size, 0),
                      [np.zeros(count, DT[dtype])])
    _same(ours[0], ref[0])
    grad = _dev(r.standard_normal((4, 5, 6, 7)).astype(DT[dtype]))
    gext = (ctypes.c_uint64 * 4)(4, 5, 6, 7)
    oext = (ctypes.c_uint64 * 3)(5, 1, 7)
    ostr = (ctypes.c_uint64 * 3)(7, 7, 1)
    # count is the GRADIENT's element count (the reference loops over gradient elements).
    ours, ref = _both(libs, "spar_cuda_launch_broadcast_reduce",
                      lambda o: (_ptr(o[0]), _ptr(grad), 4, gext, 3, oext, ostr, 4 * 5 * 6 * 7,
                                 dtype, 0),
                      [np.zeros(5 * 7, DT[dtype])])
    _close(ours[0], ref[0], 20 * RTOL[dtype])  # reduction order differs (reference: atomics)


@pytest.mark.parametrize("dtype", [F32, F64])
def test_norm_summary_and_adamw(libs, dtype):
    from spar_b200._lib import SparCudaNormSummary

    r = np.random.default_rng(19 + dtype)
    n = (1 << 20) + 3
    g = (1e-3 * r.standard_normal(n)).astype(DT[dtype])
    for lib in libs:
        assert lib.spar_cuda_gradient_norm_summary.argtypes is not None
    for case in ("finite", "inf", "nan"):
        gg = g.copy()
        if case == "inf":
            gg[1000] = np.inf
        if case == "nan":
            gg[2000] = np.nan
        dg = _dev(gg)
        sums = []
        for lib in libs:
            s = SparCudaNormSummary()
            st = lib.spar_cuda_gradient_norm_summary(ctypes.byref(s), _ptr(dg), n, dtype, 0)
            assert st.code == 0
            sums.append((s.scale, s.scaled_sum_squares, s.has_infinity, s.has_nan))
        (sa, qa, ia, na), (sb, qb, ib, nb) = sums
        assert (ia, na) == (ib, nb)
        if case == "finite":
            # The norm is scale * sqrt(scaled_sum_squares); the scale may be chosen differently.
            na_, nb_ = sa * np.sqrt(qa), sb * np.sqrt(qb)
            assert abs(na_ - nb_) <= 1e-12 * nb_
    p = r.standard_normal(n).astype(DT[dtype])
    m = (1e-3 * r.standard_normal(n)).astype(DT[dtype])
    v = (1e-6 * r.random(n)).astype(DT[dtype])
    dg = _dev(g)
    ours, ref = _both(libs, "spar_cuda_launch_adamw",
                      lambda o: (_ptr(o[0]), _ptr(dg), _ptr(o[1]), _ptr(o[2]), n, dtype, 3e-4,
                                 0.9, 0.95, 1e-8, 0.1, 1 - 0.9 ** 3, 1 - 0.95 ** 3, 0),
                      [p, m, v])
    for a, b in zip(ours, ref):
        _same(a, b)


def test_invalid_arguments_match_reference(libs):
    """Argument validation: the same calls are rejected (code 1) by both libraries."""
    prod, ref = libs
    cases = [
        ("spar_cuda_launch_binary", (1, 1, 1, 8, 7, 0, 0)),         # bad dtype
        ("spar_cuda_launch_binary", (1, 1, 1, 8, F32, 9, 0)),       # bad op
        ("spar_cuda_launch_unary", (None, 1, 8, F32, 0, 0)),        # null output
        ("spar_cuda_launch_row_reduction", (1, 1, 4, 0, F32, 1, 0)),  # mean over nothing
        ("spar_cuda_launch_rope", (1, 1, 4, 2, 3, 0, 1e4, F32, 0, 0)),  # odd feature count
        ("spar_cuda_validate_targets", (None, 1, 4, 10, I32, 0)),   # null flag
        ("spar_cuda_launch_strided_copy", (1, 1, 0, None, None, 0, 4, 2, 0)),  # element size
    ]
    for name, args in cases:
        assert getattr(prod, name).argtypes is not None and getattr(ref, name).argtypes is not None
        a, b = getattr(prod, name)(*args), getattr(ref, name)(*args)
        assert a.code == b.code == 1, (name, a.code, b.code)
