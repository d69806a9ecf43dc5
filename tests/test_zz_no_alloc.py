"""The allocation-free LayerNorm backward entry point, called through the C ABI.

Some callers cannot allocate device memory when they call into the library: a host whose device
memory is reserved up front by its own allocator, or a training loop that must not allocate in
the middle of a step. spar_b200_layernorm_backward_noalloc serves them from a static device
scratch array; these tests check that it returns what the allocating entry point returns, on two
calls in a row (the second with different inputs and fewer rows, so stale partial rows left in
the shared scratch by the first call would show), with and without accumulation into existing
gradients, that it takes nothing from the device's stream-ordered memory pool (the pool the
allocating entry point draws its scratch from), and that sizes beyond the scratch are rejected.
Collected last on purpose (file name) so a run that stops at the first failure has run the rest.
"""
import ctypes

import numpy as np
import pytest

from _util import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-5  # the per-op tolerance of the other LayerNorm tests

CU_MEMPOOL_ATTR_USED_MEM_HIGH = 8  # cuda.h CUmemPool_attribute


def _call(fn, outs, dy, x, g, mean, rstd, rows, cols, stream, acc_params=0, acc_dx=0):
    dx, dg, db = outs
    return fn(dx.data_ptr(), dg.data_ptr(), db.data_ptr(), dy.data_ptr(), x.data_ptr(),
              g.data_ptr(), mean.data_ptr(), rstd.data_ptr(), rows, cols, acc_params, acc_dx, 0,
              stream)


def _inputs(r, rows, cols, cuda):
    import torch

    from spar_b200 import ops

    x = torch.from_numpy(r.standard_normal((rows, cols)).astype(np.float32)).to(cuda)
    dy = torch.from_numpy(r.standard_normal((rows, cols)).astype(np.float32)).to(cuda)
    g = torch.from_numpy((1 + 0.1 * r.standard_normal(cols)).astype(np.float32)).to(cuda)
    b = torch.zeros(cols, device=cuda)
    _, mean, rstd = ops.layer_norm_forward(x, g, b)
    return x, dy, g, mean, rstd


@pytest.mark.parametrize("accumulate", [0, 1])
def test_layernorm_backward_noalloc_matches_allocating_entry_point(cuda, accumulate):
    import torch

    from spar_b200 import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    r = np.random.default_rng(42 + accumulate)
    for rows, cols in ((4096, 1024), (257, 768)):
        x, dy, g, mean, rstd = _inputs(r, rows, cols, cuda)
        # With accumulation both entry points start from the same non-zero dx, dgamma, dbeta.
        start = [torch.from_numpy(r.standard_normal(s).astype(np.float32)).to(cuda)
                 for s in ((rows, cols), (cols,), (cols,))]
        want = [t.clone() for t in start]
        got = [t.clone() for t in start]
        st = _call(lib.spar_b200_layernorm_backward, want, dy, x, g, mean, rstd, rows, cols, stream,
                   accumulate, accumulate)
        assert st.code == 0
        st = _call(lib.spar_b200_layernorm_backward_noalloc, got, dy, x, g, mean, rstd, rows, cols,
                   stream, accumulate, accumulate)
        assert st.code == 0
        torch.cuda.synchronize()
        for a, w in zip(got, want):
            assert rel_err(a.cpu().numpy(), w.cpu().numpy()) <= TOL


def test_layernorm_backward_noalloc_takes_nothing_from_the_memory_pool(cuda):
    """The device's current memory pool (where cudaMallocAsync draws from) records its high-water
    mark of memory in use; reset it, call the entry point, and the mark must not move. The
    allocating entry point, called the same way, moves it (the check can see an allocation)."""
    import torch

    from spar_b200 import _lib

    lib = _lib.load()
    cu = ctypes.CDLL("libcuda.so.1")
    stream = torch.cuda.current_stream().cuda_stream
    dev = ctypes.c_int()
    assert cu.cuCtxGetDevice(ctypes.byref(dev)) == 0
    pool = ctypes.c_void_p()
    assert cu.cuDeviceGetMemPool(ctypes.byref(pool), dev) == 0

    def high_after(fn):
        torch.cuda.synchronize()
        zero = ctypes.c_uint64(0)  # setting the high-water mark to 0 resets it to the current use
        assert cu.cuMemPoolSetAttribute(pool, CU_MEMPOOL_ATTR_USED_MEM_HIGH, ctypes.byref(zero)) == 0
        before = ctypes.c_uint64()
        assert cu.cuMemPoolGetAttribute(pool, CU_MEMPOOL_ATTR_USED_MEM_HIGH,
                                        ctypes.byref(before)) == 0
        assert fn().code == 0
        torch.cuda.synchronize()
        after = ctypes.c_uint64()
        assert cu.cuMemPoolGetAttribute(pool, CU_MEMPOOL_ATTR_USED_MEM_HIGH,
                                        ctypes.byref(after)) == 0
        return after.value - before.value

    r = np.random.default_rng(7)
    rows, cols = 2048, 1024
    x, dy, g, mean, rstd = _inputs(r, rows, cols, cuda)
    outs = [torch.empty_like(x), torch.empty(cols, device=cuda), torch.empty(cols, device=cuda)]
    grown = high_after(lambda: _call(lib.spar_b200_layernorm_backward_noalloc, outs, dy, x, g, mean,
                                     rstd, rows, cols, stream))
    assert grown == 0
    control = high_after(lambda: _call(lib.spar_b200_layernorm_backward, outs, dy, x, g, mean, rstd,
                                       rows, cols, stream))
    assert control > 0


def test_layernorm_backward_noalloc_rejects_sizes_beyond_scratch(cuda):
    import torch

    from spar_b200 import _lib

    lib = _lib.load()
    cols = 4096  # the static scratch holds rows of at most 2048 columns
    t = torch.zeros(8, cols, device=cuda)
    v = torch.zeros(cols, device=cuda)
    st = _call(lib.spar_b200_layernorm_backward_noalloc, [t, v, v], t, t, v, v[:8], v[:8], 8, cols,
               torch.cuda.current_stream().cuda_stream)
    assert st.code == 1
