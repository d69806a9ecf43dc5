"""The allocation-free LayerNorm backward entry point, called through the C ABI.

Some callers cannot allocate device memory when they call into the library: a host whose device
memory is reserved up front by its own allocator, or a training loop that must not allocate in
the middle of a step. spar_b200_layernorm_backward_noalloc serves them from a static device
scratch array; this test checks that it returns what the allocating entry point returns, on two
calls in a row (the second with different inputs and fewer rows, so stale partial rows left in
the shared scratch by the first call would show), and that sizes beyond the scratch are rejected.
Collected last on purpose (file name) so a run that stops at the first failure has run the rest.
"""
import numpy as np
import pytest

from _util import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-5  # the per-op tolerance of the other LayerNorm tests


def _call(fn, outs, dy, x, g, mean, rstd, rows, cols, stream):
    import torch

    dx, dg, db = outs
    return fn(dx.data_ptr(), dg.data_ptr(), db.data_ptr(), dy.data_ptr(), x.data_ptr(),
              g.data_ptr(), mean.data_ptr(), rstd.data_ptr(), rows, cols, 0, 0, 0, stream)


def test_layernorm_backward_noalloc_matches_allocating_entry_point(cuda):
    import torch

    from spar_b200 import _lib, ops

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    r = np.random.default_rng(42)
    for rows, cols in ((4096, 1024), (257, 768)):
        x = torch.from_numpy(r.standard_normal((rows, cols)).astype(np.float32)).to(cuda)
        dy = torch.from_numpy(r.standard_normal((rows, cols)).astype(np.float32)).to(cuda)
        g = torch.from_numpy((1 + 0.1 * r.standard_normal(cols)).astype(np.float32)).to(cuda)
        b = torch.zeros(cols, device=cuda)
        _, mean, rstd = ops.layer_norm_forward(x, g, b)
        want = [torch.empty_like(x), torch.empty(cols, device=cuda), torch.empty(cols, device=cuda)]
        got = [torch.empty_like(x), torch.empty(cols, device=cuda), torch.empty(cols, device=cuda)]
        st = _call(lib.spar_b200_layernorm_backward, want, dy, x, g, mean, rstd, rows, cols, stream)
        assert st.code == 0
        st = _call(lib.spar_b200_layernorm_backward_noalloc, got, dy, x, g, mean, rstd, rows, cols,
                   stream)
        assert st.code == 0
        torch.cuda.synchronize()
        for a, w in zip(got, want):
            assert rel_err(a.cpu().numpy(), w.cpu().numpy()) <= TOL


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
