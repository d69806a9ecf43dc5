"""CPU checks of the C ABI boundary: the library loads and exports every entry point that
include/*.h declares, and argument validation rejects bad calls without touching a GPU."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(spar_(?:cuda|b200)_\w+)\s*\(", text))
    return sorted(names)


def test_headers_declare_entry_points():
    names = _declared()
    assert "spar_cuda_launch_adamw" in names and "spar_b200_gemm" in names
    assert len([n for n in names if n.startswith("spar_cuda_")]) == 23


def test_library_exports_every_declared_symbol():
    from spar_b200 import _lib

    lib = _lib.load()
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_binding_table_matches_headers():
    from spar_b200 import _lib

    bound = set(_lib.exported_symbols())
    missing = [n for n in _declared() if n not in bound]
    assert not missing, f"no ctypes signature for: {missing}"


def test_invalid_arguments_rejected_without_gpu():
    """Argument validation runs before any CUDA call (reference convention: code 1)."""
    from spar_b200 import _lib, ops

    lib = _lib.load()
    st = lib.spar_b200_layernorm_forward(None, None, None, None, None, None, 4, 6, 1e-5, 0, None)
    assert st.code == 1  # cols not a multiple of 4
    st = lib.spar_b200_gemm(ctypes.byref(ops.gemm_desc(0, 0, 0, None, 0, None, 0, None, 0)), 0, None)
    assert st.code == 1
    st = lib.spar_b200_adamw_clipped(None, 0, None, 1.0, 1e-3, 0.9, 0.999, 1e-8, 0.0, 1, None, 0,
                                     None)
    assert st.code == 1
    st = lib.spar_b200_cross_entropy_forward_backward(None, None, None, None, 8, 4, 4, 1, 1.0, None,
                                                      0, None)
    assert st.code == 1


def test_layernorm_backward_rejects_misaligned_pointers_without_gpu():
    """The LayerNorm backward reads x, dy, gamma and writes dx as float4: a base pointer that is
    not 16-byte aligned is an invalid argument (code 1), checked before any CUDA call."""
    from spar_b200 import _lib

    lib = _lib.load()
    good, bad = 1 << 20, (1 << 20) + 4  # never dereferenced: validation fails first
    for fn in (lib.spar_b200_layernorm_backward, lib.spar_b200_layernorm_backward_noalloc):
        for k in range(4):  # dx, dy, x, gamma in turn
            ptrs = [good] * 4
            ptrs[k] = bad
            dx, dy, x, g = ptrs
            st = fn(dx, good, good, dy, x, g, good, good, 8, 64, 0, 0, 0, None)
            assert st.code == 1, (fn, k)


def test_zero_count_calls_succeed():
    """Zero-count calls return success without launching (reference cuda_kernels.cu convention)."""
    from spar_b200 import _lib

    lib = _lib.load()
    assert lib.spar_b200_gelu_forward(None, None, 0, 0, None).code == 0
    assert lib.spar_b200_layernorm_forward(None, None, None, None, None, None, 0, 8, 1e-5, 0,
                                           None).code == 0
    assert lib.spar_b200_causal_softmax_forward(None, None, 0, 16, 16, 1.0, 0, 0, None).code == 0


def test_error_string_and_version():
    from spar_b200 import _lib

    lib = _lib.load()
    if hasattr(lib, "spar_cuda_error_string"):
        assert lib.spar_cuda_error_string(0)
    if hasattr(lib, "spar_b200_version"):
        assert b"spar_b200" in lib.spar_b200_version()


def test_product_does_not_import_oracle():
    """The product package must never route through the CPU oracle."""
    for p in (ROOT / "spar_b200").rglob("*.py"):
        src = p.read_text()
        assert not re.search(r"^\s*(from|import)\s+oracle", src, re.M), p


if __name__ == "__main__":
    pytest.main([__file__])


def test_warmup_cosine_entry_point_matches_reference_fixture():
    """spar_b200_warmup_cosine reproduces the reference schedule bit for bit."""
    import numpy as np

    from spar_b200.lm import warmup_cosine

    f = np.load(ROOT / "tests" / "golden" / "schedule.npz")
    for s, lr in zip(f["steps"], f["lr"]):
        assert warmup_cosine(3e-4, 3e-5, 100, 900, int(s)) == lr
