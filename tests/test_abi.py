"""The C-ABI library builds, loads and exports every symbol include/*.h declares
(no compute calls: runs without a GPU)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"\b(m4_[a-z0-9_]+)\s*\(", text))
    return names


def test_header_declares_the_operator_entry_points():
    names = declared_symbols()
    for name in ("m4_memread_fwd", "m4_memread_bwd", "m4_scan_fwd", "m4_scan_bwd",
                 "m4_memread_residual_bytes", "m4_scan_residual_bytes", "m4_status_string"):
        assert name in names


def test_library_exports_every_declared_symbol():
    from mamba4_b200 import _lib

    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, name
    assert lib.m4_version().decode().startswith("mamba4_b200")
    assert lib.m4_status_string(0) == b"ok"


def test_size_queries_validate_dimensions():
    from mamba4_b200 import _lib

    lib = _lib.load()
    good = _lib.MemDims(2, 100, 3, 64, 64)
    assert lib.m4_memread_residual_bytes(ctypes.byref(good)) > 0
    for bad in (_lib.MemDims(0, 100, 3, 64, 64), _lib.MemDims(2, 100, 3, 32, 64),
                _lib.MemDims(2, 100, 3, 64, 96)):
        assert lib.m4_memread_residual_bytes(ctypes.byref(bad)) == 0
    s = _lib.ScanDims(2, 100, 3, 64, 64, 32, 64, 1, 0)
    assert lib.m4_scan_residual_bytes(ctypes.byref(s)) > 0
    assert lib.m4_scan_residual_bytes(ctypes.byref(_lib.ScanDims(2, 100, 3, 64, 64, 33, 64, 1, 0))) == 0


def test_entry_points_reject_bad_arguments_without_launching():
    from mamba4_b200 import _lib

    lib = _lib.load()
    dims = _lib.MemDims(2, 100, 3, 64, 64)
    null = [None] * 12
    assert lib.m4_memread_fwd(ctypes.byref(dims), *null, None, 0, None) == 3  # M4_ERR_NULL
    bad = _lib.MemDims(2, 100, 3, 48, 64)
    assert lib.m4_memread_fwd(ctypes.byref(bad), *null, None, 0, None) == 2  # unsupported


def test_one_token_glue_rejects_bad_arguments_without_launching():
    """`m4_memmix_prep_step` / `m4_memmix_post_step` validate dimensions,
    pointer pairing and alignment before any launch. Every call here fails
    validation (the pointer value 8 is not 16-byte aligned), so no kernel
    runs and no memory is touched."""
    from mamba4_b200 import _lib

    lib = _lib.load()
    odd = 8
    good = _lib.MemMixDims(4, 1, 8, 3096, 3096, 1.0)
    post = [odd] * 12
    assert lib.m4_memmix_post_step(ctypes.byref(good), 1e-5, *post, None) == 4            # M4_ERR_ALIGN
    two = _lib.MemMixDims(4, 2, 8, 3096, 3096, 1.0)
    assert lib.m4_memmix_post_step(ctypes.byref(two), 1e-5, *post, None) == 1             # time != 1
    unpaired = list(post)
    unpaired[5] = None                                                                    # order_out
    assert lib.m4_memmix_post_step(ctypes.byref(good), 1e-5, *unpaired, None) == 1
    wide = _lib.MemMixDims(4, 1, 17, 3096 * 3, 3096 * 3, 1.0)
    assert lib.m4_memmix_post_step(ctypes.byref(wide), 1e-5, *post, None) == 2            # > 16 heads
    window = _lib.MemMixDims(4, 4, 8, 3096, 3096, 1.0)
    assert lib.m4_memmix_prep_step(ctypes.byref(window), odd, odd, odd, 0.5, *[odd] * 9, None) == 4
    ragged = _lib.MemMixDims(4, 4, 8, 3097, 3096, 1.0)
    assert lib.m4_memmix_prep_step(ctypes.byref(ragged), odd, odd, odd, 0.5, *[odd] * 9, None) == 2
    empty = _lib.MemMixDims(0, 4, 8, 3096, 3096, 1.0)
    assert lib.m4_memmix_prep_step(ctypes.byref(empty), odd, odd, odd, 0.5, *[odd] * 9, None) == 1


def test_product_path_has_no_cpu_fallback():
    import torch
    from mamba4_b200 import mamba3_fused, selective_memory_fused

    x = torch.zeros(1, 4, 1, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_memory_fused(x, x, x, torch.ones(1, 4, 1), torch.zeros(1, 4, 1), torch.ones(1, 64))
    c = torch.zeros(1, 4, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        mamba3_fused(c, c, torch.zeros(1, 4, 64), torch.zeros(1, 4, 1), torch.zeros(1, 4, 1),
                     torch.zeros(1, 4, 1), torch.zeros(1, 4, 32), q_bias=torch.ones(1, 1, 64),
                     k_bias=torch.ones(1, 1, 64))


def test_product_package_never_imports_the_oracle():
    for path in (ROOT / "mamba4_b200").rglob("*.py"):
        text = path.read_text()
        assert "import oracle" not in text and "from oracle" not in text, path
