"""ctypes binding of the C ABI declared in include/mamba4_b200.h.

The shared library is built in-tree by `mamba4_b200.build`. There is no
fallback: if the library is missing or a call returns a nonzero status, the
caller gets an exception.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIBRARY_PATH = _HERE / "libmamba4_b200.so"

_c_int = ctypes.c_int
_p = ctypes.c_void_p
_size = ctypes.c_size_t


class MemDims(ctypes.Structure):
    """M4MemDims."""

    _fields_ = [("batch", _c_int), ("time", _c_int), ("heads", _c_int),
                ("key_dim", _c_int), ("value_dim", _c_int)]


class ScanDims(ctypes.Structure):
    """M4ScanDims."""

    _fields_ = [("batch", _c_int), ("time", _c_int), ("heads", _c_int),
                ("head_dim", _c_int), ("state_dim", _c_int), ("angle_count", _c_int),
                ("chunk", _c_int), ("bf16", _c_int), ("per_head", _c_int)]


class MixerDims(ctypes.Structure):
    """M4MixerDims."""

    _fields_ = [("rows", _c_int), ("inner", _c_int), ("heads", _c_int), ("angles", _c_int),
                ("eps", ctypes.c_float), ("stride", _c_int), ("state_dim", _c_int)]


class MemMixDims(ctypes.Structure):
    """M4MemMixDims."""

    _fields_ = [("batch", _c_int), ("time", _c_int), ("heads", _c_int), ("stride", _c_int),
                ("gate_stride", _c_int), ("beta_max", ctypes.c_float)]


# Exported symbols and their signatures (argtypes, restype).
SIGNATURES = {
    "m4_memread_residual_bytes": ([ctypes.POINTER(MemDims)], _size),
    "m4_memread_workspace_bytes": ([ctypes.POINTER(MemDims)], _size),
    "m4_memread_fwd": ([ctypes.POINTER(MemDims)] + [_p] * 12 + [_p, _size, _p], _c_int),
    "m4_memread_bwd": ([ctypes.POINTER(MemDims)] + [_p] * 9 + [_size] + [_p] * 12
                       + [_p, _size, _p], _c_int),
    "m4_memread_decode": ([ctypes.POINTER(MemDims)] + [_p] * 12 + [_p], _c_int),
    "m4_spd_solve_factor_bytes": ([_c_int, _c_int], _size),
    "m4_spd_solve_fwd": ([_c_int, _c_int] + [_p] * 4 + [_size, _p], _c_int),
    "m4_spd_solve_bwd": ([_c_int, _c_int, _p, _size] + [_p] * 4 + [_p], _c_int),
    "m4_scan_residual_bytes": ([ctypes.POINTER(ScanDims)], _size),
    "m4_scan_workspace_bytes": ([ctypes.POINTER(ScanDims)], _size),
    "m4_scan_fwd": ([ctypes.POINTER(ScanDims)] + [_p] * 11 + [_p, _size, _p], _c_int),
    "m4_scan_bwd": ([ctypes.POINTER(ScanDims)] + [_p] * 10 + [_size] + [_p] * 11
                    + [_p, _size, _p], _c_int),
    "m4_scan_bwd_noalloc": ([ctypes.POINTER(ScanDims)] + [_p] * 10 + [_size] + [_p] * 11 + [_p],
                            _c_int),
    "m4_scan_step": ([ctypes.POINTER(ScanDims)] + [_p] * 18 + [_p], _c_int),
    "m4_mixer_partial_rows": ([ctypes.POINTER(MixerDims)], _size),
    "m4_mixer_prep_fwd": ([ctypes.POINTER(MixerDims)] + [_p] * 12, _c_int),
    "m4_mixer_post_fwd": ([ctypes.POINTER(MixerDims)] + [_p] * 5, _c_int),
    "m4_mixer_post_bwd": ([ctypes.POINTER(MixerDims)] + [_p] * 9, _c_int),
    "m4_mixer_prep_bwd": ([ctypes.POINTER(MixerDims)] + [_p] * 19, _c_int),
    "m4_rmsnorm_partial_rows": ([_c_int], _size),
    "m4_rmsnorm_fwd": ([_c_int, _c_int, ctypes.c_float] + [_p] * 5, _c_int),
    "m4_rmsnorm_bwd": ([_c_int, _c_int] + [_p] * 8, _c_int),
    "m4_memmix_partial_floats": ([ctypes.POINTER(MemMixDims)], _size),
    "m4_memmix_prep_fwd": ([ctypes.POINTER(MemMixDims), _p, _p, _p, ctypes.c_float] + [_p] * 10, _c_int),
    "m4_memmix_prep_bwd": ([ctypes.POINTER(MemMixDims), _p, _p, _p, ctypes.c_float] + [_p] * 18, _c_int),
    "m4_memmix_order_scratch_floats": ([ctypes.POINTER(MemMixDims)], _size),
    "m4_memmix_order_fwd": ([ctypes.POINTER(MemMixDims)] + [_p] * 5, _c_int),
    "m4_memmix_order_bwd": ([ctypes.POINTER(MemMixDims)] + [_p] * 8, _c_int),
    "m4_memmix_post_fwd": ([ctypes.POINTER(MemMixDims), ctypes.c_float] + [_p] * 12, _c_int),
    "m4_memmix_post_bwd": ([ctypes.POINTER(MemMixDims)] + [_p] * 22, _c_int),
    "m4_add_rmsnorm_fwd": ([_c_int, _c_int, ctypes.c_float] + [_p] * 6, _c_int),
    "m4_memmix_prep_step": ([ctypes.POINTER(MemMixDims), _p, _p, _p, ctypes.c_float] + [_p] * 10, _c_int),
    "m4_memmix_post_step": ([ctypes.POINTER(MemMixDims), ctypes.c_float] + [_p] * 13, _c_int),
    "m4_cross_entropy_fwd": ([_c_int, _c_int, _c_int] + [_p] * 5, _c_int),
    "m4_cross_entropy_bwd": ([_c_int, _c_int, _c_int] + [_p] * 5, _c_int),
    "m4_device_status": ([], _c_int),
    "m4_status_string": ([_c_int], ctypes.c_char_p),
    "m4_version": ([], ctypes.c_char_p),
}

_lib = None


def load():
    """Load (once) and return the ctypes library handle; raise if absent."""
    global _lib
    if _lib is None:
        if not LIBRARY_PATH.exists():
            raise RuntimeError(
                f"mamba4_b200 CUDA library not found at {LIBRARY_PATH}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` or "
                "`python -m mamba4_b200.build`"
            )
        lib = ctypes.CDLL(str(LIBRARY_PATH))
        for name, (argtypes, restype) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        message = load().m4_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {message} (status {status})")


def ptr(tensor) -> int | None:
    """Device pointer of a tensor (None -> NULL)."""
    return None if tensor is None else tensor.data_ptr()
