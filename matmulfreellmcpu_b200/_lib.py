"""ctypes binding of libmmfree_cuda.so (the C ABI of include/mmfree_cuda.h).

The library is built in-tree by ``matmulfreellmcpu_b200.build`` into ``_lib/``. There is no
fallback: if it is missing or fails to load, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

LIB_PATH = _build.LIB

OK = 0
E_INVALID, E_CUDA, E_IO, E_RANGE, E_STATE, E_INTERNAL, E_TIMEOUT = -1, -2, -3, -4, -5, -6, -7
ACT_FLOAT, ACT_FIXED_Q510 = 0, 1
MAX_IN_DIM = 57344

VP, SZ, F, I, I64, U64 = C.c_void_p, C.c_size_t, C.c_float, C.c_int, C.c_int64, C.c_uint64

#: every exported symbol with (restype, argtypes); the header declares exactly these.
SIGNATURES = {
    "mmfree_cuda_last_error": (C.c_char_p, []),
    "mmfree_cuda_abi_version": (I, []),
    "mmfree_cuda_packed_bytes": (SZ, [SZ, SZ]),
    "mmfree_cuda_repack_ternary": (I, [VP, VP, SZ, SZ, VP]),
    "mmfree_cuda_pack_ternary_host": (I, [VP, VP, SZ, SZ]),
    "mmfree_cuda_bitlinear": (I, [VP, VP, VP, VP, F, SZ, SZ, SZ, F, VP, I, I, VP, VP]),
    "mmfree_cuda_bitlinear_noalloc": (I, [VP, VP, VP, VP, F, SZ, SZ, SZ, F, VP, I, I, VP, VP]),
    "mmfree_cuda_kernel_status": (I, [VP]),
    "mmfree_cuda_set_wait_limit": (None, [I64]),
    "mmfree_cuda_bitlinear_cluster": (I, [VP, VP, VP, VP, VP, I, SZ, SZ, SZ, F, I, VP, VP]),
    "mmfree_cuda_ternary_matmul": (I, [VP, VP, VP, SZ, SZ, SZ, VP]),
    "mmfree_cuda_seam_open": (I, [I, C.POINTER(VP)]),
    "mmfree_cuda_seam_matmul": (I, [VP, VP, SZ, SZ, VP, VP, SZ]),
    "mmfree_cuda_seam_close": (None, [VP]),
    "mmfree_cuda_rmsnorm": (I, [VP, VP, VP, SZ, SZ, F, VP]),
    "mmfree_cuda_swiglu": (I, [VP, VP, VP, SZ, VP]),
    "mmfree_cuda_hgrn_scan": (I, [VP, VP, VP, SZ, SZ, VP, VP]),
    "mmfree_cuda_rmsnorm_swishgate": (I, [VP, VP, VP, VP, SZ, SZ, F, VP]),
    "mmfree_cuda_model_open": (I, [C.c_char_p, I, I, I, C.POINTER(VP)]),
    "mmfree_cuda_model_close": (None, [VP]),
    "mmfree_cuda_nccl_unique_id": (I, [VP]),
    "mmfree_cuda_model_open_tp": (I, [C.c_char_p, I, I, I, I, I, VP, C.POINTER(VP)]),
    "mmfree_cuda_model_config": (I, [VP, VP]),
    "mmfree_cuda_blob_config": (I, [C.c_char_p, VP]),
    "mmfree_cuda_model_weight_bytes": (SZ, [VP]),
    "mmfree_cuda_generate": (I, [VP, VP, SZ, SZ, I64, F, I, U64, VP, SZ, C.POINTER(SZ)]),
    "mmfree_cuda_generate_stream": (I, [VP, VP, SZ, SZ, I64, F, I, U64, VP, VP, VP, SZ,
                                        C.POINTER(SZ)]),
    "mmfree_cuda_forward": (I, [VP, VP, SZ, VP]),
    "mmfree_cuda_forward_last": (I, [VP, VP, SZ, VP]),
    "mmfree_cuda_forward_trace": (I, [VP, VP, SZ, VP, VP]),
    "mmfree_cuda_generate_serve": (I, [VP, SZ, VP, VP, SZ, I64, F, I, U64, VP, SZ, VP]),
    "mmfree_cuda_serve_begin": (I, [VP, SZ, VP, VP, VP]),
    "mmfree_cuda_serve_step": (I, [VP, VP, VP]),
    "mmfree_cuda_serve_run": (I, [VP, SZ, VP]),
    "mmfree_cuda_serve_end": (I, [VP]),
    "mmfree_cuda_model_stream": (VP, [VP]),
    "mmfree_cuda_serve_profile": (I, [VP, SZ, VP, I, C.POINTER(I)]),
}


class KernelStats(C.Structure):
    _fields_ = [("name", C.c_char_p), ("ms", C.c_double), ("launches", C.c_int64),
                ("bytes", C.c_double), ("ops", C.c_double)]


class MmfreeError(RuntimeError):
    """A non-zero status from the C ABI; ``code`` is the MMFREE_E_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


_LIB = None


def lib() -> C.CDLL:
    """Load libmmfree_cuda.so (once). Raises if the library has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m matmulfreellmcpu_b200.build`")
        h = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = h
    return _LIB


def check(rc: int) -> None:
    if rc != OK:
        raise MmfreeError(rc, lib().mmfree_cuda_last_error().decode(errors="replace"))
