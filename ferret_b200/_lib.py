"""ctypes binding of the in-tree C-ABI library ``libferret_moe.so``.

The binding follows the reference's shim convention
(tests/compare_decode_linear.py:103-129 in xinhaoc/ferret): the library is
opened with ``ctypes.CDLL`` and called with raw device pointers, ints and the
current stream handle.  There is no fallback: if the library is missing the
import fails with instructions to build it.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libferret_moe.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "ferret_moe.h")

FERRET_SILU_MUL = 0x1
FERRET_TILE_SHIFT = 8
FERRET_UE8M0_SCALES = 0x2
FERRET_PREFILL_PAIRS = 0x4

_p = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/ferret_moe.h
SIGNATURES = {
    "ferret_version": (_i, []),
    "ferret_strerror": (ctypes.c_char_p, [_i]),
    "ferret_set_wait_timeout_ns": (_i, [ctypes.c_ulonglong]),
    "ferret_last_device_status": (_i, [_p, ctypes.POINTER(ctypes.c_int32)]),
    "ferret_selftest_wait_timeout": (_i, [ctypes.c_ulonglong, _p]),
    "ferret_moe_permute": (_i, [_p, _i, _i, _i, _p, _p, _p, _p, _sz, _p]),
    "ferret_moe_permute_workspace_size": (_sz, [_i, _i, _i]),
    "ferret_moe_align_block_size_sizes": (_i, [_i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "ferret_moe_align_block_size_workspace_size": (_sz, [_i, _i, _i]),
    "ferret_moe_align_block_size": (_i, [_p, _i, _i, _i, _i, _p, _p, _p, _p, _sz, _p]),
    "ferret_quant_act_fp8_1x128": (_i, [_p, _i, _p, _i, _i, _i, _p, _p, _p]),
    "ferret_quant_act_fp8_1x128_ue8m0": (_i, [_p, _i, _p, _i, _i, _i, _p, _p, _p]),
    "ferret_quant_act_fp8_1x128_scatter": (_i, [_p, _i, _i, _p, _p, _i, _i, _p, _p, _p, _i, _p]),
    "ferret_fp8_gather_rows": (_i, [_p, _p, _i, _p, _i, _i, _i, _p, _p, _p]),
    "ferret_fp8_grouped_gemm_nt_contiguous": (
        _i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p, _sz, _p]),
    "ferret_fp8_grouped_gemm_workspace_size": (_sz, [_i, _i]),
    "ferret_fp8_grouped_gemm_scatter": (
        _i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p]),
    "ferret_int4_blob_bytes": (_sz, [_i, _i, _i]),
    "ferret_int4_repack_w13": (_i, [_p, _p, _p, _i, _i, _i, _p]),
    "ferret_int4_moe_w13_workspace_size": (_sz, [_i, _i, _i]),
    "ferret_int4_moe_w13": (_i, [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _sz, _p]),
    "ferret_fp8_grouped_gemm_nt_contiguous_noalloc": (
        _i, [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p]),
    "ferret_moe_combine": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p]),
    "ferret_ep_handle_bytes": (_sz, []),
    "ferret_ep_init": (_i, [_i, _i, _i, _i, _i, _i, _i, _i, _p, _p, ctypes.POINTER(_p)]),
    "ferret_ep_connect": (_i, [_p, _p]),
    "ferret_ep_w13_forward": (_i, [_p, _p, _p, _i, _p, _p, _p, _p]),
    "ferret_ep_output_buffer": (_p, [_p]),
    "ferret_ep_set_events": (_i, [_p, _p, _i]),
    "ferret_ep_destroy": (_i, [_p]),
}


class FerretError(RuntimeError):
    """A ferret C-ABI call returned a non-zero code."""

    def __init__(self, what: str, code: int):
        self.code = code
        super().__init__(f"{what} failed: {strerror(code)} (code {code})")


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"ferret_b200 CUDA library not found at {LIB_PATH}; build it with "
                "`python -m ferret_b200.build` (nvcc, sm_100a)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def strerror(code: int) -> str:
    try:
        return lib().ferret_strerror(code).decode()
    except Exception:  # pragma: no cover - only when the library is absent
        return "unknown"


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise FerretError(what, rc)
