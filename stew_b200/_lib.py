"""ctypes binding of libstew_nf4.so (the C ABI declared in include/stew_nf4.h and
include/stew_step.h).

The library is built in-tree by stew_b200.build (nvcc, sm_100a).  Loading fails
loudly when it is missing: there is no CPU or Triton fallback behind this API.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

NF4B_OK = 0
NF4B_ERR_INVALID_ARG = 1
NF4B_ERR_UNSUPPORTED = 2
NF4B_ERR_ALIGNMENT = 3
NF4B_ERR_CUDA = 4
NF4B_ERR_DEVICE = 5
NF4B_F16 = 0
NF4B_F32 = 1

c_void_p = ctypes.c_void_p
c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_float = ctypes.c_float


class QStateC(ctypes.Structure):
    """nf4b_qstate."""
    _fields_ = [("absmax8", c_void_p), ("absmax32", c_void_p), ("code2", c_void_p),
                ("absmax2", c_void_p), ("offset", c_void_p), ("code", c_void_p),
                ("blocksize", c_int32), ("blocksize2", c_int32), ("nested", c_int32),
                ("reserved", c_int32)]


class DequantJobC(ctypes.Structure):
    """nf4b_dequant_job."""
    _fields_ = [("packed", c_void_p), ("out", c_void_p), ("qs", QStateC), ("numel", c_int64),
                ("out_dtype", c_int32), ("reserved", c_int32)]


class LoraC(ctypes.Structure):
    """nf4b_lora."""
    _fields_ = [("a", c_void_p), ("b", c_void_p), ("scale", c_float), ("rank", c_int32),
                ("xa", c_void_p)]


class LinearBwdItemC(ctypes.Structure):
    """nf4b_linear_bwd_item."""
    _fields_ = [("dy", c_void_p), ("packed", c_void_p), ("qs", ctypes.POINTER(QStateC)),
                ("lora", ctypes.POINTER(LoraC)), ("dyb", c_void_p), ("out_features", c_int64)]


class LinearItemC(ctypes.Structure):
    """nf4b_linear_item."""
    _fields_ = [("packed", c_void_p), ("qs", ctypes.POINTER(QStateC)), ("bias", c_void_p),
                ("lora", ctypes.POINTER(LoraC)), ("y", c_void_p), ("out_features", c_int64)]


class LoraGradsItemC(ctypes.Structure):
    """nf4b_lora_grads_item."""
    _fields_ = [("x", c_void_p), ("dy", c_void_p), ("xa", c_void_p), ("dyb", c_void_p),
                ("scale", c_float), ("da", c_void_p), ("db", c_void_p), ("in_features", c_int64),
                ("out_features", c_int64)]


# name -> (restype, argtypes); every symbol include/*.h declares
SIGNATURES = {
    "nf4b_dequant": (c_int32, [c_void_p, ctypes.POINTER(QStateC), c_void_p, c_int32, c_int64, c_void_p]),
    "nf4b_dequant_plan_bytes": (c_int64, [c_int32]),
    "nf4b_dequant_plan": (c_int32, [ctypes.POINTER(DequantJobC), c_int32, c_void_p,
                                    ctypes.POINTER(c_int64), c_void_p]),
    "nf4b_dequant_batched": (c_int32, [c_void_p, c_int32, c_int64, c_void_p]),
    "nf4b_linear_fwd": (c_int32, [c_void_p, c_void_p, ctypes.POINTER(QStateC), c_void_p,
                                  ctypes.POINTER(LoraC), c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    "nf4b_linear_bwd_dx": (c_int32, [c_void_p, c_void_p, ctypes.POINTER(QStateC),
                                     ctypes.POINTER(LoraC), c_void_p, c_void_p, c_int64, c_int64,
                                     c_int64, c_void_p]),
    "nf4b_linear_work_bytes": (c_int64, [c_int64, c_int64, c_int64, c_int32]),
    "nf4b_linear_fwd_ws": (c_int32, [c_void_p, c_void_p, ctypes.POINTER(QStateC), c_void_p,
                                     ctypes.POINTER(LoraC), c_void_p, c_int64, c_int64, c_int64,
                                     c_void_p, c_int64, c_void_p]),
    "nf4b_linear_bwd_dx_ws": (c_int32, [c_void_p, c_void_p, ctypes.POINTER(QStateC),
                                        ctypes.POINTER(LoraC), c_void_p, c_void_p, c_int64, c_int64,
                                        c_int64, c_void_p, c_int64, c_void_p]),
    "nf4b_linear_group_work_bytes": (c_int64, [c_int64, c_int64, ctypes.POINTER(c_int64), c_int32]),
    "nf4b_linear_fwd_group": (c_int32, [c_void_p, c_int64, c_int64, ctypes.POINTER(LinearItemC), c_int32,
                                        c_void_p, c_int64, c_void_p]),
    "nf4b_linear_bwd_group_work_bytes": (c_int64, [c_int64, c_int64, ctypes.POINTER(c_int64), c_int32]),
    "nf4b_linear_bwd_dx_group": (c_int32, [ctypes.POINTER(LinearBwdItemC), c_int32, c_void_p, c_int64,
                                           c_int64, c_void_p, c_int64, c_void_p]),
    "nf4b_linear_swiglu_work_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "nf4b_linear_fwd_swiglu": (c_int32, [c_void_p, c_int64, c_int64, c_void_p, ctypes.POINTER(QStateC), c_void_p,
                                         ctypes.POINTER(QStateC), c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                                         c_int64, c_void_p]),
    "nf4b_linear_bwd_dx_swiglu": (c_int32, [c_void_p, c_void_p, ctypes.POINTER(QStateC), c_void_p, c_void_p,
                                            c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64,
                                            c_void_p]),
    "nf4b_lora_grads_work_bytes": (c_int64, [c_int64, c_int64, c_int64, c_int32]),
    "nf4b_lora_grads_group_work_bytes": (c_int64, [ctypes.POINTER(LoraGradsItemC), c_int32, c_int64]),
    "nf4b_lora_grads_group": (c_int32, [ctypes.POINTER(LoraGradsItemC), c_int32, c_void_p, c_int64,
                                        c_int64, c_void_p]),
    # layer kernels of the QLoRA step (include/stew_step.h)
    "nf4b_rmsnorm_fwd": (c_int32, [c_void_p, c_void_p, c_void_p, ctypes.c_float, c_void_p, c_void_p,
                                   c_void_p, c_int64, c_int64, c_void_p]),
    "nf4b_rmsnorm_bwd": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_int64, c_int64, c_void_p]),
    "nf4b_rope_qk": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                               c_int32, c_int32, c_int32, c_int32, c_void_p]),
    "nf4b_swiglu_fwd": (c_int32, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "nf4b_swiglu_bwd": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "nf4b_ce_fwd": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "nf4b_ce_bwd": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "nf4b_lora_grads": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p,
                                  c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int32, c_void_p]),
    "nf4b_lora_grads_noalloc": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p,
                                          c_void_p, c_int64, c_int64, c_int64, c_int32, c_void_p]),
    "nf4b_quantize_work_bytes": (c_int64, [c_int64, c_int32]),
    "nf4b_quantize": (c_int32, [c_void_p, c_int32, c_int64, c_int32, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "nf4b_gemm_error_flag": (c_int32, [ctypes.POINTER(c_int32), c_int32]),
    "nf4b_dequant_error_flag": (c_int32, [ctypes.POINTER(c_int32), c_int32]),
    "nf4b_test_drop_split_ticket": (c_int32, [c_int32]),
    "nf4b_gemm_geometry": (c_int32, [ctypes.POINTER(c_int32), ctypes.POINTER(c_int32)]),
    "nf4b_status_string": (ctypes.c_char_p, [c_int32]),
    "nf4b_last_error": (ctypes.c_char_p, []),
    "nf4b_version": (ctypes.c_char_p, []),
}

_LIB = None
_LOCK = threading.Lock()


class NF4Error(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, what: str):
        self.status = status
        msg = lib().nf4b_status_string(status).decode() if _LIB is not None else str(status)
        if status == NF4B_ERR_CUDA and _LIB is not None:
            msg += "; " + _LIB.nf4b_last_error().decode()
        super().__init__(f"{what}: status {status} ({msg})")


class NF4Unsupported(NF4Error):
    """The input is outside the kernel envelope; nothing was launched."""


def lib_path() -> str:
    return _build.LIB


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            path = lib_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"stew_b200 CUDA library not built ({path} missing): run "
                    "`python -m stew_b200.build` (or __graft_entry__.build())")
            handle = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _LIB = handle
    return _LIB


def check(status: int, what: str) -> None:
    if status == NF4B_OK:
        return
    if status == NF4B_ERR_UNSUPPORTED:
        raise NF4Unsupported(status, what)
    raise NF4Error(status, what)


def gemm_error_flag(reset: bool = True) -> int:
    v = c_int32(0)
    check(lib().nf4b_gemm_error_flag(ctypes.byref(v), 1 if reset else 0), "nf4b_gemm_error_flag")
    return int(v.value)


def dequant_error_flag(reset: bool = True) -> int:
    v = c_int32(0)
    check(lib().nf4b_dequant_error_flag(ctypes.byref(v), 1 if reset else 0), "nf4b_dequant_error_flag")
    return int(v.value)


def gemm_geometry() -> tuple:
    """(SMs, resident 2-CTA clusters) the fused GEMMs plan with on the current device."""
    a, b = c_int32(0), c_int32(0)
    check(lib().nf4b_gemm_geometry(ctypes.byref(a), ctypes.byref(b)), "nf4b_gemm_geometry")
    return a.value, b.value
