"""stew_b200: the NF4 hot path of evilandangry/stew (double-quantized NF4 unpack, the
4-bit Linear forward and input-gradient backward, the rank-16 LoRA q/v adapter) on
hand-written sm_100a kernels behind a C ABI (include/stew_nf4.h).

`apply()` is the counterpart of the reference's `solution.apply()` for this path
(solution/__init__.py:19-51 -> _extra_patches.py:7-27 -> nf4.patch_bnb_dequant): it patches
bitsandbytes (and peft) when they are importable and reports what it did.
"""
from __future__ import annotations

from .nf4 import (MatMul4Bit, _code, _supported, dequantize_nf4, matmul_4bit,  # noqa: F401
                  patch_bnb_dequant)
from .quant_state import QuantState, quantize_4bit  # noqa: F401
from .lora import NF4Linear, NF4LoraFunction, NF4LoraLinear, nf4_lora_linear  # noqa: F401

__all__ = ["apply", "dequantize_nf4", "matmul_4bit", "MatMul4Bit", "QuantState", "quantize_4bit",
           "NF4Linear", "NF4LoraLinear", "NF4LoraFunction", "nf4_lora_linear", "patch_bnb_dequant"]


def apply(verbose: bool = True) -> dict:
    """Install the patches that apply in this process.  Returns {patch name: status}.
    A missing dependency is reported as skipped; a failing patch raises."""
    from . import _lib
    _lib.lib()  # the CUDA library must be present: fail loudly, never fall back
    status = {}
    for name, mod, fn in (("patch_bnb_dequant", "bitsandbytes", patch_bnb_dequant),
                          ("patch_peft_lora", "peft", None)):
        try:
            __import__(mod)
        except ImportError:
            status[name] = f"skipped ({mod} not installed)"
            continue
        if fn is None:
            from .lora import patch_peft_lora
            fn = patch_peft_lora
        fn()
        status[name] = "ok"
    if verbose:
        for k, v in status.items():
            print(f"[stew_b200] {k}: {v}")
    return status
