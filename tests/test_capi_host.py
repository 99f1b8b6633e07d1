"""CPU: the C-ABI library loads and exports every symbol include/*.h declares;
argument validation happens on the host before any launch; the bitsandbytes patch logic
(idempotence, alias rebinding, delegation of unsupported inputs) against a stand-in
bitsandbytes module."""
import ctypes
import os
import re
import sys
import types

import pytest
import torch

from tests.conftest import ROOT


def _declared_functions():
    names = set()
    inc = os.path.join(ROOT, "include")
    for h in sorted(os.listdir(inc)):
        if not h.endswith(".h"):
            continue
        txt = re.sub(r"/\*.*?\*/", "", open(os.path.join(inc, h)).read(), flags=re.S)
        names |= set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(nf4b_\w+)\s*\(", txt, flags=re.M))
    return sorted(names)


def test_library_builds_and_exports_all_declared_symbols():
    from stew_b200 import _lib, build
    build.build()
    L = _lib.lib()
    declared = _declared_functions()
    assert len(declared) >= 10
    for name in declared:
        assert hasattr(L, name), f"{name} missing from libstew_nf4.so"
    assert set(declared) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"
    assert L.nf4b_version().decode().startswith("stew_nf4")


def test_status_strings():
    from stew_b200 import _lib
    L = _lib.lib()
    for code in range(6):
        assert L.nf4b_status_string(code)
    assert b"unsupported" in L.nf4b_status_string(_lib.NF4B_ERR_UNSUPPORTED)


def test_host_validation_rejects_before_launch():
    """These return before touching the device, so they run without a GPU."""
    from stew_b200 import _lib
    L = _lib.lib()
    qs = _lib.QStateC()
    qs.code = 16
    qs.absmax32 = 16
    qs.blocksize = 48  # not a power of two
    st = L.nf4b_dequant(ctypes.c_void_p(16), ctypes.byref(qs), ctypes.c_void_p(16), 0, 96, None)
    assert st == _lib.NF4B_ERR_UNSUPPORTED
    qs.blocksize = 64
    assert L.nf4b_dequant(None, ctypes.byref(qs), ctypes.c_void_p(16), 0, 64, None) == _lib.NF4B_ERR_INVALID_ARG
    assert L.nf4b_dequant(ctypes.c_void_p(16), ctypes.byref(qs), ctypes.c_void_p(16), 7, 64, None) == \
        _lib.NF4B_ERR_UNSUPPORTED
    # numel not a multiple of the blocksize (nf4.py:69)
    assert L.nf4b_dequant(ctypes.c_void_p(16), ctypes.byref(qs), ctypes.c_void_p(16), 0, 96, None) == \
        _lib.NF4B_ERR_UNSUPPORTED
    qs.nested = 1
    qs.blocksize2 = 256
    assert L.nf4b_dequant(ctypes.c_void_p(16), ctypes.byref(qs), ctypes.c_void_p(16), 0, 64, None) == \
        _lib.NF4B_ERR_INVALID_ARG  # nested without absmax8/code2/absmax2/offset
    # nested outside {0, 1, 2}; the contracted-scale form (2) has no fused-GEMM counterpart
    qs.nested = 3
    assert L.nf4b_dequant(ctypes.c_void_p(16), ctypes.byref(qs), ctypes.c_void_p(16), 0, 64, None) == \
        _lib.NF4B_ERR_INVALID_ARG
    qs.nested = 2
    qs.absmax8 = qs.code2 = qs.absmax2 = qs.offset = 16
    assert L.nf4b_linear_fwd(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.byref(qs), None, None,
                             ctypes.c_void_p(16), 4, 64, 64, None) == _lib.NF4B_ERR_UNSUPPORTED
    qs.absmax8 = qs.code2 = qs.absmax2 = qs.offset = None
    # GEMM: K or N not a multiple of 64 -> unsupported, nothing launched
    qs.nested = 0
    assert L.nf4b_linear_fwd(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.byref(qs), None, None,
                             ctypes.c_void_p(16), 4, 96, 64, None) == _lib.NF4B_ERR_UNSUPPORTED
    # plain (not nested) state without its fp32 absmax
    qs.absmax32 = None
    assert L.nf4b_linear_fwd(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.byref(qs), None, None,
                             ctypes.c_void_p(16), 4, 64, 64, None) == _lib.NF4B_ERR_INVALID_ARG
    qs.absmax32 = 16
    lc = _lib.LoraC()
    lc.rank = 8
    lc.a = lc.b = lc.xa = 16
    assert L.nf4b_linear_fwd(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.byref(qs), None, ctypes.byref(lc),
                             ctypes.c_void_p(16), 4, 64, 64, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_lora_grads_work_bytes(100, 1536, 256, 16) > 0
    assert L.nf4b_lora_grads_work_bytes(100, 1536, 256, 8) == -1
    assert L.nf4b_dequant_plan_bytes(0) == 0 and L.nf4b_dequant_plan_bytes(3) > 0
    # grouped forward: at most 3 weights, at least 1
    items = (_lib.LinearItemC * 4)()
    assert L.nf4b_linear_fwd_group(16, 8, 64, items, 4, None, 0, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_linear_fwd_group(16, 8, 64, items, 0, None, 0, None) == _lib.NF4B_ERR_INVALID_ARG
    # layer kernels of the step: hidden not a multiple of 256, odd element counts, head_dim
    assert L.nf4b_rmsnorm_fwd(16, None, 16, 1e-6, None, 16, 16, 4, 1000, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_rmsnorm_bwd(16, 16, 16, 16, None, 16, 4, 8192, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_swiglu_fwd(16, 16, 16, 12, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_swiglu_bwd(16, 16, 16, 16, 16, 12, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_rope_qk(16, 16, 16, 16, 16, 16, 1, 1, 1, 100, 0, None) == _lib.NF4B_ERR_UNSUPPORTED
    # head cross-entropy: vocab not a multiple of 8, missing buffers, misaligned logits
    assert L.nf4b_ce_fwd(16, 16, 16, 16, 4, 1001, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_ce_bwd(16, 16, 16, 16, 4, 1001, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_ce_fwd(16, None, 16, 16, 4, 1000, None) == _lib.NF4B_ERR_INVALID_ARG
    assert L.nf4b_ce_bwd(18, 16, 16, 16, 4, 1000, None) == _lib.NF4B_ERR_ALIGNMENT
    assert L.nf4b_ce_fwd(16, 16, 16, 16, 0, 1000, None) == _lib.NF4B_OK
    assert L.nf4b_rmsnorm_fwd(None, None, 16, 1e-6, None, 16, 16, 4, 256, None) == _lib.NF4B_ERR_INVALID_ARG


def test_supported_envelope_mirrors_reference_guard():
    """nf4.py:61-70 conditions; CPU tensors are never supported (the kernels are CUDA-only)."""
    from stew_b200 import QuantState, _supported, quantize_4bit
    w = torch.randn(64, 128, dtype=torch.float16) * 0.02
    q, st = quantize_4bit(w, blocksize=64, compress_statistics=True)
    assert not _supported(q, st)  # CPU
    assert not _supported(q, None)
    bad = QuantState(st.absmax, st.shape, st.code, 64, quant_type="fp4")
    assert not _supported(q, bad)


class _FakeMatMul4Bit:
    @staticmethod
    def forward(ctx, A, B, out=None, bias=None, quant_state=None):
        return ("orig_forward", A, B)

    @staticmethod
    def backward(ctx, grad_output):
        return ("orig_backward",)


def _install_fake_bnb(monkeypatch):
    calls = []

    def dequantize_4bit(A, quant_state=None, absmax=None, out=None, blocksize=64, quant_type="fp4"):
        calls.append((A, quant_state))
        return "orig_dequant"

    def get_4bit_type(name, device=None):
        from stew_b200 import codebooks
        return codebooks.nf4_table(device or "cpu")

    bnb = types.ModuleType("bitsandbytes")
    F = types.ModuleType("bitsandbytes.functional")
    F.dequantize_4bit = dequantize_4bit
    F.get_4bit_type = get_4bit_type
    alias = types.ModuleType("bitsandbytes.nn.modules")
    alias.dequantize_4bit = dequantize_4bit
    autograd = types.ModuleType("bitsandbytes.autograd")
    fns = types.ModuleType("bitsandbytes.autograd._functions")
    fns.MatMul4Bit = type("MatMul4Bit", (), {"forward": _FakeMatMul4Bit.forward,
                                              "backward": _FakeMatMul4Bit.backward})
    bnb.functional = F
    bnb.autograd = autograd
    autograd._functions = fns
    for name, mod in (("bitsandbytes", bnb), ("bitsandbytes.functional", F),
                      ("bitsandbytes.nn.modules", alias), ("bitsandbytes.autograd", autograd),
                      ("bitsandbytes.autograd._functions", fns)):
        monkeypatch.setitem(sys.modules, name, mod)
    return F, alias, fns, calls


def test_patch_bnb_rebinds_aliases_and_is_idempotent(monkeypatch):
    from stew_b200 import nf4
    F, alias, fns, calls = _install_fake_bnb(monkeypatch)
    orig = F.dequantize_4bit
    nf4.patch_bnb_dequant()
    patched = F.dequantize_4bit
    assert patched is not orig and getattr(patched, "_stew_b200", False)
    assert alias.dequantize_4bit is patched  # nf4.py:116-119
    assert getattr(fns.MatMul4Bit.forward, "_stew_b200", False)
    assert getattr(fns.MatMul4Bit.backward, "_stew_b200", False)
    nf4.patch_bnb_dequant()  # second call is a no-op
    assert F.dequantize_4bit is patched
    # unsupported input (CPU tensor) -> the original function, with all arguments
    A = torch.zeros(8, 1, dtype=torch.uint8)
    assert F.dequantize_4bit(A, None) == "orig_dequant" and calls[-1][0] is A
    # unsupported forward -> original forward; foreign backward -> original backward
    ctx = types.SimpleNamespace(needs_input_grad=(True, False, False, False, False))
    assert fns.MatMul4Bit.forward(ctx, torch.zeros(2, 4), A, None, None, None)[0] == "orig_forward"
    assert fns.MatMul4Bit.backward(ctx, torch.zeros(1))[0] == "orig_backward"


def test_code_table_prefers_bitsandbytes_when_present(monkeypatch):
    from stew_b200 import nf4
    _install_fake_bnb(monkeypatch)
    monkeypatch.setattr(nf4, "_CODE", {})
    t = nf4._code("cpu")
    assert t.dtype == torch.float32 and t.shape == (16,)


def test_apply_reports_missing_dependencies():
    import stew_b200
    status = stew_b200.apply(verbose=False)
    if "bitsandbytes" not in sys.modules:
        assert status["patch_bnb_dequant"].startswith("skipped")
