"""patch_peft_lora on CUDA tensors: peft's lora.Linear.forward routed through the fused NF4 +
LoRA op for the adapters it fits, and peft's own forward for everything else.

peft is not installed here, so a stand-in `peft.tuners.lora.layer.Linear` provides the
attributes the patch reads (get_base_layer, active_adapters, merged, disable_adapters, r,
lora_A / lora_B / lora_dropout module dicts, scaling) and peft's composition
y = base(x) + lora_B(lora_A(dropout(x))) * scaling as its original forward; the base layer is a
4-bit Linear whose weight is the packed (n/2, 1) uint8 tensor carrying its quant_state, as a
bitsandbytes Linear4bit's is.  The fused route must match fp64 autograd (output, dX, dA, dB);
dropout > 0, a rank other than 16, a merged or disabled adapter, bf16 input and extra forward
arguments must reach peft's original forward.
Tolerances: y and dX max-normalised and elementwise 2e-3; dA, dB max-normalised 1e-3.
"""
import math
import sys
import types

import pytest
import torch

from tests.helpers import assert_gemm_close, max_rel_err
from tests.test_gpu_bnb_patch import _oracle_unpack

pytestmark = pytest.mark.gpu


class Linear4bit(torch.nn.Module):
    """The base layer: weight = packed uint8 [n/2, 1] with .quant_state (bitsandbytes' layout)."""

    def __init__(self, packed, st, bias=None):
        super().__init__()
        self.weight = torch.nn.Parameter(packed, requires_grad=False)
        self.weight.quant_state = st
        self.bias = bias

    def forward(self, x):
        from stew_b200 import matmul_4bit
        return matmul_4bit(x, self.weight.t(), self.weight.quant_state, bias=self.bias)


class LoraLinear(torch.nn.Module):
    """peft's lora.Linear: the attributes patch_peft_lora reads and peft's forward."""
    calls = 0

    def __init__(self, base, r=16, alpha=32, dropout=0.0):
        super().__init__()
        self.base_layer = base
        out_f, in_f = (int(s) for s in base.weight.quant_state.shape)
        self.r = {"default": r}
        self.scaling = {"default": alpha / r}
        self.lora_A = torch.nn.ModuleDict({"default": torch.nn.Linear(in_f, r, bias=False)})
        self.lora_B = torch.nn.ModuleDict({"default": torch.nn.Linear(r, out_f, bias=False)})
        self.lora_dropout = torch.nn.ModuleDict(
            {"default": torch.nn.Dropout(dropout) if dropout > 0 else torch.nn.Identity()})
        torch.nn.init.kaiming_uniform_(self.lora_A["default"].weight, a=math.sqrt(5))
        torch.nn.init.normal_(self.lora_B["default"].weight, std=0.01)
        self.active_adapters = ["default"]
        self.merged = False
        self.disable_adapters = False

    def get_base_layer(self):
        return self.base_layer

    def forward(self, x, *args, **kwargs):
        LoraLinear.calls += 1
        y = self.base_layer(x)
        if self.disable_adapters or self.merged:
            return y
        for name in self.active_adapters:
            a, b = self.lora_A[name], self.lora_B[name]
            h = self.lora_dropout[name](x.to(a.weight.dtype))
            y = y + (b(a(h)) * self.scaling[name]).to(y.dtype)
        return y


@pytest.fixture
def peft_patched(monkeypatch, cuda_lib):
    from stew_b200 import lora, nf4
    monkeypatch.setattr(nf4, "_WARNED", set())
    cls = type("Linear", (LoraLinear,), {"forward": LoraLinear.forward})
    layer_mod = types.ModuleType("peft.tuners.lora.layer")
    layer_mod.Linear = cls
    names = ("peft", "peft.tuners", "peft.tuners.lora", "peft.tuners.lora.layer")
    mods = [types.ModuleType(n) for n in names[:-1]] + [layer_mod]
    for parent, child, n in zip(mods, mods[1:], names[1:]):
        setattr(parent, n.rsplit(".", 1)[1], child)
    for n, m in zip(names, mods):
        monkeypatch.setitem(sys.modules, n, m)
    lora.patch_peft_lora()
    assert getattr(cls.forward, "_stew_b200", False)
    lora.patch_peft_lora()  # idempotent
    return cls


def _layer(cls, out_f=1536, in_f=1536, seed=0, **kw):
    from stew_b200 import quantize_4bit
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(out_f, in_f, generator=g, device="cuda") * 0.02).half()
    q, st = quantize_4bit(w, blocksize=64, compress_statistics=True)
    bias = (torch.randn(out_f, generator=g, device="cuda") * 0.02).half()
    torch.manual_seed(seed)
    return cls(Linear4bit(q, st, bias), **kw).cuda()


@pytest.mark.parametrize("shape", [(1536, 1536), (256, 1536)])
def test_fused_route_matches_fp64(peft_patched, shape):
    """q and v of Qwen2.5-1.5B (r 16, alpha 32, dropout 0): y, dX, dA, dB against fp64."""
    m = _layer(peft_patched, *shape, seed=shape[0])
    x = torch.randn(3, 391, shape[1], device="cuda").half().requires_grad_(True)
    dy = (torch.randn(3, 391, shape[0], device="cuda") * 0.01).half()
    c0 = LoraLinear.calls
    y = m(x)
    y.backward(dy)
    assert LoraLinear.calls == c0, "peft's own forward ran instead of the fused op"
    base = m.base_layer
    W = _oracle_unpack(base.weight, base.weight.quant_state).double()
    A = m.lora_A["default"].weight.detach().double().requires_grad_(True)
    B = m.lora_B["default"].weight.detach().double().requires_grad_(True)
    xd = x.detach().double().requires_grad_(True)
    ref = xd @ W.T + base.bias.double() + (xd @ A.T) @ B.T * 2.0
    ref.backward(dy.double())
    assert y.shape == ref.shape and y.dtype == torch.float16
    assert_gemm_close(y, ref.detach(), "y")
    assert_gemm_close(x.grad, xd.grad, "dX")
    assert max_rel_err(m.lora_A["default"].weight.grad, A.grad) <= 1e-3
    assert max_rel_err(m.lora_B["default"].weight.grad, B.grad) <= 1e-3


@pytest.mark.parametrize("case", ["dropout", "rank8", "merged", "disabled", "bf16", "kwargs"])
def test_other_adapters_keep_peft_forward(peft_patched, case):
    kw = {"dropout": 0.05} if case == "dropout" else ({"r": 8, "alpha": 16} if case == "rank8" else {})
    m = _layer(peft_patched, 256, 512, seed=7, **kw)
    if case == "merged":
        m.merged = True
    if case == "disabled":
        m.disable_adapters = True
    m.eval()
    x = torch.randn(64, 512, device="cuda").half()
    c0 = LoraLinear.calls
    if case == "bf16":
        with pytest.warns(RuntimeWarning):
            m(x.bfloat16())
    elif case == "kwargs":
        m(x, adapter_names=["default"])
    else:
        m(x)
    assert LoraLinear.calls == c0 + 1
