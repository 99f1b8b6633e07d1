"""The patched bitsandbytes entry points on CUDA tensors.

bitsandbytes itself is not installed here, so a stand-in module provides the two functions the
reference patches -- `functional.dequantize_4bit` and `autograd._functions.MatMul4Bit` -- with
bitsandbytes' calling conventions: the original dequantize applies the (1, n) -> transposed rule,
the original MatMul4Bit unpacks (the canonical (n/2, 1) layout) and calls F.linear, and its
backward is dY . W.  Their arithmetic is the oracle's (the reference's unpack restated on the
CPU), so "original" and "patched" are compared exactly as the reference's own tests compare
bitsandbytes with its patch:
  solution/test_nf4_shim.py:15-40     patched dequantize_4bit == original, both layouts
  solution/test_nf4_forward.py:10-51  patched MatMul4Bit forward / x.grad == original
plus the parts of the contract those tests leave implicit: inputs outside the envelope go to
the original function with all their arguments, and an error in the fast path latches
`_BROKEN` and hands that call and later ones to the original (solution/nf4.py:104-112).
Tolerances: the unpack bit-exact; GEMMs max-normalised and elementwise 2e-3 against fp64.
"""
import sys
import types

import pytest
import torch

from oracle import nf4_oracle as O
from tests.helpers import assert_gemm_close, to_oracle_state

pytestmark = pytest.mark.gpu


def _oracle_unpack(A: torch.Tensor, st) -> torch.Tensor:
    """The reference unpack of packed A (any view of the packed bytes) on the CPU."""
    flat = A.reshape(-1).contiguous()
    w = O.dequant_nf4(flat.cpu().numpy(), to_oracle_state(st, flat))
    return torch.from_numpy(w).to(A.device)


def _install_fake_bnb(monkeypatch):
    calls = {"dequant": 0, "forward": 0, "backward": 0}

    def dequantize_4bit(A, quant_state=None, absmax=None, out=None, blocksize=64, quant_type="fp4"):
        calls["dequant"] += 1
        w = _oracle_unpack(A, quant_state)
        return w.t() if A.shape[0] == 1 else w

    def get_4bit_type(name, device=None):
        from stew_b200 import codebooks
        return codebooks.nf4_table(device or "cpu")

    F = types.ModuleType("bitsandbytes.functional")
    F.dequantize_4bit = dequantize_4bit
    F.get_4bit_type = get_4bit_type

    class MatMul4Bit(torch.autograd.Function):
        @staticmethod
        def forward(ctx, A, B, out=None, bias=None, quant_state=None):
            calls["forward"] += 1
            Bv = B.view(-1, 1)
            W = F.dequantize_4bit(Bv, quant_state).to(A.dtype)
            ctx.state = quant_state
            ctx.dtype_A, ctx.dtype_bias = A.dtype, None if bias is None else bias.dtype
            ctx.tensors = (None, Bv)
            return torch.nn.functional.linear(A, W, bias)

        @staticmethod
        def backward(ctx, grad_output):
            calls["backward"] += 1
            _, Bv = ctx.tensors
            ga = torch.matmul(grad_output, F.dequantize_4bit(Bv, ctx.state).to(grad_output.dtype))
            gb = grad_output.reshape(-1, grad_output.shape[-1]).sum(0) if ctx.needs_input_grad[3] else None
            return ga, None, None, gb, None

    fns = types.ModuleType("bitsandbytes.autograd._functions")
    fns.MatMul4Bit = MatMul4Bit
    autograd = types.ModuleType("bitsandbytes.autograd")
    autograd._functions = fns
    bnb = types.ModuleType("bitsandbytes")
    bnb.functional = F
    bnb.autograd = autograd
    bnb.matmul_4bit = lambda A, B, quant_state, out=None, bias=None: fns.MatMul4Bit.apply(
        A, B, out, bias, quant_state)
    for name, mod in (("bitsandbytes", bnb), ("bitsandbytes.functional", F),
                      ("bitsandbytes.autograd", autograd), ("bitsandbytes.autograd._functions", fns)):
        monkeypatch.setitem(sys.modules, name, mod)
    return bnb, F, fns, calls


@pytest.fixture
def fake_bnb(monkeypatch, cuda_lib):
    from stew_b200 import nf4
    monkeypatch.setattr(nf4, "_BROKEN", False)
    monkeypatch.setattr(nf4, "_WARNED", set())
    bnb, F, fns, calls = _install_fake_bnb(monkeypatch)
    orig = (F.dequantize_4bit, fns.MatMul4Bit.forward, fns.MatMul4Bit.backward)
    yield bnb, F, fns, calls, orig
    monkeypatch.setattr(nf4, "_BROKEN", False)


def _weight(shape, nested, seed=0):
    from stew_b200 import quantize_4bit
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(shape, generator=g, device="cuda") * 0.05).to(torch.float16)
    return quantize_4bit(w, blocksize=64, compress_statistics=nested)


@pytest.mark.parametrize("nested", [True, False])
def test_patched_dequantize_matches_original_for_both_layouts(fake_bnb, nested):
    """test_nf4_shim.py:15-40: W [256, 1536] unpacked through the (n/2, 1) view and through
    its (1, n/2) transpose, which comes back transposed (nf4.py:108-109)."""
    from stew_b200 import nf4
    _, F, _, calls, (orig_deq, _, _) = fake_bnb
    q, st = _weight((256, 1536), nested)
    refs = [orig_deq(A, st) for A in (q, q.t())]
    nf4.patch_bnb_dequant()
    n0 = calls["dequant"]
    outs = [F.dequantize_4bit(A, st) for A in (q, q.t())]
    assert calls["dequant"] == n0, "the patched function fell back to the original"
    assert outs[0].shape == (256, 1536) and outs[1].shape == (1536, 256)
    for out, ref in zip(outs, refs):
        assert out.shape == ref.shape and out.dtype == ref.dtype
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), "unpack not bit-exact"


def test_patched_dequantize_hands_other_calls_to_the_original(fake_bnb):
    """absmax= or out= given, another quant type, a CPU tensor: the original, all arguments."""
    from stew_b200 import QuantState, nf4
    _, F, _, calls, _ = fake_bnb
    q, st = _weight((128, 256), True)
    nf4.patch_bnb_dequant()
    n0 = calls["dequant"]
    F.dequantize_4bit(q, st, absmax=st.absmax)
    F.dequantize_4bit(q, st, out=torch.empty(128, 256, dtype=torch.float16, device="cuda"))
    fp4 = QuantState(st.absmax, st.shape, st.code, 64, "fp4", torch.float16, st.offset, st.state2)
    F.dequantize_4bit(q, fp4)
    F.dequantize_4bit(q.cpu(), QuantState(st.absmax.cpu(), st.shape, st.code.cpu(), 64, "nf4",
                                          torch.float16, st.offset.cpu(), st.state2.to("cpu")))
    assert calls["dequant"] == n0 + 4


@pytest.mark.parametrize("nested", [True, False])
@pytest.mark.parametrize("with_bias", [True, False])
def test_patched_matmul4bit_matches_original(fake_bnb, nested, with_bias):
    """test_nf4_forward.py:10-51: x [2, 37, 256] -> [2, 37, 512] through bnb.matmul_4bit(x,
    W.t()), bias on/off, output and x.grad: the original first, then the patched path (fused
    forward and fused dX); both against fp64."""
    from stew_b200 import nf4
    bnb, _, fns, calls, _ = fake_bnb
    out_f, in_f = 512, 256
    q, st = _weight((out_f, in_f), nested, seed=1)
    g = torch.Generator(device="cuda").manual_seed(2)
    bias = (torch.randn(out_f, generator=g, device="cuda").half() if with_bias else None)
    x0 = torch.randn(2, 37, in_f, generator=g, device="cuda").half()
    dy = torch.randn(2, 37, out_f, generator=g, device="cuda").half()
    x_ref = x0.clone().requires_grad_(True)
    ref = bnb.matmul_4bit(x_ref, q.t(), quant_state=st, bias=bias)
    ref.backward(dy)
    nf4.patch_bnb_dequant()
    assert getattr(fns.MatMul4Bit.forward, "_stew_b200", False)
    c0 = dict(calls)
    x = x0.clone().requires_grad_(True)
    out = bnb.matmul_4bit(x, q.t(), quant_state=st, bias=bias)
    out.backward(dy)
    assert calls == c0, "the patched MatMul4Bit used an original function"
    assert out.shape == ref.shape and out.dtype == ref.dtype
    torch.testing.assert_close(out, ref.detach(), rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(x.grad, x_ref.grad, rtol=2e-3, atol=2e-3)
    W = _oracle_unpack(q, st).double()
    assert_gemm_close(out, x0.double() @ W.T + (0 if bias is None else bias.double()), "fwd")
    assert_gemm_close(x.grad, dy.double() @ W, "dX")


def test_matmul4bit_outside_the_envelope_uses_the_original(fake_bnb):
    """nf4.py:144-145: out= given, or a single row -> the original forward and backward."""
    from stew_b200 import nf4
    bnb, _, fns, calls, _ = fake_bnb
    q, st = _weight((128, 256), True, seed=3)
    nf4.patch_bnb_dequant()
    x1 = torch.randn(1, 256, device="cuda").half().requires_grad_(True)
    f0, b0 = calls["forward"], calls["backward"]
    y = bnb.matmul_4bit(x1, q.t(), quant_state=st)
    y.sum().backward()
    assert calls["forward"] == f0 + 1 and calls["backward"] == b0 + 1


def test_bf16_activations_take_the_reference_composition(fake_bnb):
    """bf16 activations are outside the fused envelope: the patched forward runs the unpack
    kernel + F.linear (the reference's own composition, nf4.py:148-152) with a warning, and
    the backward the unpack kernel + matmul; both match fp64 at bf16 precision."""
    from stew_b200 import nf4
    bnb, _, _, calls, _ = fake_bnb
    q, st = _weight((256, 512), True, seed=4)
    nf4.patch_bnb_dequant()
    x = torch.randn(40, 512, device="cuda").bfloat16().requires_grad_(True)
    c0 = dict(calls)
    with pytest.warns(RuntimeWarning, match="bfloat16"):
        y = bnb.matmul_4bit(x, q.t(), quant_state=st)
        y.float().sum().backward()
    assert calls == c0
    W = _oracle_unpack(q, st).double()
    ref = x.detach().double() @ W.T
    assert y.dtype == torch.bfloat16
    assert float((y.double() - ref).abs().max() / ref.abs().max()) <= 1e-2
    assert float((x.grad.double() - W.sum(0)).abs().max() / W.sum(0).abs().max()) <= 1e-2


def test_fast_path_error_latches_to_the_original(fake_bnb, monkeypatch):
    """An error inside the fast path: warn once, set _BROKEN, answer with the original --
    for that call and every later one (solution/nf4.py:104-112)."""
    from stew_b200 import nf4
    bnb, F, _, calls, _ = fake_bnb
    q, st = _weight((128, 256), True, seed=5)
    nf4.patch_bnb_dequant()

    def boom(*a, **k):
        raise RuntimeError("injected kernel failure")

    monkeypatch.setattr(nf4, "dequantize_nf4", boom)
    monkeypatch.setattr(nf4, "linear_forward", boom)
    d0 = calls["dequant"]
    with pytest.warns(RuntimeWarning, match="injected kernel failure"):
        w = F.dequantize_4bit(q, st)
    assert nf4._BROKEN and calls["dequant"] == d0 + 1
    assert torch.equal(w, _oracle_unpack(q, st))
    f0 = calls["forward"]
    x = torch.randn(8, 256, device="cuda").half()
    y = bnb.matmul_4bit(x, q.t(), quant_state=st)
    assert calls["forward"] == f0 + 1 and y.shape == (8, 128)
