"""GPU parity of the fused NF4 dequant-GEMMs (C ABI nf4b_linear_fwd / nf4b_linear_bwd_dx).

Reference: the fp64 product of the oracle-dequantised weight (bit-identical to the
reference unpack) -- i.e. what nf4.py:148-152 (unpack, then F.linear) and bitsandbytes'
MatMul4Bit.backward compute, before their fp16 output rounding.
Tolerances (tests/helpers.py, used everywhere below): max |y - ref| / max |ref| <= 2e-3, and
elementwise |y - ref| / |ref| <= 2e-3 over the entries with |ref| >= 0.05 max |ref|.
"""
import numpy as np
import pytest
import torch

from oracle import nf4_oracle as O
from tests.helpers import GEMM_MAX_REL_ERR, assert_gemm_close, max_rel_err, to_oracle_state

pytestmark = pytest.mark.gpu

QWEN = {"q": (1536, 1536), "k": (256, 1536), "v": (256, 1536), "o": (1536, 1536),
        "gate": (8960, 1536), "up": (8960, 1536), "down": (1536, 8960)}


def _weight(shape, seed, blocksize=64, nested=True):
    from stew_b200 import quantize_4bit
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(shape, generator=g, device="cuda") * 0.02).to(torch.float16)
    return quantize_4bit(w, blocksize=blocksize, compress_statistics=nested)


def _ref_weight(q, st) -> torch.Tensor:
    """Oracle-dequantised weight as fp64 on the GPU."""
    w = O.dequant_nf4(q.cpu().numpy(), to_oracle_state(st, q))
    return torch.from_numpy(w.astype(np.float64)).cuda()


def _x(n, k, seed, std=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(n, k, generator=g, device="cuda") * std).to(torch.float16)


def _check_flag():
    from stew_b200 import _lib
    assert _lib.gemm_error_flag(reset=True) == 0, "a pipeline wait timed out inside the GEMM"


@pytest.mark.parametrize("nested", [True, False])
@pytest.mark.parametrize("with_bias", [True, False])
def test_matmul4bit_forward_backward_contract(cuda_lib, nested, with_bias):
    """solution/test_nf4_forward.py:10-51: x [2, 37, 256] -> [2, 37, 512], bias on/off,
    output and x.grad (rtol = atol = 2e-3 there; here against fp64)."""
    from stew_b200 import matmul_4bit
    torch.manual_seed(0)
    out_f, in_f = 512, 256
    q, st = _weight((out_f, in_f), 11, nested=nested)
    bias = torch.randn(out_f, device="cuda", dtype=torch.float16) if with_bias else None
    x = torch.randn(2, 37, in_f, device="cuda", dtype=torch.float16).requires_grad_(True)
    g = torch.randn(2, 37, out_f, device="cuda", dtype=torch.float16)
    y = matmul_4bit(x, q.t(), st, bias=bias)
    y.backward(g)
    W = _ref_weight(q, st)
    ref = x.detach().double() @ W.T + (0 if bias is None else bias.double())
    ref_dx = g.double() @ W
    assert y.shape == ref.shape and y.dtype == torch.float16
    assert_gemm_close(y, ref, "MatMul4Bit fwd")
    torch.testing.assert_close(y.double(), ref, rtol=2e-3, atol=2e-3)
    assert x.grad.dtype == torch.float16
    assert_gemm_close(x.grad, ref_dx, "MatMul4Bit dX")
    torch.testing.assert_close(x.grad.double(), ref_dx, rtol=2e-3, atol=2e-3)
    _check_flag()


@pytest.mark.parametrize("n", [1170, 2048, 8192])
@pytest.mark.parametrize("proj", list(QWEN))
def test_fused_forward_qwen_shapes(cuda_lib, proj, n):
    """Every projection shape at every token count: the planner picks the tiling (single,
    128-token, pair, split-K) per shape and N, so each case can take a different path."""
    from stew_b200.nf4 import linear_forward
    out_f, in_f = QWEN[proj]
    q, st = _weight((out_f, in_f), 100 + list(QWEN).index(proj))
    x = _x(n, in_f, 7)
    y = linear_forward(x, q.view(-1, 1), st)
    ref = x.double() @ _ref_weight(q, st).T
    assert_gemm_close(y, ref, f"{proj} fwd N={n}")
    _check_flag()


@pytest.mark.parametrize("n", [1170, 2048, 8192])
@pytest.mark.parametrize("proj", list(QWEN))
def test_fused_backward_qwen_shapes(cuda_lib, proj, n):
    """dX = dY W with dY ~ N(0, 1e-2) (std 0.01)."""
    from stew_b200.nf4 import linear_backward_dx
    out_f, in_f = QWEN[proj]
    q, st = _weight((out_f, in_f), 200 + list(QWEN).index(proj))
    dy = _x(n, out_f, 9, std=0.01)
    dx = linear_backward_dx(dy, q.view(-1, 1), st)
    ref = dy.double() @ _ref_weight(q, st)
    assert dx.shape == (n, in_f)
    assert_gemm_close(dx, ref, f"{proj} bwd N={n}")
    _check_flag()


@pytest.mark.parametrize("n", [1, 15, 16, 17, 255, 256, 257, 600])
def test_ragged_token_counts(cuda_lib, n):
    """Token tiles that are partial, single rows, and not multiples of 16."""
    from stew_b200.nf4 import linear_backward_dx, linear_forward
    q, st = _weight((384, 320), 5)
    W = _ref_weight(q, st)
    x = _x(n, 320, n)
    assert_gemm_close(linear_forward(x, q.view(-1, 1), st), x.double() @ W.T, f"fwd N={n}")
    dy = _x(n, 384, n + 1)
    assert_gemm_close(linear_backward_dx(dy, q.view(-1, 1), st), dy.double() @ W, f"bwd N={n}")
    _check_flag()


@pytest.mark.parametrize("blocksize", [32, 64, 128, 256])
@pytest.mark.parametrize("nested", [True, False])
def test_blocksizes_and_plain_absmax(cuda_lib, blocksize, nested):
    from stew_b200.nf4 import linear_backward_dx, linear_forward
    q, st = _weight((256, 512), blocksize + int(nested), blocksize=blocksize, nested=nested)
    W = _ref_weight(q, st)
    x = _x(300, 512, 3)
    assert_gemm_close(linear_forward(x, q.view(-1, 1), st), x.double() @ W.T, "fwd")
    dy = _x(300, 256, 4)
    assert_gemm_close(linear_backward_dx(dy, q.view(-1, 1), st), dy.double() @ W, "bwd")
    _check_flag()


def test_forward_bias_and_outputs_exact_layout(cuda_lib):
    """Every output element is written (no stale values): run into a NaN-filled buffer."""
    import ctypes
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate, _stream
    q, st = _weight((192, 256), 21)
    x = _x(77, 256, 1)
    bias = torch.randn(192, device="cuda", dtype=torch.float16)
    y = torch.full((77, 192), float("nan"), dtype=torch.float16, device="cuda")
    qs = _qstate(st, x.device)
    _lib.check(_lib.lib().nf4b_linear_fwd(x.data_ptr(), q.data_ptr(), ctypes.byref(qs), bias.data_ptr(),
                                          None, y.data_ptr(), 77, 256, 192, _stream(x.device)), "fwd")
    ref = x.double() @ _ref_weight(q, st).T + bias.double()
    assert not torch.isnan(y).any()
    assert_gemm_close(y, ref, "fwd + bias")
