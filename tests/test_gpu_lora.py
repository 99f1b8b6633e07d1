"""GPU parity of the fused NF4 + LoRA (r=16, alpha=32 -> scaling 2, dropout 0) path on
the q/v shapes: forward output, dX, dA, dB against fp64 autograd of
y = x W^T + (x A^T) B^T * s with W the oracle-dequantised weight.
Tolerance: max |got - ref| / max |ref| <= 2e-3 for y and dX (fp16 outputs), and elementwise
2e-3 above 0.05 max |ref|; 1e-3 (max-normalised) for the fp32 weight gradients."""
import math

import pytest
import torch

from tests.helpers import assert_gemm_close, max_rel_err
from tests.test_gpu_gemm import _ref_weight, _weight, _x, _check_flag

pytestmark = pytest.mark.gpu


def _lora(in_f, out_f, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    bound = 1.0 / math.sqrt(in_f)  # kaiming_uniform(a=sqrt(5)) on [16, in]
    a = (torch.rand(16, in_f, generator=g, device="cuda") * 2 - 1) * bound
    b = torch.randn(out_f, 16, generator=g, device="cuda") * 0.01
    return a.requires_grad_(True), b.requires_grad_(True)


@pytest.mark.parametrize("n", [74, 1170, 2048, 8192])
@pytest.mark.parametrize("proj", ["q", "v"])
def test_fused_lora_forward_backward(cuda_lib, proj, n):
    from stew_b200 import nf4_lora_linear
    out_f, in_f = (1536, 1536) if proj == "q" else (256, 1536)
    q, st = _weight((out_f, in_f), 300 + n)
    a, b = _lora(in_f, out_f, 17)
    x = _x(n, in_f, 5).requires_grad_(True)
    dy = _x(n, out_f, 6, std=0.01)
    y = nf4_lora_linear(x, q, st, a, b, 2.0)
    y.backward(dy)
    W = _ref_weight(q, st)
    xd = x.detach().double().requires_grad_(True)
    ad = a.detach().double().requires_grad_(True)
    bd = b.detach().double().requires_grad_(True)
    ref = xd @ W.T + (xd @ ad.T) @ bd.T * 2.0
    ref.backward(dy.double())
    assert_gemm_close(y, ref.detach(), f"{proj} y N={n}")
    assert_gemm_close(x.grad, xd.grad, f"{proj} dX N={n}")
    # fp16 activations and x A^T rounded to fp16 (as peft's autocast produces it)
    assert max_rel_err(a.grad, ad.grad) <= 1e-3
    assert max_rel_err(b.grad, bd.grad) <= 1e-3
    # (no elementwise bound for dA / dB: each is a sum over tokens of products with the fp16
    # rank-16 intermediate dY B or X A^T, and at small token counts a one-ulp difference in
    # that intermediate moves a partly cancelling sum by more than 2e-3 of itself)
    assert a.grad.dtype == torch.float32 and b.grad.dtype == torch.float32
    _check_flag()


@pytest.mark.parametrize("n", [77, 1170])
@pytest.mark.parametrize("shape", [(8960, 1536), (1536, 8960)])
def test_fused_lora_on_wide_projections(cuda_lib, shape, n):
    """An adapter on the MLP shapes: with 8960 output features the backward's dY B runs over
    K = 8960, so each warp stages its slice of B in several rounds (eight 32-wide chunks a round);
    with 8960 input features the forward's X A^T does.  Same checks as above."""
    from stew_b200 import nf4_lora_linear
    out_f, in_f = shape
    q, st = _weight((out_f, in_f), 400 + n)
    a, b = _lora(in_f, out_f, 19)
    x = _x(n, in_f, 7).requires_grad_(True)
    dy = _x(n, out_f, 8, std=0.01)
    y = nf4_lora_linear(x, q, st, a, b, 2.0)
    y.backward(dy)
    W = _ref_weight(q, st)
    xd = x.detach().double().requires_grad_(True)
    ad = a.detach().double().requires_grad_(True)
    bd = b.detach().double().requires_grad_(True)
    ref = xd @ W.T + (xd @ ad.T) @ bd.T * 2.0
    ref.backward(dy.double())
    assert_gemm_close(y, ref.detach(), f"{shape} y N={n}")
    assert_gemm_close(x.grad, xd.grad, f"{shape} dX N={n}")
    assert max_rel_err(a.grad, ad.grad) <= 1e-3
    assert max_rel_err(b.grad, bd.grad) <= 1e-3
    _check_flag()


def test_lora_term_is_applied(cuda_lib):
    """With B != 0 the adapter changes the output by exactly its own contribution."""
    from stew_b200 import nf4_lora_linear
    from stew_b200.nf4 import linear_forward
    q, st = _weight((256, 512), 9)
    a, b = _lora(512, 256, 3)
    with torch.no_grad():
        b.mul_(100.0)
    x = _x(130, 512, 2)
    y = nf4_lora_linear(x, q, st, a.detach(), b.detach(), 2.0)
    base = linear_forward(x, q.view(-1, 1), st)
    delta = (x.double() @ a.detach().double().T) @ b.detach().double().T * 2.0
    assert max_rel_err(y.double() - base.double(), delta) <= 5e-3


def test_lora_module_trains(cuda_lib):
    """NF4LoraLinear: only the adapter gets gradients; one SGD step lowers the loss."""
    from stew_b200 import NF4LoraLinear
    q, st = _weight((256, 512), 4)
    m = NF4LoraLinear(q, st)
    torch.nn.init.normal_(m.lora_B, std=0.01)
    x = _x(64, 512, 8)
    target = torch.randn(64, 256, device="cuda")
    opt = torch.optim.SGD(m.parameters(), lr=1e-2)
    losses = []
    for _ in range(3):
        opt.zero_grad()
        loss = (m(x).float() - target).pow(2).mean()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0]
    assert [p.shape for p in m.parameters()] == [torch.Size([16, 512]), torch.Size([256, 16])]


@pytest.mark.parametrize("n", [1, 77, 1311])
def test_grouped_lora_grads_match_per_adapter_calls(cuda_lib, n):
    """nf4b_lora_grads_group (q and v adapters of one layer: dA, dB of both in one launch) gives
    the dA / dB of one nf4b_lora_grads call per adapter up to fp32 summation order (the group
    splits the tokens differently), repeats bit for bit (fixed reduction order), and matches the
    fp64 products."""
    import ctypes
    from stew_b200 import _lib
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator(device="cuda").manual_seed(n)
    x = torch.randn(n, 1536, generator=g, device="cuda").half()
    shapes = [(1536, 2.0), (256, 2.0)]
    items, refs, keep = [], [], []
    for out_f, s in shapes:
        dy = (torch.randn(n, out_f, generator=g, device="cuda") * 0.01).half()
        xa = torch.randn(n, 16, generator=g, device="cuda").half()
        dyb = (torch.randn(n, 16, generator=g, device="cuda") * 0.1).half()
        da = torch.full((16, 1536), float("nan"), device="cuda")
        db = torch.full((out_f, 16), float("nan"), device="cuda")
        it = _lib.LoraGradsItemC()
        it.x, it.dy, it.xa, it.dyb = x.data_ptr(), dy.data_ptr(), xa.data_ptr(), dyb.data_ptr()
        it.scale, it.da, it.db, it.in_features, it.out_features = s, da.data_ptr(), db.data_ptr(), 1536, out_f
        items.append(it)
        keep.append((dy, xa, dyb, da, db, out_f, s))
    arr = (_lib.LoraGradsItemC * 2)(*items)
    wb = int(L.nf4b_lora_grads_group_work_bytes(arr, 2, n))
    assert (wb > 0) == (n > 64), "tokens are split in ranges of at least 64"
    work = torch.zeros(wb // 4 + 4, device="cuda")  # ticket words zero before the first call
    assert L.nf4b_lora_grads_group(arr, 2, work.data_ptr(), wb, n, stream) == 0, L.nf4b_last_error()
    if wb > 0:
        assert L.nf4b_lora_grads_group(arr, 2, work.data_ptr(), wb - 4, n, stream) == _lib.NF4B_ERR_INVALID_ARG
    first = [(da.clone(), db.clone()) for _, _, _, da, db, _, _ in keep]
    assert L.nf4b_lora_grads_group(arr, 2, work.data_ptr(), wb, n, stream) == 0, L.nf4b_last_error()
    assert int(work[:1024].view(torch.int32).count_nonzero()) == 0, "ticket words must be left zero"
    for (da0, db0), (dy, xa, dyb, da, db, out_f, s) in zip(first, keep):
        torch.cuda.synchronize()
        assert torch.equal(da0, da) and torch.equal(db0, db), "a repeated call differs"
        da1 = torch.empty(16, 1536, device="cuda")
        db1 = torch.empty(out_f, 16, device="cuda")
        w1 = torch.zeros(max(int(L.nf4b_lora_grads_work_bytes(n, 1536, out_f, 16)), 16) // 4 + 4, device="cuda")
        assert L.nf4b_lora_grads(x.data_ptr(), dy.data_ptr(), xa.data_ptr(), dyb.data_ptr(), s, da1.data_ptr(),
                                 db1.data_ptr(), w1.data_ptr(), n, 1536, out_f, 16, stream) == 0
        torch.cuda.synchronize()
        assert max_rel_err(da, da1) <= 1e-5 and max_rel_err(db, db1) <= 1e-5
        assert max_rel_err(da, s * dyb.double().T @ x.double()) <= 1e-3
        assert max_rel_err(db, s * dy.double().T @ xa.double()) <= 1e-3
