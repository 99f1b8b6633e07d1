"""GPU: the layer kernels of the QLoRA step (include/stew_step.h, stew_b200.step_ops) against
fp32 torch restatements of the same formulas, forward and backward.
Tolerances (written here): forward outputs bit-identical where the rounding points are the
same (residual sum, RoPE), within 2 fp16 ulp for RMSNorm (its statistic is summed in another
order) and 1 ulp for SwiGLU (expf); input gradients within 2e-3 of
max |ref| (fp16 outputs of fp32 math)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

GRAD_TOL = 2e-3


def _rel(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max().clamp_min(1e-30))


def _ulp_close(a, b, n=1):
    """|a - b| <= n ulp of fp16 at the magnitude of b."""
    bd = b.double()
    ulp = torch.where(bd.abs() < 6.1e-5, torch.full_like(bd, 2.0 ** -24),
                      2.0 ** (torch.floor(torch.log2(bd.abs().clamp_min(1e-30))) - 10))
    return bool(((a.double() - bd).abs() <= n * ulp + 1e-12).all())


def _ref_norm(x, w, eps):
    xf = x.float()
    xn = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(torch.float16)
    return (w * xn.float()).to(torch.float16)


def _ref_norm_f32(x, w, eps):  # differentiable fp32 form for the gradient reference
    return w * x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


@pytest.mark.parametrize("rows,hidden", [(1, 256), (37, 1536), (1311, 1536), (5, 4096)])
def test_rmsnorm_forward_backward(cuda_lib, rows, hidden):
    from stew_b200.step_ops import rms_norm
    g = torch.Generator(device="cuda").manual_seed(rows)
    x = (torch.randn(rows, hidden, device="cuda", generator=g) * 3).half()
    w = torch.rand(hidden, device="cuda", generator=g) + 0.5
    dy = torch.randn(rows, hidden, device="cuda", generator=g).half()
    xr = x.clone().requires_grad_(True)
    y = rms_norm(xr, w, 1e-6)
    y.backward(dy)
    assert _ulp_close(y, _ref_norm(x, w, 1e-6), 2)  # rsqrt of a differently ordered sum
    xf = x.float().requires_grad_(True)
    _ref_norm_f32(xf, w, 1e-6).backward(dy.float())
    assert _rel(xr.grad, xf.grad) <= GRAD_TOL


def test_add_rmsnorm_forward_backward(cuda_lib):
    from stew_b200.step_ops import add_rms_norm
    rows, hidden = 300, 1536
    g = torch.Generator(device="cuda").manual_seed(1)
    res = torch.randn(rows, hidden, device="cuda", generator=g).half()
    delta = (torch.randn(rows, hidden, device="cuda", generator=g) * 0.1).half()
    w = torch.ones(hidden, device="cuda")
    ds = (torch.randn(rows, hidden, device="cuda", generator=g) * 0.3).half()
    dy = torch.randn(rows, hidden, device="cuda", generator=g).half()
    r, d = res.clone().requires_grad_(True), delta.clone().requires_grad_(True)
    s, y = add_rms_norm(r, d, w, 1e-6)
    (s.float() * ds.float()).sum().add((y.float() * dy.float()).sum()).backward()
    assert torch.equal(s, res + delta)
    assert _ulp_close(y, _ref_norm(res + delta, w, 1e-6), 2)
    sf = (res + delta).float().requires_grad_(True)
    (sf * ds.float()).sum().add((_ref_norm_f32(sf, w, 1e-6) * dy.float()).sum()).backward()
    assert _rel(r.grad, sf.grad) <= GRAD_TOL and torch.equal(r.grad, d.grad)


def _ref_rope(x, cos, sin):
    xf = x.float()
    d = xf.shape[-1] // 2
    rot = torch.cat([-xf[..., d:], xf[..., :d]], dim=-1)
    return xf * cos[:, None, :] + rot * sin[:, None, :]


@pytest.mark.parametrize("tokens", [1, 77, 1311])
def test_rope_qk_forward_backward(cuda_lib, tokens):
    from stew_b200.qlora_step import rope_tables
    from stew_b200.step_ops import rope_qk
    g = torch.Generator(device="cuda").manual_seed(tokens)
    pos = torch.randint(0, 512, (tokens,), device="cuda", generator=g)
    cos, sin = rope_tables(pos, 128, 1e6)
    q = torch.randn(tokens, 12, 128, device="cuda", generator=g).half()
    k = torch.randn(tokens, 2, 128, device="cuda", generator=g).half()
    dq = torch.randn(tokens, 12, 128, device="cuda", generator=g).half()
    dk = torch.randn(tokens, 2, 128, device="cuda", generator=g).half()
    qr, kr = q.clone().requires_grad_(True), k.clone().requires_grad_(True)
    qo, ko = rope_qk(qr, kr, cos, sin)
    (qo.float() * dq.float()).sum().add((ko.float() * dk.float()).sum()).backward()
    assert torch.equal(qo, _ref_rope(q, cos, sin).half())
    assert torch.equal(ko, _ref_rope(k, cos, sin).half())
    qf, kf = q.float().requires_grad_(True), k.float().requires_grad_(True)
    (_ref_rope(qf, cos, sin) * dq.float()).sum().add((_ref_rope(kf, cos, sin) * dk.float()).sum()).backward()
    assert _rel(qr.grad, qf.grad) <= GRAD_TOL and _rel(kr.grad, kf.grad) <= GRAD_TOL


@pytest.mark.parametrize("n,cols", [(1, 8), (1311, 8960)])
def test_swiglu_forward_backward(cuda_lib, n, cols):
    from stew_b200.step_ops import swiglu
    g = torch.Generator(device="cuda").manual_seed(n)
    gate = (torch.randn(n, cols, device="cuda", generator=g) * 2).half()
    up = torch.randn(n, cols, device="cuda", generator=g).half()
    dm = torch.randn(n, cols, device="cuda", generator=g).half()
    gr, ur = gate.clone().requires_grad_(True), up.clone().requires_grad_(True)
    m = swiglu(gr, ur)
    m.backward(dm)
    # the reference kernel's rounding points (solution/swiglu.py): g * sigmoid(g) * u, one rounding
    gd = gate.double()
    ref = gd * torch.sigmoid(gd) * up.double()
    assert _ulp_close(m, ref)
    gf, uf = gate.float().requires_grad_(True), up.float().requires_grad_(True)
    (F.silu(gf) * uf).backward(dm.float())
    assert _rel(gr.grad, gf.grad) <= GRAD_TOL and _rel(ur.grad, uf.grad) <= GRAD_TOL


def test_step_ops_argument_checks(cuda_lib):
    from stew_b200 import _lib
    L = _lib.lib()
    assert L.nf4b_rmsnorm_fwd(16, None, 16, 1e-6, None, 16, 16, 4, 1000, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_swiglu_fwd(16, 16, 16, 12, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_rope_qk(16, 16, 16, 16, 16, 16, 1, 1, 1, 100, 0, None) == _lib.NF4B_ERR_UNSUPPORTED


@pytest.mark.parametrize("rows,vocab,hidden", [(1, 1000, 64), (77, 4096, 256), (1307, 151936, 1536)])
def test_head_cross_entropy_forward_backward(cuda_lib, rows, vocab, hidden):
    """Fused LM-head loss (nf4b_ce_fwd/_bwd) against F.cross_entropy on the same fp16 logits
    in fp32: the summed loss within 1e-5 relative (summation order), dh within 2e-3 of
    max |ref| (fp16 gradient of the logits, scaled by 1024 on the way); ignored labels (-100)
    add nothing."""
    from stew_b200.step_ops import head_cross_entropy
    g = torch.Generator(device="cuda").manual_seed(rows + vocab)
    h = (torch.randn(rows, hidden, generator=g, device="cuda") * 2.0).half()
    emb = (torch.randn(vocab, hidden, generator=g, device="cuda") * 0.05).half()
    labels = torch.randint(0, vocab, (rows,), generator=g, device="cuda")
    if rows > 2:
        labels[::7] = -100
    hx = h.clone().requires_grad_(True)
    loss = head_cross_entropy(hx, emb, labels)
    loss.backward()
    hr = h.clone().requires_grad_(True)
    logits = hr @ emb.t()  # the same fp16 GEMM
    ref = F.cross_entropy(logits.float(), labels, reduction="sum", ignore_index=-100)
    ref.backward()
    assert abs(float(loss) - float(ref)) <= 1e-5 * abs(float(ref)) + 1e-4
    assert _rel(hx.grad, hr.grad.float()) <= GRAD_TOL
    if rows > 2:  # an ignored row's gradient is exactly zero
        assert float(hx.grad[0].abs().max()) == 0.0
