"""GPU: the SwiGLU applied in the gate/up GEMM's epilogue (nf4b_linear_fwd_swiglu).

It must give, bit for bit, what the two-step form gives -- the grouped gate/up launch
(nf4b_linear_fwd_group) followed by the SwiGLU kernel m = fp16(g * sigmoid(g) * u)
(nf4b_swiglu_fwd, the rounding points of the reference's SwiGLU kernel, solution/swiglu.py:16-23,
called by solution/unpad.py:60-63): both launches plan the same tiles, so every accumulator sums the
same K ranges in the same order.  Covered: single-CTA, 2-CTA pair, split-K and 128-token plans
(the planner's choice per token count, and forced), ragged token counts, the Qwen2.5-1.5B MLP
shape, plain and double-quantized states; g and u also against the fp64 product of the
oracle-dequantised weights (GEMM tolerance); and the autograd op's backward against the
unfused composition.
"""
import ctypes

import pytest
import torch

from tests.helpers import assert_gemm_close
from tests.test_gpu_gemm import _ref_weight, _weight, _x

pytestmark = pytest.mark.gpu


def _two_step(x, gate, up):
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate, _stream
    L = _lib.lib()
    (pg, sg), (pu, su) = gate, up
    n, in_f = x.shape
    out_f = int(sg.shape[0])
    g = torch.empty(n, out_f, dtype=torch.float16, device="cuda")
    u = torch.empty_like(g)
    m = torch.empty_like(g)
    items = (_lib.LinearItemC * 2)()
    qs = [_qstate(sg, x.device), _qstate(su, x.device)]
    for j, (packed, q, y) in enumerate(((pg, qs[0], g), (pu, qs[1], u))):
        items[j].packed, items[j].qs, items[j].bias, items[j].lora = packed.data_ptr(), ctypes.pointer(q), None, None
        items[j].y, items[j].out_features = y.data_ptr(), out_f
    outs = (ctypes.c_int64 * 2)(out_f, out_f)
    wb = max(int(L.nf4b_linear_group_work_bytes(n, in_f, outs, 2)), 256)
    ws = torch.zeros(wb, dtype=torch.uint8, device="cuda")
    _lib.check(L.nf4b_linear_fwd_group(x.data_ptr(), n, in_f, items, 2, ws.data_ptr(), wb, _stream(x.device)), "grp")
    _lib.check(L.nf4b_swiglu_fwd(g.data_ptr(), u.data_ptr(), m.data_ptr(), g.numel(), _stream(x.device)), "swiglu")
    return g, u, m


def _fused(x, gate, up):
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate, _stream
    L = _lib.lib()
    (pg, sg), (pu, su) = gate, up
    n, in_f = x.shape
    out_f = int(sg.shape[0])
    g = torch.full((n, out_f), float("nan"), dtype=torch.float16, device="cuda")
    u = torch.full_like(g, float("nan"))
    m = torch.full_like(g, float("nan"))
    wb = max(int(L.nf4b_linear_swiglu_work_bytes(n, in_f, out_f)), 256)
    ws = torch.zeros(wb, dtype=torch.uint8, device="cuda")
    qg, qu = _qstate(sg, x.device), _qstate(su, x.device)
    _lib.check(L.nf4b_linear_fwd_swiglu(x.data_ptr(), n, in_f, pg.data_ptr(), ctypes.byref(qg), pu.data_ptr(),
                                        ctypes.byref(qu), g.data_ptr(), u.data_ptr(), m.data_ptr(), out_f,
                                        ws.data_ptr(), wb, _stream(x.device)), "swiglu fused")
    assert int(ws[:4100].count_nonzero()) == 0, "split-K counters must be left zero"
    return g, u, m


@pytest.mark.parametrize("pair", ["auto", "0", "1"])
@pytest.mark.parametrize("n", [1, 77, 600, 1170, 2048, 8192])
def test_fused_swiglu_equals_two_step_qwen_mlp(cuda_lib, monkeypatch, n, pair):
    from stew_b200 import _lib
    if pair != "auto":
        monkeypatch.setenv("STEW_NF4_PAIR", pair)
    gate, up = _weight((8960, 1536), 1), _weight((8960, 1536), 2)
    x = _x(n, 1536, 3)
    g0, u0, m0 = _two_step(x, gate, up)
    g1, u1, m1 = _fused(x, gate, up)
    torch.cuda.synchronize()
    assert torch.equal(g0, g1) and torch.equal(u0, u1), "gate/up differ from the grouped launch"
    assert torch.equal(m0, m1), "SwiGLU differs from the SwiGLU kernel"
    if n in (77, 1170):
        assert_gemm_close(g1, x.double() @ _ref_weight(*gate).T, "gate")
        assert_gemm_close(u1, x.double() @ _ref_weight(*up).T, "up")
    assert _lib.gemm_error_flag(reset=True) == 0


@pytest.mark.parametrize("tile_n", ["128", "256"])
@pytest.mark.parametrize("shape,n", [((256, 512), 300), ((640, 768), 1), ((384, 4096), 77)])
@pytest.mark.parametrize("nested", [True, False])
def test_fused_swiglu_small_and_split_shapes(cuda_lib, monkeypatch, shape, n, nested, tile_n):
    """Few tiles (split-K on long K), 128-token tiles, ragged token counts, plain absmax."""
    monkeypatch.setenv("STEW_NF4_TILE_N", tile_n)
    gate = _weight(shape, 10 + n, nested=nested)
    up = _weight(shape, 20 + n, nested=nested)
    x = _x(n, shape[1], 4)
    g0, u0, m0 = _two_step(x, gate, up)
    g1, u1, m1 = _fused(x, gate, up)
    torch.cuda.synchronize()
    assert torch.equal(g0, g1) and torch.equal(u0, u1) and torch.equal(m0, m1)


def test_swiglu_projection_autograd_matches_composition(cuda_lib):
    """The MLP's autograd op: m and dX equal the unfused composition (grouped projection +
    SwiGLU kernel) bit for bit."""
    from stew_b200.lora import NF4Linear, grouped_projection, swiglu_projection
    from stew_b200.step_ops import swiglu
    (pg, sg), (pu, su) = _weight((8960, 1536), 5), _weight((8960, 1536), 6)
    gate, up = NF4Linear(pg, sg), NF4Linear(pu, su)
    x0 = _x(1170, 1536, 7)
    dm = _x(1170, 8960, 8, std=0.01)
    xa = x0.clone().requires_grad_(True)
    ma = swiglu_projection(xa, gate, up)
    ma.backward(dm)
    xb = x0.clone().requires_grad_(True)
    gb, ub = grouped_projection(xb, [gate, up])
    mb = swiglu(gb, ub)
    mb.backward(dm)
    torch.cuda.synchronize()
    assert torch.equal(ma, mb)
    assert torch.equal(xa.grad, xb.grad)


@pytest.mark.parametrize("pair", ["auto", "0", "1"])
@pytest.mark.parametrize("n", [1, 77, 1170, 2048, 8192])
def test_down_dx_with_swiglu_backward_equals_two_step(cuda_lib, monkeypatch, n, pair):
    """nf4b_linear_bwd_dx_swiglu (down's dX with the SwiGLU backward in its epilogue) gives, bit for
    bit, dX of down (nf4b_linear_bwd_dx_ws) followed by nf4b_swiglu_bwd -- single-CTA, pair and
    split-K plans of the Qwen2.5-1.5B down projection (1536 x 8960)."""
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate, _stream
    if pair != "auto":
        monkeypatch.setenv("STEW_NF4_PAIR", pair)
    L = _lib.lib()
    pd, sd = _weight((1536, 8960), 31)
    dy = _x(n, 1536, 32, std=0.01)
    gate = _x(n, 8960, 33, std=2.0)
    up = _x(n, 8960, 34)
    qd = _qstate(sd, dy.device)
    wb = max(int(L.nf4b_linear_work_bytes(n, 8960, 1536, 1)), 256)
    ws = torch.zeros(wb, dtype=torch.uint8, device="cuda")
    st = _stream(dy.device)
    dm = torch.empty(n, 8960, dtype=torch.float16, device="cuda")
    _lib.check(L.nf4b_linear_bwd_dx_ws(dy.data_ptr(), pd.data_ptr(), ctypes.byref(qd), None, None, dm.data_ptr(),
                                       n, 8960, 1536, ws.data_ptr(), wb, st), "bwd")
    dg0, du0 = torch.empty_like(dm), torch.empty_like(dm)
    _lib.check(L.nf4b_swiglu_bwd(dm.data_ptr(), gate.data_ptr(), up.data_ptr(), dg0.data_ptr(), du0.data_ptr(),
                                 dm.numel(), st), "swiglu bwd")
    dg1 = torch.full_like(dm, float("nan"))
    du1 = torch.full_like(dm, float("nan"))
    _lib.check(L.nf4b_linear_bwd_dx_swiglu(dy.data_ptr(), pd.data_ptr(), ctypes.byref(qd), gate.data_ptr(),
                                           up.data_ptr(), dg1.data_ptr(), du1.data_ptr(), n, 8960, 1536,
                                           ws.data_ptr(), wb, st), "bwd swiglu")
    torch.cuda.synchronize()
    assert torch.equal(dg0, dg1) and torch.equal(du0, du1)
    assert int(ws[:4100].count_nonzero()) == 0
    assert _lib.gemm_error_flag(reset=True) == 0


@pytest.mark.parametrize("fused_backward", [False, True])
@pytest.mark.parametrize("recompute", [False, True])
def test_mlp_op_matches_composition(cuda_lib, recompute, fused_backward):
    """lora.MLPFunction against the composition it replaces -- grouped gate/up projection, SwiGLU
    kernel, down projection -- output and dX bit for bit, with the SwiGLU backward as its own
    kernel or in down's dX epilogue; with recompute the backward's second gate/up launch gives
    the same."""
    from stew_b200.lora import NF4Linear, grouped_projection, nf4_mlp
    from stew_b200.step_ops import swiglu
    (pg, sg), (pu, su), (pd, sd) = _weight((8960, 1536), 41), _weight((8960, 1536), 42), _weight((1536, 8960), 43)
    gate, up, down = NF4Linear(pg, sg), NF4Linear(pu, su), NF4Linear(pd, sd)
    x0 = _x(1170, 1536, 44)
    dy = _x(1170, 1536, 45, std=0.01)
    xa = x0.clone().requires_grad_(True)
    ya = nf4_mlp(xa, gate, up, down, recompute=recompute, fused_backward=fused_backward)
    ya.backward(dy)
    xb = x0.clone().requires_grad_(True)
    gb, ub = grouped_projection(xb, [gate, up])
    yb = down(swiglu(gb, ub))
    yb.backward(dy)
    torch.cuda.synchronize()
    assert torch.equal(ya, yb)
    assert torch.equal(xa.grad, xb.grad)
