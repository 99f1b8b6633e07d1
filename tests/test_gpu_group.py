"""GPU: grouped forward launches (nf4b_linear_fwd_group) -- q/k/v and gate/up sharing one
activation in ONE launch -- against the fp64 product of the oracle-dequantised weights and
against one launch per projection; and the grouped autograd op of the QLoRA step against
separate fused projections.  Tolerances (written here): max |y - ref| / max |ref| <= 2e-3;
grouped vs separate launches <= 1e-3 (split-K plans differ); gradients <= 2e-3."""
import ctypes

import pytest
import torch

from tests.helpers import GEMM_MAX_REL_ERR, max_rel_err
from tests.test_gpu_gemm import _check_flag, _ref_weight, _weight, _x

pytestmark = pytest.mark.gpu


def _items(specs, n, dev="cuda"):
    """specs: (out_f, in_f, seed, with_bias, with_lora) -> C items + the tensors they point to."""
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate
    items = (_lib.LinearItemC * len(specs))()
    keep = []
    for i, (out_f, in_f, seed, with_bias, with_lora) in enumerate(specs):
        q, st = _weight((out_f, in_f), seed)
        qs = _qstate(st, q.device)
        bias = _x(1, out_f, seed + 1).reshape(out_f) if with_bias else None
        y = torch.full((n, out_f), float("nan"), dtype=torch.float16, device=dev)
        lc = a = b = xa = None
        if with_lora:
            g = torch.Generator(device=dev).manual_seed(seed + 2)
            a = ((torch.rand(16, in_f, generator=g, device=dev) * 2 - 1) / in_f ** 0.5).half()
            b = (torch.randn(out_f, 16, generator=g, device=dev) * 0.05).half()
            xa = torch.empty(n, 16, dtype=torch.float16, device=dev)
            lc = _lib.LoraC()
            lc.a, lc.b, lc.scale, lc.rank, lc.xa = a.data_ptr(), b.data_ptr(), 2.0, 16, xa.data_ptr()
        items[i].packed = q.data_ptr()
        items[i].qs = ctypes.pointer(qs)
        items[i].bias = None if bias is None else bias.data_ptr()
        items[i].lora = None if lc is None else ctypes.pointer(lc)
        items[i].y = y.data_ptr()
        items[i].out_features = out_f
        keep.append(dict(q=q, st=st, qs=qs, bias=bias, y=y, lc=lc, a=a, b=b, xa=xa))
    return items, keep


def _ref(x, k):
    ref = x.double() @ _ref_weight(k["q"], k["st"]).T
    if k["bias"] is not None:
        ref = ref + k["bias"].double()
    if k["lc"] is not None:
        ref = ref + 2.0 * (x.double() @ k["a"].double().T) @ k["b"].double().T
    return ref


QKV = [(1536, 1536, 11, True, True), (256, 1536, 12, True, False), (256, 1536, 13, True, True)]
GATE_UP = [(8960, 1536, 21, False, False), (8960, 1536, 22, False, False)]


@pytest.mark.parametrize("specs", [QKV, GATE_UP, QKV[1:]], ids=["qkv", "gate_up", "kv"])
@pytest.mark.parametrize("n", [77, 1170, 2048])
def test_grouped_forward_matches_reference_and_separate(cuda_lib, specs, n):
    from stew_b200 import _lib
    from stew_b200.nf4 import _stream
    L = _lib.lib()
    x = _x(n, 1536, 3)
    items, keep = _items(specs, n)
    outs = (ctypes.c_int64 * len(specs))(*[s[0] for s in specs])
    need = int(L.nf4b_linear_group_work_bytes(n, 1536, outs, len(specs)))
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    _lib.check(L.nf4b_linear_fwd_group(x.data_ptr(), n, 1536, items, len(specs), ws.data_ptr(),
                                       ws.numel(), _stream(x.device)), "group")
    torch.cuda.synchronize()
    for k in keep:
        assert not torch.isnan(k["y"]).any()
        assert max_rel_err(k["y"], _ref(x, k)) <= GEMM_MAX_REL_ERR
    # one launch per projection gives the same outputs
    for k, (out_f, in_f, *_r) in zip(keep, specs):
        y1 = torch.empty_like(k["y"])
        _lib.check(L.nf4b_linear_fwd(x.data_ptr(), k["q"].data_ptr(), ctypes.byref(k["qs"]),
                                     None if k["bias"] is None else k["bias"].data_ptr(),
                                     None if k["lc"] is None else ctypes.byref(k["lc"]), y1.data_ptr(), n,
                                     in_f, out_f, _stream(x.device)), "single")
        torch.cuda.synchronize()
        assert max_rel_err(k["y"], y1.double()) <= 1e-3
    assert int(ws[:4096].count_nonzero()) == 0
    _check_flag()


def test_grouped_argument_checks(cuda_lib):
    from stew_b200 import _lib
    L = _lib.lib()
    items = (_lib.LinearItemC * 4)()
    assert L.nf4b_linear_fwd_group(16, 8, 64, items, 4, None, 0, None) == _lib.NF4B_ERR_UNSUPPORTED
    assert L.nf4b_linear_fwd_group(16, 8, 64, items, 0, None, 0, None) == _lib.NF4B_ERR_INVALID_ARG


def test_grouped_projection_autograd_matches_separate(cuda_lib):
    """GroupedNF4Function (one forward launch for q/k/v) vs the three fused modules called
    one by one: outputs, dX, and the adapters' gradients."""
    from stew_b200.lora import NF4Linear, NF4LoraLinear, grouped_projection
    torch.manual_seed(0)
    mods = []
    for out_f, seed, lora in ((1536, 31, True), (256, 32, False), (256, 33, True)):
        q, st = _weight((out_f, 1536), seed)
        bias = (torch.randn(out_f, device="cuda") * 0.02).half()
        if lora:
            m = NF4LoraLinear(q, st, bias=bias, device="cuda")
            torch.nn.init.normal_(m.lora_B, std=0.02)
        else:
            m = NF4Linear(q, st, bias=bias)
        mods.append(m)
    x = _x(700, 1536, 5)
    dys = [_x(700, m.out_features, 6 + i, std=0.01) for i, m in enumerate(mods)]
    xg = x.clone().requires_grad_(True)
    outs = grouped_projection(xg, mods)
    sum((o.float() * d.float()).sum() for o, d in zip(outs, dys)).backward()
    g_grads = [(p.grad.clone()) for m in mods if isinstance(m, NF4LoraLinear) for p in (m.lora_A, m.lora_B)]
    for m in mods:
        for p in m.parameters():
            p.grad = None
    xs = x.clone().requires_grad_(True)
    outs_s = [m(xs) for m in mods]
    sum((o.float() * d.float()).sum() for o, d in zip(outs_s, dys)).backward()
    s_grads = [p.grad for m in mods if isinstance(m, NF4LoraLinear) for p in (m.lora_A, m.lora_B)]
    for a, b in zip(outs, outs_s):
        assert max_rel_err(a, b.double()) <= 1e-3
    assert max_rel_err(xg.grad, xs.grad.double()) <= 2e-3
    for a, b in zip(g_grads, s_grads):
        assert max_rel_err(a, b.double()) <= 2e-3
    _check_flag()


BWD_QKV = [(1536, 1536, 41, True), (256, 1536, 42, False), (256, 1536, 43, True)]
BWD_GATE_UP = [(8960, 1536, 51, False), (8960, 1536, 52, False)]


@pytest.mark.parametrize("specs", [BWD_QKV, BWD_GATE_UP, BWD_QKV[:1]], ids=["qkv", "gate_up", "q"])
@pytest.mark.parametrize("n", [77, 1170, 2048])
def test_grouped_backward_matches_reference_and_sum_of_singles(cuda_lib, specs, n):
    """dX = sum_i dY_i W_i (+ 2 (dY_i B_i) A_i for adapters) in one K-concatenated GEMM."""
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate, _stream
    L = _lib.lib()
    in_f = 1536
    items = (_lib.LinearBwdItemC * len(specs))()
    keep = []
    ref = torch.zeros(n, in_f, dtype=torch.float64, device="cuda")
    for i, (out_f, _, seed, lora) in enumerate(specs):
        q, st = _weight((out_f, in_f), seed)
        qs = _qstate(st, q.device)
        dy = _x(n, out_f, seed + 5, std=0.01)
        ref += dy.double() @ _ref_weight(q, st)
        lc = a = b = dyb = None
        if lora:
            g = torch.Generator(device="cuda").manual_seed(seed + 7)
            a = ((torch.rand(16, in_f, generator=g, device="cuda") * 2 - 1) / in_f ** 0.5).half()
            b = (torch.randn(out_f, 16, generator=g, device="cuda") * 0.05).half()
            dyb = torch.empty(n, 16, dtype=torch.float16, device="cuda")
            lc = _lib.LoraC()
            lc.a, lc.b, lc.scale, lc.rank, lc.xa = a.data_ptr(), b.data_ptr(), 2.0, 16, None
            ref += 2.0 * (dy.double() @ b.double()) @ a.double()
        items[i].dy = dy.data_ptr()
        items[i].packed = q.data_ptr()
        items[i].qs = ctypes.pointer(qs)
        items[i].lora = None if lc is None else ctypes.pointer(lc)
        items[i].dyb = None if dyb is None else dyb.data_ptr()
        items[i].out_features = out_f
        # keep every buffer the C structs point to alive until the last launch
        keep.append(dict(q=q, st=st, qs=qs, dy=dy, lc=lc, dyb=dyb, a=a, b=b, out_f=out_f))
    outs = (ctypes.c_int64 * len(specs))(*[s[0] for s in specs])
    need = int(L.nf4b_linear_bwd_group_work_bytes(n, in_f, outs, len(specs)))
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    dx = torch.full((n, in_f), float("nan"), dtype=torch.float16, device="cuda")
    _lib.check(L.nf4b_linear_bwd_dx_group(items, len(specs), dx.data_ptr(), n, in_f, ws.data_ptr(),
                                          ws.numel(), _stream(dx.device)), "bwd group")
    torch.cuda.synchronize()
    assert not torch.isnan(dx).any()
    assert max_rel_err(dx, ref) <= GEMM_MAX_REL_ERR
    # the adapters' dY B went to dyb
    for k in keep:
        if k["lc"] is not None:
            assert max_rel_err(k["dyb"], k["dy"].double() @ k["b"].double()) <= GEMM_MAX_REL_ERR
    # same as the per-projection launches summed
    total = torch.zeros(n, in_f, dtype=torch.float64, device="cuda")
    for k in keep:
        one = torch.empty(n, in_f, dtype=torch.float16, device="cuda")
        dyb1 = torch.empty(n, 16, dtype=torch.float16, device="cuda") if k["lc"] is not None else None
        _lib.check(L.nf4b_linear_bwd_dx(k["dy"].data_ptr(), k["q"].data_ptr(), ctypes.byref(k["qs"]),
                                        None if k["lc"] is None else ctypes.byref(k["lc"]),
                                        None if dyb1 is None else dyb1.data_ptr(), one.data_ptr(), n, in_f,
                                        k["out_f"], _stream(dx.device)), "single bwd")
        total += one.double()
    torch.cuda.synchronize()
    assert max_rel_err(dx, total) <= 2e-3
    assert int(ws[:4096].count_nonzero()) == 0
    _check_flag()
