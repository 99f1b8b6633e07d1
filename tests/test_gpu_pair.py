"""GPU: the 2-CTA cluster tiling of the fused NF4 GEMMs (STEW_NF4_PAIR=1: 256-row x 512-token
tiles, two cta_group::2 MMAs over both CTAs of a pair per decoded weight stage) against the
single-CTA tiling (STEW_NF4_PAIR=0) and against the fp64 product of the oracle-dequantised
weights.

Unsplit, both tilings run the same K order per output, so their outputs must agree bit for
bit; when either plan splits K (few tiles) the fp32 partial sums are added in another order and
the two agree within 1e-3 of max |y|.  Both must be within the GEMM tolerance of the
reference (max |y - ref| / max |ref| <= 2e-3).  Covered: the Qwen2.5-1.5B shapes, weights
whose row count leaves the second CTA of the last pair partly or wholly outside the weight
(192, 384 rows), ragged token counts (a partial tile with or without tokens in its second
MMA, each MMA's tokens split between the two CTAs at n_h/2), bias,
LoRA, split-K plans (few tiles), grouped forward (q/k/v) and the K-concatenated grouped
backward."""
import ctypes

import pytest
import torch

from tests.helpers import GEMM_MAX_REL_ERR, max_rel_err
from tests.test_gpu_gemm import _check_flag, _ref_weight, _weight, _x

pytestmark = pytest.mark.gpu


@pytest.fixture
def pair_available(cuda_lib):
    from stew_b200 import _lib
    sms, slots = _lib.gemm_geometry()
    assert sms > 0
    if slots == 0:
        pytest.skip("device runs no 2-CTA clusters")
    return slots


def _run_fwd(monkeypatch, mode, x, q, st, out_f, bias=None, lora=None):
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate, _stream
    monkeypatch.setenv("STEW_NF4_PAIR", mode)
    L = _lib.lib()
    n, in_f = x.shape
    qs = _qstate(st, q.device)
    need = int(L.nf4b_linear_work_bytes(n, in_f, out_f, 0))
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    y = torch.full((n, out_f), float("nan"), dtype=torch.float16, device="cuda")
    _lib.check(L.nf4b_linear_fwd_ws(x.data_ptr(), q.data_ptr(), ctypes.byref(qs),
                                    None if bias is None else bias.data_ptr(),
                                    None if lora is None else ctypes.byref(lora), y.data_ptr(), n, in_f,
                                    out_f, ws.data_ptr(), ws.numel(), _stream(x.device)), "fwd")
    torch.cuda.synchronize()
    assert int(ws[:4096].count_nonzero()) == 0
    return y, need


def _run_bwd(monkeypatch, mode, dy, q, st, in_f, lora=None, dyb=None):
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate, _stream
    monkeypatch.setenv("STEW_NF4_PAIR", mode)
    L = _lib.lib()
    n, out_f = dy.shape
    qs = _qstate(st, q.device)
    need = int(L.nf4b_linear_work_bytes(n, in_f, out_f, 1))
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    dx = torch.full((n, in_f), float("nan"), dtype=torch.float16, device="cuda")
    _lib.check(L.nf4b_linear_bwd_dx_ws(dy.data_ptr(), q.data_ptr(), ctypes.byref(qs),
                                       None if lora is None else ctypes.byref(lora),
                                       None if dyb is None else dyb.data_ptr(), dx.data_ptr(), n, in_f,
                                       out_f, ws.data_ptr(), ws.numel(), _stream(dy.device)), "bwd")
    torch.cuda.synchronize()
    assert int(ws[:4096].count_nonzero()) == 0
    return dx, need


def _same(a, b, split):
    """Bit-equal when neither launch split K, else within 1e-3 of max |b|."""
    if split:
        assert max_rel_err(a, b.double()) <= 1e-3
    else:
        assert torch.equal(a, b)


SHAPES = [(1536, 1536), (256, 1536), (8960, 1536), (1536, 8960), (192, 256), (384, 512)]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{o}x{i}" for o, i in SHAPES])
@pytest.mark.parametrize("n", [1, 77, 300, 1170, 2048])
def test_pair_matches_single_and_reference(pair_available, monkeypatch, shape, n):
    out_f, in_f = shape
    q, st = _weight(shape, 900 + out_f % 97 + n)
    w = _ref_weight(q, st)
    x = _x(n, in_f, 5 + n)
    bias = _x(1, out_f, 7).reshape(out_f)
    y1, s1 = _run_fwd(monkeypatch, "1", x, q, st, out_f, bias=bias)
    y0, s0 = _run_fwd(monkeypatch, "0", x, q, st, out_f, bias=bias)
    assert not torch.isnan(y1).any()
    _same(y1, y0, s1 or s0)
    assert max_rel_err(y1, x.double() @ w.T + bias.double()) <= GEMM_MAX_REL_ERR
    dy = _x(n, out_f, 9 + n, std=0.01)
    d1, s1 = _run_bwd(monkeypatch, "1", dy, q, st, in_f)
    d0, s0 = _run_bwd(monkeypatch, "0", dy, q, st, in_f)
    assert not torch.isnan(d1).any()
    _same(d1, d0, s1 or s0)
    assert max_rel_err(d1, dy.double() @ w) <= GEMM_MAX_REL_ERR
    _check_flag()


@pytest.mark.parametrize("n", [77, 1170])
def test_pair_lora_forward_backward(pair_available, monkeypatch, n):
    """LoRA slab of a pair: each CTA stages its own weight rows and its half of the tokens."""
    from stew_b200 import _lib
    out_f, in_f = 1536, 1536
    q, st = _weight((out_f, in_f), 77)
    w = _ref_weight(q, st)
    g = torch.Generator(device="cuda").manual_seed(3)
    a = ((torch.rand(16, in_f, generator=g, device="cuda") * 2 - 1) / in_f ** 0.5).half()
    b = (torch.randn(out_f, 16, generator=g, device="cuda") * 0.05).half()
    x = _x(n, in_f, 11)
    outs, split = [], False
    for mode in ("1", "0"):
        xa = torch.empty(n, 16, dtype=torch.float16, device="cuda")
        lc = _lib.LoraC()
        lc.a, lc.b, lc.scale, lc.rank, lc.xa = a.data_ptr(), b.data_ptr(), 2.0, 16, xa.data_ptr()
        y, sp = _run_fwd(monkeypatch, mode, x, q, st, out_f, lora=lc)
        outs.append(y)
        split = split or bool(sp)
    ref = x.double() @ w.T + 2.0 * (x.double() @ a.double().T) @ b.double().T
    _same(outs[0], outs[1], split)
    assert max_rel_err(outs[0], ref) <= GEMM_MAX_REL_ERR
    dy = _x(n, out_f, 13, std=0.01)
    grads, split = [], False
    for mode in ("1", "0"):
        dyb = torch.empty(n, 16, dtype=torch.float16, device="cuda")
        lc = _lib.LoraC()
        lc.a, lc.b, lc.scale, lc.rank, lc.xa = a.data_ptr(), b.data_ptr(), 2.0, 16, None
        d, sp = _run_bwd(monkeypatch, mode, dy, q, st, in_f, lora=lc, dyb=dyb)
        grads.append(d)
        split = split or bool(sp)
    ref = dy.double() @ w + 2.0 * (dy.double() @ b.double()) @ a.double()
    _same(grads[0], grads[1], split)
    assert max_rel_err(grads[0], ref) <= GEMM_MAX_REL_ERR
    _check_flag()


def test_pair_grouped_forward_and_backward(pair_available, monkeypatch):
    """q/k/v in one grouped forward launch and their dX in one K-concatenated backward launch,
    pairs against single CTAs (each weight's rows rounded up to whole 256-row pair tiles)."""
    from tests.test_gpu_group import QKV, _items, _ref
    from stew_b200 import _lib
    from stew_b200.nf4 import _stream
    L = _lib.lib()
    n = 1170
    x = _x(n, 1536, 3)
    res, split = {}, False
    for mode in ("1", "0"):
        monkeypatch.setenv("STEW_NF4_PAIR", mode)
        items, keep = _items(QKV, n)
        outs = (ctypes.c_int64 * 3)(*[s_[0] for s_ in QKV])
        need = int(L.nf4b_linear_group_work_bytes(n, 1536, outs, 3))
        split = split or need > 0
        ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
        _lib.check(L.nf4b_linear_fwd_group(x.data_ptr(), n, 1536, items, 3, ws.data_ptr(), ws.numel(),
                                           _stream(x.device)), "group")
        torch.cuda.synchronize()
        res[mode] = [k["y"].clone() for k in keep]
        for k in keep:
            assert max_rel_err(k["y"], _ref(x, k)) <= GEMM_MAX_REL_ERR
        # backward over the same three weights
        bitems = (_lib.LinearBwdItemC * 3)()
        dys = []
        for i, k in enumerate(keep):
            dy = _x(n, QKV[i][0], 50 + i, std=0.01)
            dys.append(dy)
            bitems[i].dy = dy.data_ptr()
            bitems[i].packed = k["q"].data_ptr()
            bitems[i].qs = ctypes.pointer(k["qs"])
            bitems[i].lora = None
            bitems[i].dyb = None
            bitems[i].out_features = QKV[i][0]
        need = int(L.nf4b_linear_bwd_group_work_bytes(n, 1536, outs, 3))
        res[mode + "split"] = need > 0
        ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
        dx = torch.full((n, 1536), float("nan"), dtype=torch.float16, device="cuda")
        _lib.check(L.nf4b_linear_bwd_dx_group(bitems, 3, dx.data_ptr(), n, 1536, ws.data_ptr(), ws.numel(),
                                              _stream(dx.device)), "bwd group")
        torch.cuda.synchronize()
        ref = sum(dy.double() @ _ref_weight(k["q"], k["st"]) for dy, k in zip(dys, keep))
        assert max_rel_err(dx, ref) <= GEMM_MAX_REL_ERR
        res[mode + "dx"] = dx.clone()
    for a, b in zip(res["1"], res["0"]):
        _same(a, b, split)
    _same(res["1dx"], res["0dx"], res["1split"] or res["0split"])
    _check_flag()


@pytest.mark.parametrize("shape", [(1536, 1536), (256, 1536), (8960, 1536), (1536, 8960), (384, 512)],
                         ids=lambda s: f"{s[0]}x{s[1]}")
@pytest.mark.parametrize("n", [1, 77, 300, 1311])
def test_narrow_token_tiles_match_wide(cuda_lib, monkeypatch, shape, n):
    """128-token tiles (STEW_NF4_TILE_N=128, what the planner picks for launches with few
    tiles) against 256-token tiles: the same K order per output, so bit-equal unless either
    plan splits K; both within the GEMM tolerance of the reference."""
    out_f, in_f = shape
    q, st = _weight(shape, 700 + out_f % 89 + n)
    w = _ref_weight(q, st)
    x = _x(n, in_f, 15 + n)
    dy = _x(n, out_f, 19 + n, std=0.01)
    monkeypatch.setenv("STEW_NF4_TILE_N", "128")
    y1, s1 = _run_fwd(monkeypatch, "0", x, q, st, out_f)
    d1, t1 = _run_bwd(monkeypatch, "0", dy, q, st, in_f)
    monkeypatch.setenv("STEW_NF4_TILE_N", "256")
    y0, s0 = _run_fwd(monkeypatch, "0", x, q, st, out_f)
    d0, t0 = _run_bwd(monkeypatch, "0", dy, q, st, in_f)
    assert not torch.isnan(y1).any() and not torch.isnan(d1).any()
    _same(y1, y0, s1 or s0)
    _same(d1, d0, t1 or t0)
    assert max_rel_err(y1, x.double() @ w.T) <= GEMM_MAX_REL_ERR
    assert max_rel_err(d1, dy.double() @ w) <= GEMM_MAX_REL_ERR
    _check_flag()
