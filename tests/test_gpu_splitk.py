"""GPU: split-K launches of the fused NF4 GEMMs (nf4b_linear_fwd_ws / nf4b_linear_bwd_dx_ws).

Shapes with fewer output tiles than SMs split each tile's K reduction over several CTAs
and add the fp32 partials in the last CTA of the tile.  The result must match the fp64
product of the oracle-dequantised weight within the GEMM tolerance (max |y - ref| /
max |ref| <= 2e-3), match the unsplit launch up to fp32 summation order (<= 1e-3 of the
same measure), include the LoRA term and the bias exactly once, and leave the
workspace counters zero for the next call.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as O
from tests.helpers import GEMM_MAX_REL_ERR, max_rel_err, to_oracle_state

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _wide_tiles(monkeypatch):
    """The split-K plans under test are those of 256-token tiles (the planner would give these
    shapes 128-token tiles without a split; that tiling is covered in test_gpu_pair.py)."""
    monkeypatch.setenv("STEW_NF4_TILE_N", "256")

SPLIT_VS_UNSPLIT = 1e-3


def _weight(shape, seed):
    from stew_b200 import quantize_4bit
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(shape, generator=g, device="cuda") * 0.02).to(torch.float16)
    return quantize_4bit(w, blocksize=64, compress_statistics=True)


def _ref_weight(q, st):
    w = O.dequant_nf4(q.cpu().numpy(), to_oracle_state(st, q))
    return torch.from_numpy(w.astype(np.float64)).cuda()


def _rand(n, k, seed, std=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(n, k, generator=g, device="cuda") * std).to(torch.float16)


def _flag_clear():
    from stew_b200 import _lib
    assert _lib.gemm_error_flag(reset=True) == 0


def _ws(nbytes):
    return torch.zeros(max(nbytes, 256), dtype=torch.uint8, device="cuda")


def _counters(ws, m_rows=None, n=None):
    """The workspace's leading counter region (per-tile arrivals and finished partials, 4 KB,
    then the launch's exit count; the same for every shape)."""
    return ws[:4096 + 4]


def _fwd(L, x, q, qs, bias, lc, y, n, in_f, out_f, ws):
    from stew_b200.nf4 import _stream
    from stew_b200 import _lib
    _lib.check(L.nf4b_linear_fwd_ws(x.data_ptr(), q.data_ptr(), ctypes.byref(qs),
                                    None if bias is None else bias.data_ptr(),
                                    None if lc is None else ctypes.byref(lc), y.data_ptr(), n, in_f,
                                    out_f, None if ws is None else ws.data_ptr(),
                                    0 if ws is None else ws.numel(), _stream(x.device)), "fwd_ws")


def _bwd(L, dy, q, qs, lc, dyb, dx, n, in_f, out_f, ws):
    from stew_b200.nf4 import _stream
    from stew_b200 import _lib
    _lib.check(L.nf4b_linear_bwd_dx_ws(dy.data_ptr(), q.data_ptr(), ctypes.byref(qs),
                                       None if lc is None else ctypes.byref(lc),
                                       None if dyb is None else dyb.data_ptr(), dx.data_ptr(), n, in_f,
                                       out_f, None if ws is None else ws.data_ptr(),
                                       0 if ws is None else ws.numel(), _stream(dy.device)), "bwd_ws")


# (out, in, n): k/v at 1170 and 8192 tokens (10 / 64 tiles, 2 ranges), q/o at 1170 (60 tiles,
# 2 ranges), down at 1170 and 2048 (60 / 96 tiles, 2 / 3 ranges), a ragged long-K shape
# (3 tiles, 4 ranges)
CASES = [(256, 1536, 1170), (256, 1536, 8192), (1536, 1536, 1170), (1536, 8960, 1170),
         (1536, 8960, 2048), (384, 4096, 77)]


@pytest.mark.parametrize("out_f,in_f,n", CASES)
def test_split_forward_matches_reference_and_unsplit(cuda_lib, out_f, in_f, n):
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate
    L = _lib.lib()
    need = int(L.nf4b_linear_work_bytes(n, in_f, out_f, 0))
    assert need > 0, "this shape is expected to split"
    q, st = _weight((out_f, in_f), out_f + in_f)
    qs = _qstate(st, q.device)
    x = _rand(n, in_f, 1)
    bias = _rand(1, out_f, 2).reshape(out_f)
    ws = _ws(need)
    y_split = torch.full((n, out_f), float("nan"), dtype=torch.float16, device="cuda")
    y_plain = torch.empty_like(y_split)
    _fwd(L, x, q, qs, bias, None, y_split, n, in_f, out_f, ws)
    _fwd(L, x, q, qs, bias, None, y_plain, n, in_f, out_f, None)
    torch.cuda.synchronize()
    ref = x.double() @ _ref_weight(q, st).T + bias.double()
    assert not torch.isnan(y_split).any()
    assert max_rel_err(y_split, ref) <= GEMM_MAX_REL_ERR
    assert max_rel_err(y_split, y_plain.double()) <= SPLIT_VS_UNSPLIT
    assert int(_counters(ws, out_f, n).count_nonzero()) == 0, "split-K counters must be left zero"
    _flag_clear()


@pytest.mark.parametrize("out_f,in_f,n", [(1536, 256, 1170), (8960, 1536, 1170), (8960, 1536, 2048),
                                          (4096, 384, 77)])
def test_split_backward_matches_reference_and_unsplit(cuda_lib, out_f, in_f, n):
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate
    L = _lib.lib()
    need = int(L.nf4b_linear_work_bytes(n, in_f, out_f, 1))
    assert need > 0, "this shape is expected to split"
    q, st = _weight((out_f, in_f), 7 * out_f + in_f)
    qs = _qstate(st, q.device)
    dy = _rand(n, out_f, 3, std=0.01)
    ws = _ws(need)
    dx_split = torch.full((n, in_f), float("nan"), dtype=torch.float16, device="cuda")
    dx_plain = torch.empty_like(dx_split)
    _bwd(L, dy, q, qs, None, None, dx_split, n, in_f, out_f, ws)
    _bwd(L, dy, q, qs, None, None, dx_plain, n, in_f, out_f, None)
    torch.cuda.synchronize()
    ref = dy.double() @ _ref_weight(q, st)
    assert not torch.isnan(dx_split).any()
    assert max_rel_err(dx_split, ref) <= GEMM_MAX_REL_ERR
    assert max_rel_err(dx_split, dx_plain.double()) <= SPLIT_VS_UNSPLIT
    assert int(_counters(ws, in_f, n).count_nonzero()) == 0
    _flag_clear()


def test_split_lora_term_added_once(cuda_lib):
    """q projection (1536 x 1536) at 1170 tokens with the rank-16 adapter: forward and
    backward through split launches against fp64."""
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate
    L = _lib.lib()
    out_f, in_f, n = 1536, 1536, 1170
    assert int(L.nf4b_linear_work_bytes(n, in_f, out_f, 0)) > 0
    assert int(L.nf4b_linear_work_bytes(n, in_f, out_f, 1)) > 0
    q, st = _weight((out_f, in_f), 5)
    qs = _qstate(st, q.device)
    W = _ref_weight(q, st)
    g = torch.Generator(device="cuda").manual_seed(9)
    a = ((torch.rand(16, in_f, generator=g, device="cuda") * 2 - 1) / in_f ** 0.5).half()
    b = (torch.randn(out_f, 16, generator=g, device="cuda") * 0.05).half()
    x = _rand(n, in_f, 4)
    dy = _rand(n, out_f, 5, std=0.01)
    xa = torch.empty(n, 16, dtype=torch.float16, device="cuda")
    dyb = torch.empty(n, 16, dtype=torch.float16, device="cuda")
    lc = _lib.LoraC()
    lc.a, lc.b, lc.scale, lc.rank, lc.xa = a.data_ptr(), b.data_ptr(), 2.0, 16, xa.data_ptr()
    ws = _ws(max(int(L.nf4b_linear_work_bytes(n, in_f, out_f, d)) for d in (0, 1)))
    y = torch.empty(n, out_f, dtype=torch.float16, device="cuda")
    dx = torch.empty(n, in_f, dtype=torch.float16, device="cuda")
    _fwd(L, x, q, qs, None, lc, y, n, in_f, out_f, ws)
    _bwd(L, dy, q, qs, lc, dyb, dx, n, in_f, out_f, ws)
    torch.cuda.synchronize()
    xd, dyd, ad, bd = x.double(), dy.double(), a.double(), b.double()
    ref_y = xd @ W.T + 2.0 * (xa.double() @ bd.T)
    ref_dx = dyd @ W + 2.0 * (dyb.double() @ ad)
    assert max_rel_err(y, ref_y) <= GEMM_MAX_REL_ERR
    assert max_rel_err(dx, ref_dx) <= GEMM_MAX_REL_ERR
    # the adapter's own size: without it the error would be of order |lora| / |y|
    lora_y = 2.0 * (xa.double() @ bd.T)
    assert lora_y.abs().max() > 20 * GEMM_MAX_REL_ERR * ref_y.abs().max()
    _flag_clear()


def test_workspace_reuse_and_argument_checks(cuda_lib):
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate
    L = _lib.lib()
    out_f, in_f, n = 256, 1536, 1170
    need = int(L.nf4b_linear_work_bytes(n, in_f, out_f, 0))
    assert need > 0
    assert int(L.nf4b_linear_work_bytes(8192, 1536, 8960, 0)) == 0  # 2240 tiles: no split
    q, st = _weight((out_f, in_f), 31)
    qs = _qstate(st, q.device)
    W = _ref_weight(q, st)
    ws = _ws(need)
    y = torch.empty(n, out_f, dtype=torch.float16, device="cuda")
    for seed in range(3):  # back-to-back calls on one workspace
        x = _rand(n, in_f, 40 + seed)
        _fwd(L, x, q, qs, None, None, y, n, in_f, out_f, ws)
        torch.cuda.synchronize()
        assert max_rel_err(y, x.double() @ W.T) <= GEMM_MAX_REL_ERR
    from stew_b200.nf4 import _stream
    small = L.nf4b_linear_fwd_ws(x.data_ptr(), q.data_ptr(), ctypes.byref(qs), None, None, y.data_ptr(),
                                 n, in_f, out_f, ws.data_ptr(), need - 1, _stream(x.device))
    assert small == _lib.NF4B_ERR_INVALID_ARG
    odd = L.nf4b_linear_fwd_ws(x.data_ptr(), q.data_ptr(), ctypes.byref(qs), None, None, y.data_ptr(),
                               n, in_f, out_f, ws.data_ptr() + 16, need, _stream(x.device))
    assert odd == _lib.NF4B_ERR_ALIGNMENT
    _flag_clear()


def test_one_workspace_across_shapes(cuda_lib):
    """A workspace reused by launches with different tile counts and split factors
    (k: 10 tiles x 2, q: 60 tiles x 2, ragged: 3 tiles x 4, in an interleaved order)."""
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate
    L = _lib.lib()
    shapes = [(256, 1536, 1170), (1536, 1536, 1170), (384, 4096, 77)]
    ws = _ws(max(int(L.nf4b_linear_work_bytes(n, i, o, 0)) for o, i, n in shapes))
    prep = []
    for o, i, n in shapes:
        q, st = _weight((o, i), 3 * o + i)
        # st owns the device tables that qs points to: keep it alive
        prep.append((o, i, n, q, st, _qstate(st, q.device), _ref_weight(q, st)))
    for rep in range(2):
        for o, i, n, q, _st, qs, W in prep[::1 if rep == 0 else -1]:
            x = _rand(n, i, 50 + rep)
            y = torch.empty(n, o, dtype=torch.float16, device="cuda")
            _fwd(L, x, q, qs, None, None, y, n, i, o, ws)
            torch.cuda.synchronize()
            assert max_rel_err(y, x.double() @ W.T) <= GEMM_MAX_REL_ERR, (o, i, n)
            assert int(_counters(ws).count_nonzero()) == 0
    _flag_clear()


def test_split_result_is_deterministic(cuda_lib):
    """The last K range of a tile sums all ranges in range order, whichever finishes last:
    repeated split launches are bit-identical."""
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate
    L = _lib.lib()
    out_f, in_f, n = 1536, 8960, 1170  # down projection: 60 tiles x 2 ranges
    q, st = _weight((out_f, in_f), 77)
    qs = _qstate(st, q.device)
    ws = _ws(int(L.nf4b_linear_work_bytes(n, in_f, out_f, 0)))
    x = _rand(n, in_f, 78)
    ys = []
    for _ in range(5):
        y = torch.empty(n, out_f, dtype=torch.float16, device="cuda")
        _fwd(L, x, q, qs, None, None, y, n, in_f, out_f, ws)
        ys.append(y)
    torch.cuda.synchronize()
    assert all(torch.equal(ys[0], y) for y in ys[1:])
    _flag_clear()



@pytest.mark.parametrize("pair", ["0", "1"])
def test_counters_recover_after_a_range_gives_up(cuda_lib, monkeypatch, pair):
    """A K range that gives up before taking its ticket (a pipeline wait that ran out) leaves
    its tile's counts behind; the last CTA to leave the launch clears them, so the next call on
    the same workspace is correct.  The give-up is injected on the host (a one-shot hook makes
    work unit 0 skip its ticket): no wait actually runs out and nothing faults."""
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate
    monkeypatch.setenv("STEW_NF4_PAIR", pair)
    L = _lib.lib()
    out_f, in_f, n = 1536, 8960, 1170  # down projection: split on single CTAs and on pairs
    need = int(L.nf4b_linear_work_bytes(n, in_f, out_f, 0))
    assert need > 0
    q, st = _weight((out_f, in_f), 91)
    qs = _qstate(st, q.device)
    ws = _ws(need)
    x = _rand(n, in_f, 92)
    _flag_clear()
    assert L.nf4b_test_drop_split_ticket(-1) == _lib.NF4B_ERR_INVALID_ARG
    assert L.nf4b_test_drop_split_ticket(0) == _lib.NF4B_OK
    y_bad = torch.zeros(n, out_f, dtype=torch.float16, device="cuda")
    _fwd(L, x, q, qs, None, None, y_bad, n, in_f, out_f, ws)
    torch.cuda.synchronize()
    assert _lib.gemm_error_flag(reset=True) == 4, "the dropped ticket is recorded"
    assert int(_counters(ws).count_nonzero()) == 0, "counters left behind by the dropped range"
    ref = x.double() @ _ref_weight(q, st).T
    ys = []
    for _ in range(2):  # the hook was one-shot: both calls are whole and identical
        y = torch.full((n, out_f), float("nan"), dtype=torch.float16, device="cuda")
        _fwd(L, x, q, qs, None, None, y, n, in_f, out_f, ws)
        ys.append(y)
    torch.cuda.synchronize()
    assert not torch.isnan(ys[0]).any()
    assert max_rel_err(ys[0], ref) <= GEMM_MAX_REL_ERR
    assert torch.equal(ys[0], ys[1])
    assert int(_counters(ws).count_nonzero()) == 0
    _flag_clear()


# (direction, out, in, n, STEW_NF4_PAIR): the last K range of a tile reads the other ranges'
# partials either through bulk copies into its idle ring (the default) or with per-thread L2
# loads (STEW_NF4_SPLIT_STAGED=0).  Both add the ranges in range order, so the outputs must be
# bit-identical.  down at 1,170 tokens (60 tiles x 2 ranges; as pairs 512-token partials, eight
# 64-token rounds), a 3-tile shape with 4 ranges (three staged partials), gate backward at
# 1,170 tokens on single CTAs and on pairs.
STAGED_CASES = [("fwd", 1536, 8960, 1170, "0"), ("fwd", 384, 4096, 77, "0"), ("fwd", 1536, 8960, 1170, "1"),
                ("bwd", 8960, 1536, 1170, "0"), ("bwd", 8960, 1536, 1170, "1")]


@pytest.mark.parametrize("kind,out_f,in_f,n,pair", STAGED_CASES)
def test_staged_reduction_bit_identical_to_l2_loads(cuda_lib, monkeypatch, kind, out_f, in_f, n, pair):
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate
    monkeypatch.setenv("STEW_NF4_PAIR", pair)
    L = _lib.lib()
    bwd = kind == "bwd"
    need = int(L.nf4b_linear_work_bytes(n, in_f, out_f, 1 if bwd else 0))
    assert need > 0, "this shape is expected to split"
    q, st = _weight((out_f, in_f), 3 * out_f + in_f)
    qs = _qstate(st, q.device)
    a = _rand(n, out_f if bwd else in_f, 5, std=0.01 if bwd else 1.0)
    ws = _ws(need)
    outs = {}
    for staged in ("1", "0"):
        monkeypatch.setenv("STEW_NF4_SPLIT_STAGED", staged)
        o = torch.full((n, in_f if bwd else out_f), float("nan"), dtype=torch.float16, device="cuda")
        if bwd:
            _bwd(L, a, q, qs, None, None, o, n, in_f, out_f, ws)
        else:
            _fwd(L, a, q, qs, None, None, o, n, in_f, out_f, ws)
        outs[staged] = o
    torch.cuda.synchronize()
    W = _ref_weight(q, st)
    ref = a.double() @ W if bwd else a.double() @ W.T
    assert not torch.isnan(outs["1"]).any()
    assert max_rel_err(outs["1"], ref) <= GEMM_MAX_REL_ERR
    assert torch.equal(outs["1"], outs["0"])
    assert int(_counters(ws).count_nonzero()) == 0
    _flag_clear()


def test_staged_reduction_grouped_gate_up_backward(cuda_lib, monkeypatch):
    """The step's gate/up dX (one K-concatenated launch, split pairs at 1,170 tokens): staged and
    L2-load reductions bit-identical, and both within the GEMM bound of the fp64 product."""
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate, _stream
    monkeypatch.delenv("STEW_NF4_TILE_N")  # the planner's own choice, as in the step
    L = _lib.lib()
    n, in_f = 1170, 1536
    specs = [(8960, 61), (8960, 62)]
    items = (_lib.LinearBwdItemC * len(specs))()
    keep = []
    ref = torch.zeros(n, in_f, dtype=torch.float64, device="cuda")
    for i, (out_f, seed) in enumerate(specs):
        q, st = _weight((out_f, in_f), seed)
        qs = _qstate(st, q.device)
        dy = _rand(n, out_f, seed + 5, std=0.01)
        ref += dy.double() @ _ref_weight(q, st)
        items[i].dy = dy.data_ptr()
        items[i].packed = q.data_ptr()
        items[i].qs = ctypes.pointer(qs)
        items[i].lora = None
        items[i].dyb = None
        items[i].out_features = out_f
        keep.append((q, st, qs, dy))
    outs_c = (ctypes.c_int64 * len(specs))(*[s[0] for s in specs])
    need = int(L.nf4b_linear_bwd_group_work_bytes(n, in_f, outs_c, len(specs)))
    assert need > 0, "expected a split plan"
    ws = _ws(need)
    outs = {}
    for staged in ("1", "0"):
        monkeypatch.setenv("STEW_NF4_SPLIT_STAGED", staged)
        dx = torch.full((n, in_f), float("nan"), dtype=torch.float16, device="cuda")
        _lib.check(L.nf4b_linear_bwd_dx_group(items, len(specs), dx.data_ptr(), n, in_f, ws.data_ptr(),
                                              ws.numel(), _stream(dx.device)), "bwd group")
        outs[staged] = dx
    torch.cuda.synchronize()
    assert not torch.isnan(outs["1"]).any()
    assert max_rel_err(outs["1"], ref) <= GEMM_MAX_REL_ERR
    assert torch.equal(outs["1"], outs["0"])
    assert int(_counters(ws).count_nonzero()) == 0
    _flag_clear()


@pytest.mark.parametrize("splits,pair", [("1", "0"), ("3", "0"), ("4", "0"), ("2", "1"), ("3", "1")])
def test_forced_split_count(cuda_lib, monkeypatch, splits, pair):
    """STEW_NF4_SPLITS sets the K ranges of the chosen tiling (down projection at 1,170 tokens,
    140 stages): the workspace follows it, the output stays within the GEMM bound of the fp64
    product and within the split-vs-unsplit bound of the unsplit launch, counters left zero."""
    from stew_b200 import _lib
    from stew_b200.nf4 import _qstate
    monkeypatch.setenv("STEW_NF4_PAIR", pair)
    L = _lib.lib()
    out_f, in_f, n = 1536, 8960, 1170
    q, st = _weight((out_f, in_f), 101)
    qs = _qstate(st, q.device)
    x = _rand(n, in_f, 102)
    monkeypatch.setenv("STEW_NF4_SPLITS", "1")
    assert int(L.nf4b_linear_work_bytes(n, in_f, out_f, 0)) == 0, "one range: no workspace"
    y1 = torch.empty(n, out_f, dtype=torch.float16, device="cuda")
    _fwd(L, x, q, qs, None, None, y1, n, in_f, out_f, None)
    monkeypatch.setenv("STEW_NF4_SPLITS", splits)
    need = int(L.nf4b_linear_work_bytes(n, in_f, out_f, 0))
    assert (need > 0) == (splits != "1")
    ws = _ws(need)
    y = torch.full((n, out_f), float("nan"), dtype=torch.float16, device="cuda")
    _fwd(L, x, q, qs, None, None, y, n, in_f, out_f, ws if need > 0 else None)
    torch.cuda.synchronize()
    assert not torch.isnan(y).any()
    assert max_rel_err(y, x.double() @ _ref_weight(q, st).T) <= GEMM_MAX_REL_ERR
    assert max_rel_err(y, y1.double()) <= SPLIT_VS_UNSPLIT
    assert int(_counters(ws).count_nonzero()) == 0
    _flag_clear()
