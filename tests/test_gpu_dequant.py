"""GPU parity of the standalone unpack (C ABI nf4b_dequant / nf4b_dequant_batched):
bit-exact against the reference kernel's golden vectors and the oracle, mirroring
solution/test_nf4_unpack.py (shapes incl. the (100, 64) edge, blocksize 64/128, nested on
and off, the (1, n) transposed view) and test_nf4_shim.py."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as O
from tests.helpers import case_inputs, golden, sha, to_oracle_state, to_torch_state

pytestmark = pytest.mark.gpu

QWEN_SHAPES = [(1536, 1536), (256, 1536), (8960, 1536), (1536, 8960), (100, 64)]


def _cases():
    meta, _ = golden()
    return meta["cases"]


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint16 if a.dtype == np.float16 else np.uint32)


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_dequant_matches_reference_golden(cuda_lib, case):
    from stew_b200 import dequantize_nf4
    _, arrays = golden()
    packed, st = case_inputs(case, arrays)
    q = torch.from_numpy(packed).cuda()
    out = dequantize_nf4(q, to_torch_state(st, "cuda"))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert got.shape == tuple(case["shape"])
    assert sha(got) == case["sha_out"], "differs from the reference kernel's output"
    if case["full"]:
        assert np.array_equal(_bits(got), _bits(arrays[f"{case['name']}/out"]))


@pytest.mark.parametrize("nested", [True, False])
@pytest.mark.parametrize("shape", QWEN_SHAPES)
@pytest.mark.parametrize("blocksize", [64, 128])
def test_dequant_bit_exact_qwen_shapes(cuda_lib, nested, shape, blocksize):
    """test_nf4_unpack.py:12-31 on the real layer shapes, but bit-exact (not 1e-4 mismatch)."""
    from stew_b200 import _supported, dequantize_nf4, quantize_4bit
    torch.manual_seed(0)
    W = torch.randn(shape, device="cuda", dtype=torch.float16) * 0.05
    q, st = quantize_4bit(W, blocksize=blocksize, compress_statistics=nested)
    assert _supported(q, st)
    out = dequantize_nf4(q, st)
    ref = O.dequant_nf4(q.cpu().numpy(), to_oracle_state(st, q))
    assert out.shape == W.shape and out.dtype == torch.float16
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(ref))


@pytest.mark.parametrize("blocksize", [32, 64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_contracted_scale_variant_against_oracle(cuda_lib, blocksize, dtype):
    """fma_scale (nf4b_qstate.nested == 2): the nested scale as one fused multiply-add, the form
    a GPU build of nf4.py:36-39 may take -- bit-exact against the oracle's restatement of it
    on the bulk-copy path (fp16; blocksize 32 in its two-table variant) and the general path
    (fp32).  The default stays the two-rounding form, and in fp16 the two differ in fewer than
    1e-4 of the outputs, the mismatch fraction solution/test_nf4_unpack.py:29-30 allows."""
    from stew_b200 import dequantize_nf4, quantize_4bit
    g = torch.Generator(device="cuda").manual_seed(11)
    W = (torch.randn(1536, 1536, generator=g, device="cuda") * 0.02).to(dtype)
    q, st = quantize_4bit(W, blocksize=blocksize, compress_statistics=True)
    ost = to_oracle_state(st, q)
    assert np.any(O.block_scales(ost) != O.block_scales(ost, fma=True))  # the variant matters here
    packed = q.cpu().numpy()
    fused = dequantize_nf4(q, st, fma_scale=True).cpu().numpy()
    plain = dequantize_nf4(q, st).cpu().numpy()
    assert np.array_equal(_bits(fused), _bits(O.dequant_nf4(packed, ost, fma=True)))
    assert np.array_equal(_bits(plain), _bits(O.dequant_nf4(packed, ost)))
    if dtype == torch.float16:  # fp32 outputs keep the scale's last bit
        assert np.mean(_bits(fused) != _bits(plain)) < 1e-4
    # plain (not nested) states have no offset to contract: the option changes nothing
    q2, st2 = quantize_4bit(W, blocksize=blocksize, compress_statistics=False)
    assert torch.equal(dequantize_nf4(q2, st2, fma_scale=True), dequantize_nf4(q2, st2))


def test_dequant_transposed_view(cuda_lib):
    """test_nf4_unpack.py:34-42: a (1, n) view of the packed tensor unpacks identically."""
    from stew_b200 import dequantize_nf4, quantize_4bit
    W = torch.randn(512, 256, device="cuda", dtype=torch.float16) * 0.05
    q, st = quantize_4bit(W, blocksize=64, compress_statistics=True)
    assert torch.equal(dequantize_nf4(q.t(), st), dequantize_nf4(q, st))


def test_dequant_unaligned_buffers(cuda_lib):
    """A packed view starting at an odd byte and an output not 16-byte aligned take the
    byte-wise path and still agree bit for bit."""
    from stew_b200 import _lib, dequantize_nf4, quantize_4bit
    W = torch.randn(64, 256, device="cuda", dtype=torch.float16) * 0.05
    q, st = quantize_4bit(W, blocksize=64, compress_statistics=True)
    ref = dequantize_nf4(q, st)
    buf = torch.zeros(q.numel() + 3, dtype=torch.uint8, device="cuda")
    buf[3:].copy_(q.reshape(-1))
    q_odd = buf[3:]
    out_buf = torch.zeros(ref.numel() + 1, dtype=torch.float16, device="cuda")
    out_view = out_buf[1:]
    from stew_b200.nf4 import _qstate, _stream
    qs = _qstate(st, q.device)
    _lib.check(_lib.lib().nf4b_dequant(q_odd.data_ptr(), ctypes.byref(qs), out_view.data_ptr(), 0,
                                       ref.numel(), _stream(q.device)), "nf4b_dequant")
    assert torch.equal(out_view.view(ref.shape), ref)


@pytest.mark.parametrize("nested", [True, False])
def test_dequant_fp32_output(cuda_lib, nested):
    from stew_b200 import dequantize_nf4, quantize_4bit
    W = torch.randn(256, 512, device="cuda", dtype=torch.float32) * 0.05
    q, st = quantize_4bit(W, blocksize=64, compress_statistics=nested)
    assert st.dtype == torch.float32
    out = dequantize_nf4(q, st)
    ref = O.dequant_nf4(q.cpu().numpy(), to_oracle_state(st, q))
    assert out.dtype == torch.float32
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(ref))


def test_dequant_empty(cuda_lib):
    from stew_b200 import QuantState, dequantize_nf4
    st = QuantState(torch.zeros(0, device="cuda"), (0, 64), None, 64, "nf4", torch.float16)
    out = dequantize_nf4(torch.zeros(0, dtype=torch.uint8, device="cuda"), st)
    assert out.shape == (0, 64)


def test_batched_sweep_equals_single_calls(cuda_lib):
    """One launch over many tensors == one nf4b_dequant per tensor (the per-step sweep)."""
    from stew_b200 import quantize_4bit
    from stew_b200.sweep import DequantSweep
    from stew_b200 import dequantize_nf4
    shapes = [(1536, 1536), (256, 1536), (256, 1536), (1536, 1536), (8960, 1536), (100, 64),
              (1536, 8960)]
    ws = []
    for i, s in enumerate(shapes):
        torch.manual_seed(i)
        ws.append(quantize_4bit(torch.randn(s, device="cuda", dtype=torch.float16) * 0.02,
                                blocksize=64, compress_statistics=(i % 3 != 2)))
    sweep = DequantSweep(ws)
    outs = sweep.run()
    for (q, st), o in zip(ws, outs):
        assert torch.equal(o, dequantize_nf4(q, st))


def test_plan_work_counter_is_reset_between_launches(cuda_lib):
    """Batched launches take their work from a counter held in the plan, which the last warp
    of each launch sets back to zero: the same plan launched again and again, and two plans
    launched in turn on one stream, give the single-call outputs every time."""
    from stew_b200 import _lib, dequantize_nf4, quantize_4bit
    from stew_b200.sweep import DequantSweep
    sets = []
    for base, shapes in ((0, [(1536, 1536), (256, 1536), (8960, 1536)]), (10, [(1536, 8960), (100, 64)])):
        ws = []
        for i, s in enumerate(shapes):
            g = torch.Generator(device="cuda").manual_seed(base + i)
            ws.append(quantize_4bit((torch.randn(s, generator=g, device="cuda") * 0.02).half(),
                                    blocksize=64, compress_statistics=(i % 2 == 0)))
        sets.append((ws, DequantSweep(ws), [dequantize_nf4(q, st) for q, st in ws]))
    for rep in range(3):
        for ws, sweep, want in sets:
            for o in sweep.outputs:  # a launch that did no work would leave the zeros
                o.zero_()
            outs = sweep.run()
            for o, w in zip(outs, want):
                assert torch.equal(o, w), rep
    torch.cuda.synchronize()
    assert _lib.dequant_error_flag(reset=True) == 0


def test_whole_model_sweep_properties(cuda_lib):
    """Full config-1 size (28 layers x 7 projections, 1.31 B weights): batched sweep ==
    single calls (digest of digests), and random blocks of every matrix bit-exact against
    the oracle."""
    from stew_b200.sweep import DequantSweep, qwen_model_weights
    ws = qwen_model_weights(layers=28, device="cuda", seed=0)
    sweep = DequantSweep(ws)
    outs = sweep.run()
    torch.cuda.synchronize()
    rng = np.random.default_rng(0)
    from stew_b200 import dequantize_nf4
    for idx in rng.choice(len(ws), size=12, replace=False):
        q, st = ws[idx]
        single = dequantize_nf4(q, st)
        assert torch.equal(single, outs[idx])
    for (q, st), o in zip(ws, outs):
        nb = o.numel() // st.blocksize
        blocks = rng.choice(nb, size=64, replace=False)
        qn = q.reshape(-1, st.blocksize // 2)[torch.from_numpy(blocks).cuda()].cpu().numpy()
        sub = to_oracle_state(st, q)
        scales = O.block_scales(sub)[blocks]
        code = O.nf4_codebook()
        hi = (code[(qn >> 4).astype(np.int64)] * scales[:, None]).astype(np.float32)
        lo = (code[(qn & 15).astype(np.int64)] * scales[:, None]).astype(np.float32)
        ref = np.stack([hi, lo], -1).reshape(len(blocks), -1).astype(np.float16)
        got = o.reshape(-1, st.blocksize)[torch.from_numpy(blocks).cuda()].cpu().numpy()
        assert np.array_equal(_bits(got), _bits(ref))


def test_batched_plan_mixed_blocksizes_against_oracle(cuda_lib):
    """A plan of jobs with every blocksize (32: two scales per 64-value chunk), nested and
    plain, ragged tails of fewer than 32 chunks, and an empty job between them: every output
    bit-exact against the oracle, and no bulk-copy wait ran out."""
    from stew_b200 import QuantState, _lib, quantize_4bit
    from stew_b200.sweep import DequantSweep
    shapes = [((64, 512), 32, True), ((100, 64), 64, False), ((33, 128), 128, True), ((7, 256), 256, False),
              ((256, 1536), 32, False), ((1536, 1536), 256, True), ((100, 64), 32, True)]
    ws = []
    for i, (shape, bs, nested) in enumerate(shapes):
        g = torch.Generator(device="cuda").manual_seed(40 + i)
        w = (torch.randn(shape, generator=g, device="cuda") * 0.02).half()
        ws.append(quantize_4bit(w, blocksize=bs, compress_statistics=nested))
    empty = (torch.zeros(0, dtype=torch.uint8, device="cuda"),
             QuantState(torch.zeros(0, device="cuda"), (0, 64), None, 64, "nf4", torch.float16))
    ws.insert(3, empty)
    sweep = DequantSweep(ws)
    outs = sweep.run()
    torch.cuda.synchronize()
    assert _lib.dequant_error_flag(reset=True) == 0
    for (q, st), o in zip(ws, outs):
        if o.numel() == 0:
            continue
        ref = O.dequant_nf4(q.cpu().numpy(), to_oracle_state(st, q))
        assert np.array_equal(_bits(o.cpu().numpy()), _bits(ref)), (tuple(st.shape), st.blocksize)
