"""Shared test helpers: golden fixtures, oracle <-> torch conversions, tolerances."""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import torch

from oracle import nf4_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN_DIR = os.path.join(HERE, "golden")

# GEMM tolerance: max |y - ref| / max |ref| over the output, ref = fp64 product of the
# reference-dequantised weights (fp32-accumulated fp16 GEMM + one fp16 output rounding).
GEMM_MAX_REL_ERR = 2e-3
# Elementwise form of the same bound: max |y - ref| / |ref| over every entry whose |ref| is
# at least ELEM_FLOOR of max |ref| (below it, fp32 accumulation error of a near-cancelling
# sum dominates the entry's own size), so one bad tile of small values cannot hide behind
# the output's largest entry.
ELEM_REL_ERR = 2e-3
ELEM_FLOOR = 0.05


def golden():
    with open(os.path.join(GOLDEN_DIR, "nf4_golden.json")) as f:
        meta = json.load(f)
    arrays = np.load(os.path.join(GOLDEN_DIR, "nf4_golden.npz"))
    return meta, arrays


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def case_inputs(case, arrays):
    """(packed, QState) of a golden case: stored arrays, or regenerated from the seed and
    checked against the stored input digests."""
    name = case["name"]
    packed, st = O.golden_inputs(tuple(case["shape"]), case["blocksize"], case["nested"],
                                 case["dtype"], case["kind"], case["seed"])
    if case["full"]:
        packed = arrays[f"{name}/packed"]
        st.absmax = arrays[f"{name}/absmax"]
        if case["nested"]:
            st.state2.absmax = arrays[f"{name}/absmax2"]
    assert sha(packed) == case["sha_packed"], "golden input drifted (packed)"
    assert sha(np.asarray(st.absmax)) == case["sha_absmax"], "golden input drifted (absmax)"
    return packed, st


def to_torch_state(st: O.QState, device):
    """stew_b200.QuantState of an oracle QState on `device`."""
    from stew_b200.quant_state import QuantState
    dtype = torch.float16 if st.dtype == "float16" else torch.float32
    code = torch.from_numpy(O.nf4_codebook()).to(device)
    if not st.nested:
        return QuantState(torch.from_numpy(np.asarray(st.absmax, np.float32)).to(device), st.shape,
                          code, st.blocksize, "nf4", dtype)
    s2 = QuantState(torch.from_numpy(st.state2.absmax).to(device), st.state2.absmax.shape,
                    torch.from_numpy(st.state2.code).to(device), st.state2.blocksize,
                    quant_type="dynamic", dtype=torch.float32)
    return QuantState(torch.from_numpy(np.asarray(st.absmax, np.uint8)).to(device), st.shape, code,
                      st.blocksize, "nf4", dtype,
                      torch.tensor(st.offset, dtype=torch.float32, device=device), s2)


def to_oracle_state(st, packed: torch.Tensor):
    """Oracle QState (numpy) of a stew_b200 / bitsandbytes-style QuantState."""
    dtype = "float16" if st.dtype == torch.float16 else "float32"
    if not st.nested:
        return O.QState(absmax=st.absmax.float().cpu().numpy(), shape=tuple(st.shape),
                        code=O.nf4_codebook(), blocksize=st.blocksize, dtype=dtype, nested=False)
    return O.QState(absmax=st.absmax.cpu().numpy(), shape=tuple(st.shape), code=O.nf4_codebook(),
                    blocksize=st.blocksize, dtype=dtype, nested=True,
                    offset=float(st.offset.float().cpu()),
                    state2=O.State2(absmax=st.state2.absmax.float().cpu().numpy(),
                                    code=st.state2.code.float().cpu().numpy(),
                                    blocksize=st.state2.blocksize))


def seeded_weight(shape, seed, device="cpu"):
    """fp16 weight drawn N(0, 0.02) from a seed (the whole-model sweep's weight distribution)."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * 0.02).to(torch.float16).to(device)


def max_rel_err(y: torch.Tensor, ref: torch.Tensor) -> float:
    ref = ref.detach().double()
    return float((y.detach().double() - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def elem_rel_err(y: torch.Tensor, ref: torch.Tensor, floor: float = ELEM_FLOOR) -> float:
    """max |y - ref| / |ref| over the entries with |ref| >= floor * max |ref|."""
    ref = ref.double()
    a = ref.abs()
    keep = a >= floor * a.max()
    if not bool(keep.any()):
        return 0.0
    return float(((y.double() - ref).abs()[keep] / a[keep]).max())


def assert_gemm_close(y: torch.Tensor, ref: torch.Tensor, what: str = "") -> None:
    """Both GEMM bounds: max-normalised and elementwise above the floor."""
    m, e = max_rel_err(y, ref), elem_rel_err(y, ref)
    assert m <= GEMM_MAX_REL_ERR, f"{what} max-normalised error {m:.3e}"
    assert e <= ELEM_REL_ERR, f"{what} elementwise error {e:.3e} (|ref| >= {ELEM_FLOOR} max)"
