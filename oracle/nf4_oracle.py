"""CPU oracle for the NF4 hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker: only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg import it.  The product (stew_b200) never calls it, and nothing
here is ever timed as the product.

What it restates (reference = evilandangry/stew):

* ``dequant_nf4`` -- the double-quantized NF4 unpack of solution/nf4.py:30-50
  (`_nf4_unpack`) as driven by `dequantize_nf4` (solution/nf4.py:73-92):
    scale[r] = code2[absmax8[r]] * absmax2[r // bs2] + offset   (nested, nf4.py:36-39)
    scale[r] = absmax[r]                                         (plain,  nf4.py:41)
    out[r*bs + 2j]   = code[b >> 4] * scale[r]                   (nf4.py:45)
    out[r*bs + 2j+1] = code[b & 15] * scale[r]                   (nf4.py:46)
  all in fp32 with one rounding per operation (multiply, then add -- no FMA),
  then ONE rounding to the output dtype (nf4.py:49-50).
  ``fma=True`` gives the contracted variant -- the nested scale as one fused
  multiply-add, rounded once (``fma_f32``) -- which a GPU compiler may emit for
  nf4.py:36-39; the reference's own test allows for it with a mismatch
  fraction below 1e-4 (solution/test_nf4_unpack.py:29-30).
* ``linear_fwd_ref`` / ``linear_bwd_ref`` -- the patched MatMul4Bit forward
  (nf4.py:142-159: unpack, then F.linear) and bitsandbytes' unchanged
  MatMul4Bit backward (grad_A = dY . W), evaluated in fp32/fp64 on the
  reference-dequantised weights, plus peft's LoRA term y += (x A^T) B^T * s.

Codebooks and the quantizer live in bitsandbytes 0.50.2 (a pinned third-party
dependency of the reference, README.md:156-158, absent from this environment).
They are restated from their published descriptions:

* NF4 table: the 16 values printed in the QLoRA paper (Dettmers et al. 2023,
  Appendix E).  ``nf4_construction`` rebuilds them from the paper's recipe
  (normal quantiles, asymmetric 8 positive / 7 negative + exact zero) to
  within 2e-7 -- the paper's table is the canonical one.
* Second-level "dynamic" 8-bit map: the signed dynamic tree quantization of
  Dettmers et al. 2022 ("8-bit Optimizers via Block-wise Quantization") --
  one sign, a run of exponent-marker bits selecting a decade 10^-6..10^0,
  linear fraction inside the decade.  Restated in ``dynamic_map_signed``.
* Quantizer: blockwise absmax scaling and nearest-code rounding (QLoRA §3).
  Its bit-compatibility with bitsandbytes' own quantizer is NOT pinned here
  (no bitsandbytes in this environment); the decode arithmetic above is
  pinned against the reference kernel itself, see tests/golden/.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

# QLoRA paper, Appendix E: the NF4 data type.
NF4_PUBLISHED = np.array([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0], dtype=np.float32)


def nf4_codebook() -> np.ndarray:
    """The 16-entry NF4 table as fp32 (what `_code()` returns, nf4.py:53-58)."""
    return NF4_PUBLISHED.copy()


def nf4_construction() -> np.ndarray:
    """Rebuild NF4 from the paper's recipe: quantiles of N(0,1) at probabilities
    evenly spaced between 1-delta and 1/2, delta = (1/30 + 1/32)/2, with 8
    positive and 7 negative levels plus an exact zero, normalised to [-1, 1]."""
    from scipy.stats import norm
    delta = 0.5 * (1.0 / 30 + 1.0 / 32)
    pos = norm.ppf(np.linspace(1.0 - delta, 0.5, 9)[:-1])
    neg = -norm.ppf(np.linspace(1.0 - delta, 0.5, 8)[:-1])
    v = np.sort(np.concatenate([pos, [0.0], neg]))
    return (v / v.max()).astype(np.float32)


def dynamic_map_signed() -> np.ndarray:
    """Signed dynamic tree map, 256 fp32 entries, sorted ascending.

    Decade e (e = 0..6) covers magnitudes 10^(e-6) * [0.1, 1]; it is split into
    2^e equal intervals whose midpoints are the codes, mirrored for the sign.
    With 0 and +1.0 added that is 2*127 + 2 = 256 codes.  Evaluated in fp32 torch
    arithmetic (linspace, midpoint, decade product), as the dependency builds it."""
    import torch
    vals = []
    for e in range(7):
        edges = torch.linspace(0.1, 1.0, 2 ** e + 1, dtype=torch.float32)
        mids = (edges[:-1] + edges[1:]) / 2.0
        dec = torch.tensor(10.0 ** (e - 6), dtype=torch.float32)
        vals.extend((dec * mids).tolist())
        vals.extend((-dec * mids).tolist())
    vals.append(0.0)
    vals.append(1.0)
    assert len(vals) == 256
    return np.sort(np.array(vals, dtype=np.float32))


@dataclass
class State2:
    """Second-level quantization state (bitsandbytes QuantState.state2)."""
    absmax: np.ndarray          # fp32 [n_blocks2]
    code: np.ndarray            # fp32 [256]
    blocksize: int = 256


@dataclass
class QState:
    """The QuantState fields the reference reads (nf4.py:61-70, :80-91)."""
    absmax: np.ndarray          # uint8 [n_blocks] if nested, else fp32 [n_blocks]
    shape: tuple
    code: np.ndarray            # fp32 [16] (the reference ignores it and uses _code())
    blocksize: int
    dtype: str = "float16"      # "float16" or "float32"
    quant_type: str = "nf4"
    nested: bool = True
    offset: float = 0.0
    state2: State2 | None = None
    extra: dict = field(default_factory=dict)


def _nearest(values: np.ndarray, table: np.ndarray) -> np.ndarray:
    """Index of the nearest table entry (table sorted ascending); ties go to the
    lower index.  Evaluated on midpoints, the way a decision tree would."""
    mids = (table[:-1].astype(np.float64) + table[1:].astype(np.float64)) / 2.0
    return np.searchsorted(mids, values.astype(np.float64), side="right").astype(np.int64)


def quantize_nf4(w: np.ndarray, blocksize: int = 64, nested: bool = True,
                 bs2: int = 256, out_dtype: str = "float16"):
    """Blockwise NF4 quantization of a 2-D weight (any float dtype).

    Returns (packed uint8 [n/2, 1], QState).  Byte j holds element 2j in its high
    nibble and element 2j+1 in its low nibble (the order nf4.py:45-47 decodes)."""
    assert w.ndim == 2
    n = w.size
    assert n % blocksize == 0 and n % 2 == 0
    flat = w.reshape(-1).astype(np.float32)
    blocks = flat.reshape(-1, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    safe = np.where(absmax == 0, np.float32(1.0), absmax)
    normed = (blocks / safe[:, None]).astype(np.float32)
    code = nf4_codebook()
    idx = _nearest(normed.reshape(-1), code).astype(np.uint8)
    packed = ((idx[0::2] << 4) | idx[1::2]).astype(np.uint8).reshape(-1, 1)
    if not nested:
        st = QState(absmax=absmax, shape=tuple(w.shape), code=code, blocksize=blocksize,
                    dtype=out_dtype, nested=False)
        return packed, st
    offset = np.float32(absmax.mean(dtype=np.float64))
    centred = (absmax - offset).astype(np.float32)
    nb = centred.size
    pad = (-nb) % bs2
    cp = np.concatenate([centred, np.zeros(pad, np.float32)]).reshape(-1, bs2)
    absmax2 = np.abs(cp).max(axis=1).astype(np.float32)
    safe2 = np.where(absmax2 == 0, np.float32(1.0), absmax2)
    code2 = dynamic_map_signed()
    q8 = _nearest((cp / safe2[:, None]).astype(np.float32).reshape(-1), code2)[:nb]
    st = QState(absmax=q8.astype(np.uint8), shape=tuple(w.shape), code=code,
                blocksize=blocksize, dtype=out_dtype, nested=True, offset=float(offset),
                state2=State2(absmax=absmax2, code=code2, blocksize=bs2))
    return packed, st


def fma_f32(a, b, c) -> np.ndarray:
    """fp32 a*b + c rounded ONCE (round to nearest even), elementwise.  The float64 product
    of two fp32 values is exact; TwoSum gives the float64 sum s and its exact error e
    (a*b + c = s + e).  s rounds to fp32 as the exact sum does unless s lies exactly halfway
    between two fp32 values, where the sign of e decides the side."""
    p = np.asarray(a, np.float32).astype(np.float64) * np.asarray(b, np.float32).astype(np.float64)
    c = np.broadcast_to(np.asarray(c, np.float32).astype(np.float64), p.shape)
    s = p + c
    bv = s - p
    e = (p - (s - bv)) + (c - bv)
    with np.errstate(over="ignore"):
        r = s.astype(np.float32)
    r64 = r.astype(np.float64)
    toward = np.where(s > r64, np.float32(np.inf), np.float32(-np.inf)).astype(np.float32)
    n = np.nextafter(r, toward)
    n64 = n.astype(np.float64)
    tie = (s != r64) & (s == (r64 + n64) * 0.5) & (e != 0)
    return np.where(tie & (np.sign(e) == np.sign(n64 - s)), n, r).astype(np.float32)


def block_scales(st: QState, fma: bool = False) -> np.ndarray:
    """Per-block fp32 scale, nf4.py:36-41: code2[q] * absmax2[r // bs2], then + offset,
    each an IEEE fp32 operation rounded on its own (fma: one fused multiply-add)."""
    if not st.nested:
        return np.asarray(st.absmax, dtype=np.float32)
    q = np.asarray(st.absmax).astype(np.int64)
    r = np.arange(q.size)
    outer = np.asarray(st.state2.absmax, np.float32)[r // st.state2.blocksize]
    c2 = np.asarray(st.state2.code, np.float32)[q]
    if fma:
        return fma_f32(c2, outer, np.float32(st.offset))
    prod = (c2 * outer).astype(np.float32)
    return (prod + np.float32(st.offset)).astype(np.float32)


def dequant_nf4(packed: np.ndarray, st: QState, code: np.ndarray | None = None,
                fma: bool = False) -> np.ndarray:
    """Restates `_nf4_unpack` (nf4.py:30-50) for the whole tensor; returns st.shape
    in st.dtype.  `code` defaults to the NF4 table (the reference's `_code()`); fma: the
    nested scale as one fused multiply-add (the contracted variant)."""
    code = nf4_codebook() if code is None else np.asarray(code, np.float32)
    b = np.asarray(packed, np.uint8).reshape(-1)
    n = int(np.prod(st.shape))
    assert n == 2 * b.size and n % st.blocksize == 0
    scale = block_scales(st, fma=fma)
    hb = st.blocksize // 2
    bb = b.reshape(-1, hb)
    hi = (code[(bb >> 4).astype(np.int64)] * scale[:, None]).astype(np.float32)
    lo = (code[(bb & 15).astype(np.int64)] * scale[:, None]).astype(np.float32)
    vals = np.stack([hi, lo], axis=-1).reshape(-1)
    return vals.astype(np.float16 if st.dtype == "float16" else np.float32).reshape(st.shape)


# ---------------------------------------------------------------- GEMM references
def linear_fwd_ref(x: np.ndarray, w16: np.ndarray, bias=None, lora_a=None, lora_b=None,
                   scaling: float = 0.0) -> np.ndarray:
    """Y = X W^T (+ bias) (+ (X A^T) B^T * s), fp64 accumulation of the fp16
    operands.  The fp32-accumulated product of the reference-dequantised weight,
    which is what nf4.py:148-152 computes (unpack, then F.linear) before the fp16
    output rounding; LoRA as peft lora.Linear (y += lora_B(lora_A(x)) * scaling)."""
    xf = x.astype(np.float64)
    y = xf @ w16.astype(np.float64).T
    if bias is not None:
        y += bias.astype(np.float64)
    if lora_a is not None:
        y += (xf @ lora_a.astype(np.float64).T) @ lora_b.astype(np.float64).T * scaling
    return y


def linear_bwd_ref(dy: np.ndarray, w16: np.ndarray, x=None, lora_a=None, lora_b=None,
                   scaling: float = 0.0):
    """dX = dY W (bitsandbytes MatMul4Bit.backward on the re-dequantised weight),
    plus the LoRA contributions: dX += s (dY B) A, dA = s (dY B)^T X, dB = s dY^T (X A^T).
    Returns (dX, dA, dB), fp64."""
    dyf = dy.astype(np.float64)
    dx = dyf @ w16.astype(np.float64)
    da = db = None
    if lora_a is not None:
        a = lora_a.astype(np.float64)
        b = lora_b.astype(np.float64)
        dyb = dyf @ b
        dx += dyb @ a * scaling
        xf = x.astype(np.float64)
        da = scaling * dyb.T @ xf
        db = scaling * dyf.T @ (xf @ a.T)
    return dx, da, db


# ---------------------------------------------------------------- golden inputs
def golden_inputs(shape, bs, nested, dtype, kind, seed):
    """Seeded inputs of one golden case (tests/golden/make_golden.py): `normal` = weights
    N(0, 0.02) quantized by `quantize_nf4`; `random` = uniformly random packed bytes and
    8-bit codes with second-level scales spread over 10^-9..10^6 and a random offset."""
    rng = np.random.default_rng(seed)
    if kind == "normal":
        w = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float16)
        return quantize_nf4(w, blocksize=bs, nested=nested, out_dtype=dtype)
    n = shape[0] * shape[1]
    nb = n // bs
    packed = rng.integers(0, 256, size=(n // 2, 1), dtype=np.uint8)
    if nested:
        q8 = rng.integers(0, 256, size=nb, dtype=np.uint8)
        nb2 = -(-nb // 256)
        absmax2 = (10.0 ** rng.uniform(-9, 6, size=nb2)).astype(np.float32)
        st = QState(absmax=q8, shape=tuple(shape), code=nf4_codebook(), blocksize=bs, dtype=dtype,
                    nested=True, offset=float(np.float32(rng.uniform(-3, 3))),
                    state2=State2(absmax=absmax2, code=dynamic_map_signed(), blocksize=256))
    else:
        absmax = (10.0 ** rng.uniform(-9, 6, size=nb)).astype(np.float32)
        st = QState(absmax=absmax, shape=tuple(shape), code=nf4_codebook(), blocksize=bs, dtype=dtype,
                    nested=False)
    return packed, st
