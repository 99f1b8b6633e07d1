"""The NF4 hot path behind the reference's Python interface.

Mirrors evilandangry/stew solution/nf4.py name for name:

  _code(device)                 nf4.py:53-58   the 16-entry NF4 table per device
  _supported(A, st)             nf4.py:61-70   the envelope check
  dequantize_nf4(A, st)         nf4.py:73-92   unpack -> C ABI nf4b_dequant
  patch_bnb_dequant()           nf4.py:95-120  rebinds bitsandbytes' dequantize_4bit
  _patch_matmul4bit_forward()   nf4.py:123-162 MatMul4Bit forward (fused nf4b_linear_fwd)
                                               and backward (fused nf4b_linear_bwd_dx)

plus `MatMul4Bit` / `matmul_4bit`, the same autograd contract for callers that do not
have bitsandbytes.  Behaviour:
  * the forward and the input-gradient backward never write the fp16 weight to HBM:
    the unpack runs inside the tensor-core GEMM (fp16 activations, feature counts that
    are multiples of 64, 16-byte aligned rows -- the fused envelope, `_fused_ok`);
  * activations outside the fused envelope (bf16/fp32 under another autocast, odd
    feature counts) take the reference's own composition, the unpack kernel followed by
    F.linear / matmul (nf4.py:148-152), with a one-time warning naming the cause;
  * the patched bitsandbytes entry points keep the reference's latch (nf4.py:104-112):
    an error inside the fast path sets `_BROKEN`, warns once, and that call and every
    later one go to bitsandbytes' original function ("never break training because of
    the speed-up");
  * the library itself must be present: `apply()` loads it first and raises when it is
    missing, and `MatMul4Bit` / `dequantize_nf4` raise; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import sys
import warnings

import torch

from . import _lib, codebooks
from ._lib import NF4Unsupported, QStateC

_CODE: dict = {}
_BROKEN = False     # the patched bitsandbytes functions fell back for good (nf4.py:25-26)
_WARNED: set = set()


def _warn_once(key: str, msg: str) -> None:
    if key not in _WARNED:
        _WARNED.add(key)
        warnings.warn(f"stew_b200: {msg}", RuntimeWarning, stacklevel=3)


def _code(device) -> torch.Tensor:
    """NF4 table on `device` (fp32 [16]); bitsandbytes' own table when it is importable."""
    key = str(device)
    if key not in _CODE:
        try:
            import bitsandbytes.functional as BF  # the reference's source of the table
            t = BF.get_4bit_type("nf4", device=device).to(torch.float32).contiguous()
        except Exception:  # noqa: BLE001  (not installed: the published table)
            t = codebooks.nf4_table(device)
        _CODE[key] = t
    return _CODE[key]


def _supported(A, st) -> bool:
    """True when the kernels can unpack packed weight A with quant state st (nf4.py:61-70)."""
    return (st is not None and isinstance(A, torch.Tensor) and A.is_cuda and A.dtype == torch.uint8
            and getattr(st, "quant_type", None) == "nf4"
            and st.dtype in (torch.float16, torch.float32)
            and st.blocksize in (32, 64, 128, 256)
            and len(st.shape) == 2
            and st.shape.numel() == 2 * A.numel()
            and st.shape.numel() % st.blocksize == 0
            and (not st.nested or st.state2.blocksize == 256))


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class _QCache:
    """Device-side views of a quant state's tables, kept alive with the state."""
    __slots__ = ("c", "keep")


def _qstate(st, device) -> QStateC:
    """nf4b_qstate for `st` on `device`, converted once and cached on the state object."""
    cache = getattr(st, "_nf4b_cache", None)
    key = (str(device), st.absmax.data_ptr())
    if cache is not None and cache[0] == key:
        return cache[1].c
    keep = []
    c = QStateC()
    c.blocksize = int(st.blocksize)
    code = _code(device)
    keep.append(code)
    c.code = code.data_ptr()
    if st.nested:
        absmax8 = st.absmax.contiguous()
        code2 = st.state2.code.to(device=device, dtype=torch.float32).contiguous()
        absmax2 = st.state2.absmax.to(device=device, dtype=torch.float32).contiguous()
        off = st.offset
        if isinstance(off, torch.Tensor):
            off = off.to(device=device, dtype=torch.float32).reshape(1).contiguous()
        else:
            off = torch.tensor([float(off)], dtype=torch.float32, device=device)
        keep += [absmax8, code2, absmax2, off]
        c.absmax8, c.code2, c.absmax2, c.offset = (absmax8.data_ptr(), code2.data_ptr(),
                                                   absmax2.data_ptr(), off.data_ptr())
        c.blocksize2 = int(st.state2.blocksize)
        c.nested = 1
    else:
        absmax32 = st.absmax.to(device=device, dtype=torch.float32).contiguous()
        keep.append(absmax32)
        c.absmax32 = absmax32.data_ptr()
        c.nested = 0
    entry = _QCache()
    entry.c, entry.keep = c, keep
    try:
        st._nf4b_cache = (key, entry)
    except AttributeError:  # a state that refuses attributes: convert on every call
        pass
    return c


def dequantize_nf4(A: torch.Tensor, st, *, fma_scale: bool = False) -> torch.Tensor:
    """Unpacked weight of shape st.shape and dtype st.dtype (callers check _supported).

    fma_scale: compute a nested state's block scale as one fused multiply-add,
    fmaf(code2[q], absmax2, offset) rounded once, instead of the multiply then the add
    (nf4.py:36-39) -- the contracted form a GPU build of the reference may emit, which its
    test tolerates (solution/test_nf4_unpack.py:29-30).  A debug form for diffing against
    such a build; no effect on plain states."""
    flat = A.reshape(-1)
    out = torch.empty(st.shape, dtype=st.dtype, device=A.device)
    if out.numel() == 0:
        return out
    with torch.cuda.device(A.device):
        qs = _qstate(st, A.device)
        if fma_scale and qs.nested:
            qs = QStateC.from_buffer_copy(qs)
            qs.nested = 2
        dt = _lib.NF4B_F16 if st.dtype == torch.float16 else _lib.NF4B_F32
        _lib.check(_lib.lib().nf4b_dequant(flat.data_ptr(), ctypes.byref(qs), out.data_ptr(), dt,
                                           out.numel(), _stream(A.device)), "nf4b_dequant")
    return out


# (device index, stream handle) -> the stream's workspace (uint8, zeroed once): the split-K
# partials of the fused GEMMs and the token-range partials of the LoRA weight gradients, behind
# leading counter / ticket words that every call leaves zero.  Calls on one stream never overlap,
# so one buffer per stream serves both.
_WORK = {}


def _workspace(device, n: int, in_f: int, out_f: int, backward: bool):
    """(pointer, bytes) of the split-K workspace of nf4b_linear_*_ws for the current stream
    of `device`, or (None, 0) when this shape runs unsplit.  One workspace per stream: its
    counter words are zero between calls (allocated zeroed, left zero by every call), and
    calls on one stream never overlap."""
    return _workspace_bytes(device, int(_lib.lib().nf4b_linear_work_bytes(n, in_f, out_f,
                                                                          1 if backward else 0)))


def _workspace_bytes(device, need: int):
    """The stream's split-K workspace grown to `need` bytes ((None, 0) when need is 0)."""
    if need <= 0:
        return None, 0
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    buf = _WORK.get(key)
    if buf is None or buf.numel() < need:
        buf = torch.zeros(need, dtype=torch.uint8, device=device)
        _WORK[key] = buf
    return buf.data_ptr(), buf.numel()


def _fused_ok(A: torch.Tensor, out_f: int, in_f: int) -> bool:
    """The fused kernels' envelope: fp16 activations, feature counts that are multiples
    of 64 (one K stage), 16-byte aligned rows."""
    return (A.dtype == torch.float16 and in_f % 64 == 0 and out_f % 64 == 0
            and A.data_ptr() % 16 == 0)


def _unfused_reason(A: torch.Tensor, out_f: int, in_f: int) -> str:
    if A.dtype != torch.float16:
        return f"{A.dtype} activations"
    if in_f % 64 or out_f % 64:
        return f"feature counts {out_f}x{in_f} not multiples of 64"
    return "activations not 16-byte aligned"


def linear_forward(A: torch.Tensor, Bv: torch.Tensor, st, bias=None) -> torch.Tensor:
    """Y = A W^T (+ bias) for the NF4 weight (Bv, st): the fused tensor-core kernel inside
    its envelope (`_fused_ok`); outside it, the reference's composition (the unpack kernel,
    then F.linear, nf4.py:148-152) with a one-time warning."""
    out_f, in_f = int(st.shape[0]), int(st.shape[1])
    if _fused_ok(A, out_f, in_f) and (bias is None or bias.dtype == torch.float16):
        x = A.reshape(-1, in_f).contiguous()
        y = torch.empty(x.shape[0], out_f, dtype=torch.float16, device=A.device)
        b = None if bias is None else bias.contiguous()
        with torch.cuda.device(A.device):
            qs = _qstate(st, A.device)
            work, wbytes = _workspace(A.device, x.shape[0], in_f, out_f, False)
            _lib.check(_lib.lib().nf4b_linear_fwd_ws(
                x.data_ptr(), Bv.data_ptr(), ctypes.byref(qs), None if b is None else b.data_ptr(),
                None, y.data_ptr(), x.shape[0], in_f, out_f, work, wbytes, _stream(A.device)),
                "nf4b_linear_fwd_ws")
        return y.reshape(*A.shape[:-1], out_f)
    why = _unfused_reason(A, out_f, in_f) if not _fused_ok(A, out_f, in_f) else "a non-fp16 bias"
    _warn_once("fwd:" + why, f"{why}: the forward runs the unpack kernel + F.linear (not fused)")
    weight = dequantize_nf4(Bv, st).to(A.dtype)
    return torch.nn.functional.linear(A, weight, None if bias is None else bias.to(A.dtype))


def linear_backward_dx(grad_output: torch.Tensor, Bv: torch.Tensor, st) -> torch.Tensor:
    """dX = dY W with W re-unpacked inside the GEMM (bitsandbytes MatMul4Bit.backward grad_A)."""
    out_f, in_f = int(st.shape[0]), int(st.shape[1])
    if _fused_ok(grad_output, out_f, in_f):
        dy = grad_output.reshape(-1, out_f).contiguous()
        dx = torch.empty(dy.shape[0], in_f, dtype=torch.float16, device=dy.device)
        with torch.cuda.device(dy.device):
            qs = _qstate(st, dy.device)
            work, wbytes = _workspace(dy.device, dy.shape[0], in_f, out_f, True)
            _lib.check(_lib.lib().nf4b_linear_bwd_dx_ws(
                dy.data_ptr(), Bv.data_ptr(), ctypes.byref(qs), None, None, dx.data_ptr(),
                dy.shape[0], in_f, out_f, work, wbytes, _stream(dy.device)), "nf4b_linear_bwd_dx_ws")
        return dx.reshape(*grad_output.shape[:-1], in_f)
    why = _unfused_reason(grad_output, out_f, in_f)
    _warn_once("bwd:" + why, f"{why}: the backward runs the unpack kernel + matmul (not fused)")
    weight = dequantize_nf4(Bv, st).to(grad_output.dtype)
    return torch.matmul(grad_output, weight)


def _forward_impl(ctx, A, B, bias, st):
    Bv = B.view(-1, 1)  # the canonical packed layout (nf4.py:146)
    output = linear_forward(A, Bv, st, bias)
    ctx.is_empty = False
    ctx.state = st
    ctx.dtype_A, ctx.dtype_B = A.dtype, Bv.dtype
    ctx.dtype_bias = None if bias is None else bias.dtype
    ctx.tensors = (None, Bv) if any(ctx.needs_input_grad[:2]) else (None, None)
    ctx._stew_b200 = True
    return output


def _backward_impl(ctx, grad_output):
    req_a = ctx.needs_input_grad[0]
    req_bias = ctx.needs_input_grad[3]
    _, Bv = ctx.tensors
    grad_a = grad_bias = None
    if req_bias:
        grad_bias = grad_output.reshape(-1, grad_output.shape[-1]).sum(0, dtype=ctx.dtype_bias)
    if req_a:
        grad_a = linear_backward_dx(grad_output, Bv, ctx.state).to(ctx.dtype_A)
    return grad_a, None, None, grad_bias, None


def _forward_guard(A, B, out, st) -> bool:
    """nf4.py:144-145: no out=, CUDA input with more than one row, supported state."""
    return out is None and A.is_cuda and A.numel() > A.shape[-1] and _supported(B, st)


class MatMul4Bit(torch.autograd.Function):
    """bitsandbytes' MatMul4Bit contract (forward(ctx, A, B, out, bias, quant_state),
    B = the packed weight, typically weight.t()), on the fused kernels."""

    @staticmethod
    def forward(ctx, A, B, out=None, bias=None, quant_state=None):
        if not _forward_guard(A, B, out, quant_state):
            raise NF4Unsupported(_lib.NF4B_ERR_UNSUPPORTED, "MatMul4Bit: input outside the NF4 envelope")
        return _forward_impl(ctx, A, B, bias, quant_state)

    @staticmethod
    def backward(ctx, grad_output):
        return _backward_impl(ctx, grad_output)


def matmul_4bit(A, B, quant_state, out=None, bias=None):
    """bitsandbytes.matmul_4bit(A, B, quant_state, out, bias)."""
    return MatMul4Bit.apply(A, B, out, bias, quant_state)


# ------------------------------------------------------------------ bitsandbytes patches
def _latch(err: Exception) -> None:
    """The reference's `_BROKEN` latch (nf4.py:104-112, :147-150): after the first error in
    a patched fast path, this process uses bitsandbytes' original functions."""
    global _BROKEN
    _BROKEN = True
    _warn_once("broken", f"fast path failed ({err!r}); bitsandbytes' original functions are "
                         "used from now on")


def patch_bnb_dequant():
    """Rebind bitsandbytes.functional.dequantize_4bit (and every bitsandbytes module
    attribute aliasing it, nf4.py:116-119) to the sm_100a unpack; then patch MatMul4Bit."""
    import bitsandbytes.functional as BF

    orig = BF.dequantize_4bit
    if getattr(orig, "_stew_b200", False):
        return

    def dequantize_4bit(A, quant_state=None, absmax=None, out=None, blocksize=64,
                        quant_type="fp4"):
        if not _BROKEN and absmax is None and out is None and _supported(A, quant_state):
            try:
                out_ = dequantize_nf4(A, quant_state)
                # bitsandbytes' rule: a (1, n) packed view gets the result transposed back
                return out_.t() if A.shape[0] == 1 else out_
            except Exception as e:  # noqa: BLE001  (nf4.py:110-111)
                _latch(e)
        return orig(A, quant_state, absmax, out, blocksize, quant_type)

    dequantize_4bit._stew_b200 = True
    dequantize_4bit._stew_b200_orig = orig
    BF.dequantize_4bit = dequantize_4bit
    for name, mod in list(sys.modules.items()):
        if name.startswith("bitsandbytes") and getattr(mod, "dequantize_4bit", None) is orig:
            mod.dequantize_4bit = dequantize_4bit
    _patch_matmul4bit_forward()


def _patch_matmul4bit_forward():
    """Send MatMul4Bit's forward through the fused dequant-GEMM and its backward through
    the fused dequant-GEMM of dY . W.  Anything outside the envelope (out= given, a
    single row, other quant types) keeps the original path; a backward whose forward
    did not run here is handed to the original backward."""
    from bitsandbytes.autograd import _functions as BFN

    cls = BFN.MatMul4Bit
    orig_f = cls.forward
    if getattr(orig_f, "_stew_b200", False):
        return
    orig_b = cls.backward

    def forward(ctx, A, B, out=None, bias=None, quant_state=None):
        if not _BROKEN and _forward_guard(A, B, out, quant_state):
            try:
                return _forward_impl(ctx, A, B, bias, quant_state)
            except Exception as e:  # noqa: BLE001  (nf4.py:150-151)
                _latch(e)
                ctx._stew_b200 = False
        return orig_f(ctx, A, B, out, bias, quant_state)

    def backward(ctx, grad_output):
        if not _BROKEN and getattr(ctx, "_stew_b200", False):
            try:
                return _backward_impl(ctx, grad_output)
            except Exception as e:  # noqa: BLE001  (same latch; ctx holds bitsandbytes' fields)
                _latch(e)
        return orig_b(ctx, grad_output)

    forward._stew_b200 = True
    backward._stew_b200 = True
    cls.forward = staticmethod(forward)
    cls.backward = staticmethod(backward)
