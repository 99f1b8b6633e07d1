"""QuantState with the attributes of bitsandbytes' QuantState that the NF4 path
reads (solution/nf4.py:61-70, :80-91), and a blockwise NF4 quantizer with the
calling convention of bitsandbytes.functional.quantize_4bit.

The kernels accept a bitsandbytes QuantState just as well (duck typing); this
class exists so the path runs where bitsandbytes is not installed.

The quantizer is weight-loading set-up (the reference gets it from bitsandbytes):
blockwise absmax -> nearest NF4 code (ties to the lower code), high nibble first;
with compress_statistics the fp32 absmax values are centred on their mean and
stored as 8-bit codes of the signed dynamic map in blocks of 256.  It is written
with torch tensor ops so it runs on the GPU for the full-model sweeps.
"""
from __future__ import annotations

import torch

from . import codebooks


class QuantState:
    def __init__(self, absmax, shape, code=None, blocksize=64, quant_type="nf4",
                 dtype=torch.float16, offset=None, state2=None):
        self.absmax = absmax
        self.shape = torch.Size(shape)
        self.code = code
        self.blocksize = int(blocksize)
        self.quant_type = quant_type
        self.dtype = dtype
        self.offset = offset
        self.state2 = state2
        self.nested = state2 is not None

    def to(self, device):
        def mv(t):
            return t.to(device) if isinstance(t, torch.Tensor) else t
        s2 = None
        if self.state2 is not None:
            s2 = QuantState(mv(self.state2.absmax), self.state2.shape, mv(self.state2.code),
                            self.state2.blocksize, dtype=self.state2.dtype)
        return QuantState(mv(self.absmax), self.shape, mv(self.code), self.blocksize,
                          self.quant_type, self.dtype, mv(self.offset), s2)

    def __repr__(self):
        return (f"QuantState(shape={tuple(self.shape)}, blocksize={self.blocksize}, "
                f"nested={self.nested}, dtype={self.dtype})")


def _nearest(values: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    mids = (table[:-1].double() + table[1:].double()) / 2.0
    return torch.searchsorted(mids, values.double().contiguous(), right=True)


_MIDS = {}


def _mids_f32(table: torch.Tensor) -> torch.Tensor:
    """Midpoints of adjacent codes (fp64), each raised to the smallest fp32 >= it, so that
    `v >= mid` in fp32 decides exactly as in fp64 for fp32 v."""
    key = (str(table.device), table.data_ptr(), table.numel())
    if key not in _MIDS:
        t = table.double().cpu()
        mids = (t[:-1] + t[1:]) / 2.0
        m32 = mids.float()
        up = torch.nextafter(m32, torch.full_like(m32, float("inf")))
        m32 = torch.where(m32.double() < mids, up, m32)
        _MIDS[key] = (m32.to(table.device), table)
    return _MIDS[key][0]


def _quantize_cuda(A: torch.Tensor, blocksize: int, compress_statistics: bool):
    """The quantizer kernels of the library (nf4b_quantize): same output as the torch
    formulation below, bit for bit."""
    import ctypes
    from . import _lib
    dev = A.device
    n = A.numel()
    w = A.reshape(-1)
    if w.dtype not in (torch.float16, torch.float32):
        w = w.float()
    w = w.contiguous()
    dt = _lib.NF4B_F16 if w.dtype == torch.float16 else _lib.NF4B_F32
    nb = n // blocksize
    code = codebooks.nf4_table(dev)
    packed = torch.empty(n // 2, dtype=torch.uint8, device=dev)
    absmax = torch.empty(nb, dtype=torch.float32, device=dev)
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    with torch.cuda.device(dev):
        if not compress_statistics:
            _lib.check(L.nf4b_quantize(w.data_ptr(), dt, n, blocksize, _mids_f32(code).data_ptr(), None,
                                       packed.data_ptr(), absmax.data_ptr(), None, None, None, None,
                                       stream), "nf4b_quantize")
            return packed.reshape(-1, 1), QuantState(absmax, A.shape, code, blocksize, "nf4", A.dtype)
        code2 = codebooks.dynamic8_signed(dev)
        q8 = torch.empty(nb, dtype=torch.uint8, device=dev)
        absmax2 = torch.empty((nb + 255) // 256, dtype=torch.float32, device=dev)
        offset = torch.empty(1, dtype=torch.float32, device=dev)
        work = torch.empty(int(L.nf4b_quantize_work_bytes(n, blocksize)) // 8 + 2, dtype=torch.float64,
                           device=dev)
        _lib.check(L.nf4b_quantize(w.data_ptr(), dt, n, blocksize, _mids_f32(code).data_ptr(),
                                   _mids_f32(code2).data_ptr(), packed.data_ptr(), absmax.data_ptr(),
                                   q8.data_ptr(), absmax2.data_ptr(), offset.data_ptr(), work.data_ptr(),
                                   stream), "nf4b_quantize")
    state2 = QuantState(absmax2, absmax2.shape, code2, 256, quant_type="dynamic", dtype=torch.float32)
    return packed.reshape(-1, 1), QuantState(q8, A.shape, code, blocksize, "nf4", A.dtype, offset[0],
                                             state2)


@torch.no_grad()
def quantize_4bit(A: torch.Tensor, blocksize: int = 64, compress_statistics: bool = True,
                  quant_type: str = "nf4", quant_storage=torch.uint8):
    """NF4-quantize a 2-D weight.  Returns (packed uint8 [numel/2, 1], QuantState).
    CUDA tensors go through the library's quantizer kernels; CPU tensors through the torch
    formulation (the same arithmetic)."""
    if quant_type != "nf4":
        raise ValueError("only nf4 is implemented")
    if quant_storage != torch.uint8:
        raise ValueError("only uint8 storage is implemented")
    n = A.numel()
    if n % blocksize or n % 2:
        raise ValueError("numel must be a multiple of the blocksize")
    if A.is_cuda and blocksize in (32, 64, 128, 256):
        return _quantize_cuda(A, blocksize, compress_statistics)
    return _quantize_torch(A, blocksize, compress_statistics)


def _quantize_torch(A: torch.Tensor, blocksize: int, compress_statistics: bool):
    dev = A.device
    blocks = A.reshape(-1, blocksize).float()
    absmax = blocks.abs().amax(dim=1)
    safe = torch.where(absmax == 0, torch.ones_like(absmax), absmax)
    normed = blocks / safe[:, None]
    code = codebooks.nf4_table(dev)
    idx = _nearest(normed.reshape(-1), code).to(torch.uint8)
    packed = ((idx[0::2] << 4) | idx[1::2]).reshape(-1, 1)
    if not compress_statistics:
        return packed, QuantState(absmax, A.shape, code, blocksize, "nf4", A.dtype)
    offset = absmax.double().mean().float()
    centred = absmax - offset
    nb = centred.numel()
    pad = (-nb) % 256
    cp = torch.cat([centred, centred.new_zeros(pad)]).reshape(-1, 256)
    absmax2 = cp.abs().amax(dim=1)
    safe2 = torch.where(absmax2 == 0, torch.ones_like(absmax2), absmax2)
    code2 = codebooks.dynamic8_signed(dev)
    q8 = _nearest((cp / safe2[:, None]).reshape(-1), code2)[:nb].to(torch.uint8)
    state2 = QuantState(absmax2, absmax2.shape, code2, 256, quant_type="dynamic",
                        dtype=torch.float32)
    return packed, QuantState(q8, A.shape, code, blocksize, "nf4", A.dtype, offset, state2)
