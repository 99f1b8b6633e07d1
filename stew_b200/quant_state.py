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


@torch.no_grad()
def quantize_4bit(A: torch.Tensor, blocksize: int = 64, compress_statistics: bool = True,
                  quant_type: str = "nf4", quant_storage=torch.uint8):
    """NF4-quantize a 2-D weight.  Returns (packed uint8 [numel/2, 1], QuantState)."""
    if quant_type != "nf4":
        raise ValueError("only nf4 is implemented")
    if quant_storage != torch.uint8:
        raise ValueError("only uint8 storage is implemented")
    n = A.numel()
    if n % blocksize or n % 2:
        raise ValueError("numel must be a multiple of the blocksize")
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
