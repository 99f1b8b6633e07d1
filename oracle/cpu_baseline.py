"""The reference's NF4 path on host CPU cores -- TEST/BENCH INFRASTRUCTURE ONLY.

A vectorised torch restatement of `_nf4_unpack` (solution/nf4.py:30-50) and of the
patched forward (unpack, then F.linear in fp32, nf4.py:148-152), run with every host
thread.  bench.py times it as the CPU baseline / `--impl reference` arm; it is never part
of the product path.  Bit-identical to oracle.nf4_oracle.dequant_nf4 (tested).
"""
from __future__ import annotations

import torch


def torch_unpack(packed: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, blocksize: int,
                 nested: bool, code2=None, absmax2=None, offset=None, out_dtype=torch.float16):
    """nf4.py:33-50 on CPU tensors: scale = code2[q] * absmax2[r // 256] + offset (two
    roundings) or absmax[r]; value = code[nibble] * scale in fp32; one rounding out."""
    b = packed.reshape(-1, blocksize // 2).to(torch.int64)
    if nested:
        r = torch.arange(b.shape[0])
        scale = code2[absmax.to(torch.int64)] * absmax2[r // 256]
        scale = scale + offset
    else:
        scale = absmax.float()
    hi = code[b >> 4] * scale[:, None]
    lo = code[b & 15] * scale[:, None]
    return torch.stack([hi, lo], dim=-1).reshape(-1).to(out_dtype)


def unpack_state(packed: torch.Tensor, st, code: torch.Tensor) -> torch.Tensor:
    """torch_unpack for a QuantState-like object whose tensors are on the CPU."""
    if st.nested:
        off = st.offset if isinstance(st.offset, torch.Tensor) else torch.tensor(float(st.offset))
        out = torch_unpack(packed, st.absmax, code, st.blocksize, True, st.state2.code.float(),
                           st.state2.absmax.float(), off.float(), st.dtype)
    else:
        out = torch_unpack(packed, st.absmax, code, st.blocksize, False, out_dtype=st.dtype)
    return out.reshape(st.shape)


def linear_forward_cpu(x: torch.Tensor, packed: torch.Tensor, st, code: torch.Tensor) -> torch.Tensor:
    """Unpack, then an fp32 F.linear (the patched forward's two steps on the CPU)."""
    w = unpack_state(packed, st, code).float()
    return torch.nn.functional.linear(x.float(), w)
