"""Codebooks of the NF4 format.

NF4: the 16 values of the NormalFloat-4 data type as printed in the QLoRA paper
(Dettmers et al. 2023, Appendix E) -- the table bitsandbytes' get_4bit_type("nf4")
returns and the reference reads through `_code()` (solution/nf4.py:53-58).

DYNAMIC8_SIGNED: the 256-entry signed dynamic tree map that double quantization
stores the block absmax values in (Dettmers et al. 2022, "8-bit Optimizers via
Block-wise Quantization"): for decade e = 0..6, magnitudes 10^(e-6) * m where m runs
over the midpoints of 2^e equal steps of [0.1, 1], both signs, plus 0 and +1.0.
"""
from __future__ import annotations

import torch

NF4 = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)


def nf4_table(device="cpu") -> torch.Tensor:
    return torch.tensor(NF4, dtype=torch.float32, device=device)


def dynamic8_signed(device="cpu") -> torch.Tensor:
    vals = []
    for e in range(7):
        edges = torch.linspace(0.1, 1.0, 2 ** e + 1, dtype=torch.float32)
        mids = (edges[:-1] + edges[1:]) / 2.0
        dec = torch.tensor(10.0 ** (e - 6), dtype=torch.float32)
        vals.append(dec * mids)
        vals.append(-dec * mids)
    vals.append(torch.tensor([0.0, 1.0], dtype=torch.float32))
    table = torch.sort(torch.cat(vals)).values
    assert table.numel() == 256
    return table.to(device)
