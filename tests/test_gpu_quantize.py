"""GPU: the quantizer kernels (nf4b_quantize) against the torch formulation of the same
quantizer (stew_b200.quant_state._quantize_torch), bit for bit: packed codes, block absmax,
the double-quantization offset, absmax2 and the 8-bit codes; including values exactly on
the code midpoints (they take the upper code in both) and all-zero blocks."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _compare(A, blocksize, nested):
    from stew_b200.quant_state import _quantize_cuda, _quantize_torch
    pk, st = _quantize_cuda(A, blocksize, nested)
    pt, tt = _quantize_torch(A, blocksize, nested)
    assert torch.equal(pk, pt)
    assert torch.equal(st.absmax, tt.absmax)
    assert st.nested == tt.nested
    if nested:
        assert torch.equal(st.offset.reshape(()), tt.offset.reshape(()).to(st.offset.dtype))
        assert torch.equal(st.state2.absmax, tt.state2.absmax)
        assert torch.equal(st.state2.code, tt.state2.code)
    return pk, st


@pytest.mark.parametrize("shape", [(64, 64), (100, 64), (256, 1536), (1536, 8960)])
@pytest.mark.parametrize("blocksize", [32, 64, 128, 256])
@pytest.mark.parametrize("nested", [True, False])
def test_quantizer_kernel_matches_torch(cuda_lib, shape, blocksize, nested):
    g = torch.Generator(device="cuda").manual_seed(sum(shape) + blocksize)
    A = (torch.randn(shape, generator=g, device="cuda") * 0.02).half()
    if A.numel() % blocksize:
        pytest.skip("numel not a multiple of the blocksize")
    _compare(A, blocksize, nested)


def test_quantizer_midpoints_zero_blocks_and_fp32(cuda_lib):
    from stew_b200 import codebooks
    from stew_b200.quant_state import _mids_f32
    mids = _mids_f32(codebooks.nf4_table("cuda"))
    A = torch.randn(64, 256, device="cuda")
    A[0, :] = 0.0                          # an all-zero block
    A[1, 0] = 1.0                          # absmax exactly 1: the others land on midpoints
    A[1, 1:16] = mids
    A[1, 16:31] = -mids.flip(0)
    A[2, 0] = -1.0
    A[2, 1:16] = mids
    _compare(A, 64, True)                  # fp32 input
    _compare(A.half(), 64, True)           # fp16 input


def test_quantize_then_unpack_round_trip(cuda_lib):
    """The kernel-quantized weight unpacks (nf4b_dequant) to the oracle's dequantisation."""
    import numpy as np
    from oracle import nf4_oracle as O
    from stew_b200 import dequantize_nf4, quantize_4bit
    from tests.helpers import to_oracle_state
    A = (torch.randn(256, 1536, device="cuda") * 0.02).half()
    q, st = quantize_4bit(A, 64, True)
    W = dequantize_nf4(q, st)
    ref = O.dequant_nf4(q.cpu().numpy(), to_oracle_state(st, q))
    assert np.array_equal(W.cpu().numpy().view(np.uint16), ref.astype(np.float16).view(np.uint16))
    # the widest gap of the NF4 code (0.723 .. 1.0) bounds the error at ~0.139 x the block absmax
    assert float((W.float() - A.float()).abs().max()) <= 0.14 * float(A.float().abs().max())
