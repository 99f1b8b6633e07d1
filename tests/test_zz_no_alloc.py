"""GPU: nf4b_lora_grads_noalloc, the LoRA weight-gradient entry point for callers that cannot
allocate device memory (their framework already holds the GPU's memory in its own pool, or
they run where allocating is not allowed), gives the same dA / dB as nf4b_lora_grads with a
caller-provided scratch buffer -- called through the C ABI, twice in a row, so the second
call runs on the scratch array the first one left behind.  Oversized problems are refused
before anything is launched.

This file is named to be collected last."""
import ctypes

import pytest
import torch

from tests.helpers import max_rel_err

pytestmark = pytest.mark.gpu

LORA_GRAD_TOL = 1e-3  # the LoRA weight-gradient tolerance of tests/test_gpu_lora.py


def _inputs(n, in_f, out_f, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(n, in_f, generator=g, device="cuda").half()
    dy = (torch.randn(n, out_f, generator=g, device="cuda") * 0.01).half()
    xa = torch.randn(n, 16, generator=g, device="cuda").half()
    dyb = (torch.randn(n, 16, generator=g, device="cuda") * 0.1).half()
    return x, dy, xa, dyb


def test_noalloc_lora_grads_match_caller_scratch_version(cuda_lib):
    from stew_b200 import _lib
    L = cuda_lib
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # two calls in a row: the q and the v shape of the adapter
    for call, (n, in_f, out_f) in enumerate(((1170, 1536, 1536), (2048, 1536, 256))):
        x, dy, xa, dyb = _inputs(n, in_f, out_f, 40 + call)
        da_ref = torch.empty(16, in_f, device="cuda")
        db_ref = torch.empty(out_f, 16, device="cuda")
        wb = int(L.nf4b_lora_grads_work_bytes(n, in_f, out_f, 16))
        assert 0 < wb <= L.nf4b_lora_grads_work_bytes(n, in_f, out_f, 16)
        work = torch.empty(wb // 4 + 4, device="cuda")
        rc = L.nf4b_lora_grads(x.data_ptr(), dy.data_ptr(), xa.data_ptr(), dyb.data_ptr(), 2.0,
                               da_ref.data_ptr(), db_ref.data_ptr(), work.data_ptr(), n, in_f, out_f,
                               16, stream)
        assert rc == 0, L.nf4b_last_error()
        da = torch.full((16, in_f), float("nan"), device="cuda")
        db = torch.full((out_f, 16), float("nan"), device="cuda")
        rc = L.nf4b_lora_grads_noalloc(x.data_ptr(), dy.data_ptr(), xa.data_ptr(), dyb.data_ptr(),
                                       2.0, da.data_ptr(), db.data_ptr(), n, in_f, out_f, 16, stream)
        assert rc == 0, L.nf4b_last_error()
        torch.cuda.synchronize()
        assert not torch.isnan(da).any() and not torch.isnan(db).any()
        assert max_rel_err(da, da_ref) <= LORA_GRAD_TOL
        assert max_rel_err(db, db_ref) <= LORA_GRAD_TOL
        # and both against fp64: dA = s (dY B)^T X, dB = s dY^T (X A^T)
        assert max_rel_err(da, 2.0 * dyb.double().T @ x.double()) <= LORA_GRAD_TOL
        assert max_rel_err(db, 2.0 * dy.double().T @ xa.double()) <= LORA_GRAD_TOL
    assert _lib.NF4B_OK == 0


def test_noalloc_refuses_problems_larger_than_its_scratch(cuda_lib):
    from stew_b200 import _lib
    L = cuda_lib
    big_in = 1 << 20  # 16 x 2^20 fp32 partial sums = 64 MiB > the fixed scratch
    assert L.nf4b_lora_grads_work_bytes(4096, big_in, 64, 16) > (8 << 20)
    p = ctypes.c_void_p(256)  # never dereferenced: the size check comes first
    rc = L.nf4b_lora_grads_noalloc(p, p, p, p, 2.0, p, p, 4096, big_in, 64, 16, None)
    assert rc == _lib.NF4B_ERR_UNSUPPORTED
    assert b"NF4B_NOALLOC_SCRATCH_BYTES" in L.nf4b_last_error()
