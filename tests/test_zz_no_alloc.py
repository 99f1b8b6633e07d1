"""GPU: nf4b_lora_grads_noalloc, the LoRA weight-gradient entry point for callers that cannot
allocate device memory (their framework already holds the GPU's memory in its own pool, or
they run where allocating is not allowed), gives the same dA / dB as nf4b_lora_grads with a
caller-provided scratch buffer -- called through the C ABI, twice in a row, so the second
call runs on the scratch array the first one left behind (its ticket words must have been left
zero).  Its fixed array covers the scratch of every rank-16 problem, so it refuses none; the
size check that would refuse one stays as a guard.

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
        work = torch.zeros(wb // 4 + 4, device="cuda")  # ticket words zero before the first call
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


def test_noalloc_scratch_covers_every_rank16_problem(cuda_lib):
    """The scratch of a rank-16 problem is at most ~2.4 MB (two token-range partials of 8 KB per
    SM plus 4 KB of ticket words), below the fixed 4 MiB array for every shape and token count;
    wrong ranks are refused before anything is launched."""
    from stew_b200 import _lib
    L = cuda_lib
    limit = 4 << 20
    worst = 0
    for n in (1, 64, 65, 1170, 2048, 8192, 1 << 20):
        for in_f in (8, 256, 1536, 8960, 8192, 12800, 18816, 1 << 20):
            for out_f in (8, 256, 1536, 8960):
                worst = max(worst, int(L.nf4b_lora_grads_work_bytes(n, in_f, out_f, 16)))
    assert 0 < worst <= limit
    p = ctypes.c_void_p(256)  # never dereferenced: the rank check comes before any launch
    rc = L.nf4b_lora_grads_noalloc(p, p, p, p, 2.0, p, p, 4096, 1536, 1536, 8, None)
    assert rc == _lib.NF4B_ERR_UNSUPPORTED
