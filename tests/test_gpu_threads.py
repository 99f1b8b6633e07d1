"""GPU: the C ABI works from any host thread -- worker threads that reach it with no CUDA
context bound (a framework's device guard is a no-op when it believes the device is
already current) and torch's autograd worker threads."""
import threading

import pytest
import torch

from tests.helpers import GEMM_MAX_REL_ERR, max_rel_err
from tests.test_gpu_gemm import _ref_weight, _weight, _x

pytestmark = pytest.mark.gpu


def _run_in_thread(fn):
    box = {}

    def target():
        try:
            box["out"] = fn()
        except Exception as e:  # noqa: BLE001
            box["err"] = e

    t = threading.Thread(target=target)
    t.start()
    t.join()
    if "err" in box:
        raise box["err"]
    return box["out"]


def test_fwd_bwd_dequant_from_fresh_threads(cuda_lib):
    from stew_b200 import dequantize_nf4
    from stew_b200.nf4 import linear_backward_dx, linear_forward
    q, st = _weight((512, 256), 31)
    W = _ref_weight(q, st)
    x = _x(74, 256, 1)
    dy = _x(74, 512, 2)
    for _ in range(2):  # before and after the main thread has used every kernel
        y = _run_in_thread(lambda: linear_forward(x, q.view(-1, 1), st))
        dx = _run_in_thread(lambda: linear_backward_dx(dy, q.view(-1, 1), st))
        w = _run_in_thread(lambda: dequantize_nf4(q, st))
        torch.cuda.synchronize()
        assert max_rel_err(y, x.double() @ W.T) <= GEMM_MAX_REL_ERR
        assert max_rel_err(dx, dy.double() @ W) <= GEMM_MAX_REL_ERR
        assert torch.equal(w.double(), W)
        linear_forward(x, q.view(-1, 1), st)
        linear_backward_dx(dy, q.view(-1, 1), st)


def test_autograd_worker_thread(cuda_lib):
    from stew_b200 import matmul_4bit
    q, st = _weight((512, 256), 32)
    x = _x(2 * 37, 256, 3).reshape(2, 37, 256).requires_grad_(True)
    y = matmul_4bit(x, q.t(), st)
    g = torch.randn_like(y)
    y.backward(g)
    ref = g.double().reshape(-1, 512) @ _ref_weight(q, st)
    assert max_rel_err(x.grad.reshape(-1, 256), ref) <= GEMM_MAX_REL_ERR
