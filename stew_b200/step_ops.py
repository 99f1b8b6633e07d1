"""Autograd wrappers of the layer kernels of the packed-token QLoRA step (C ABI
include/stew_step.h): RMSNorm, RMSNorm fused with the residual add, rotary embedding of q and
k, SwiGLU and the LM head's cross-entropy -- the counterparts of the reference's
solution/rmsnorm.py (RMSNormFn :59-92, AddRMSNormFn :192-233), solution/rope.py (:71-92),
solution/swiglu.py (:42-66) and solution/head_loss.py.  fp16 activations, fp32 math; the CUDA
kernels are the only implementation (no torch fallback)."""
from __future__ import annotations

import torch

from . import _lib
from .nf4 import _stream


def _c(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


def _w32(w: torch.Tensor) -> torch.Tensor:
    return _c(w if w.dtype == torch.float32 else w.float())


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        x2 = _c(x.reshape(-1, x.shape[-1]))
        w32 = _w32(w)
        rows, hidden = x2.shape
        y = torch.empty_like(x2)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        _lib.check(_lib.lib().nf4b_rmsnorm_fwd(x2.data_ptr(), None, w32.data_ptr(), float(eps), None,
                                               y.data_ptr(), rstd.data_ptr(), rows, hidden,
                                               _stream(x.device)), "nf4b_rmsnorm_fwd")
        ctx.save_for_backward(x2, w32, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w32, rstd = ctx.saved_tensors
        rows, hidden = x2.shape
        dy2 = _c(dy.reshape(rows, hidden).to(torch.float16))
        dx = torch.empty_like(x2)
        _lib.check(_lib.lib().nf4b_rmsnorm_bwd(dy2.data_ptr(), x2.data_ptr(), w32.data_ptr(),
                                               rstd.data_ptr(), None, dx.data_ptr(), rows, hidden,
                                               _stream(dx.device)), "nf4b_rmsnorm_bwd")
        return dx.view(ctx.shape), None, None


class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, res, delta, w, eps):
        r2 = _c(res.reshape(-1, res.shape[-1]))
        d2 = _c(delta.reshape(r2.shape))
        w32 = _w32(w)
        rows, hidden = r2.shape
        s = torch.empty_like(r2)
        y = torch.empty_like(r2)
        rstd = torch.empty(rows, dtype=torch.float32, device=res.device)
        _lib.check(_lib.lib().nf4b_rmsnorm_fwd(r2.data_ptr(), d2.data_ptr(), w32.data_ptr(), float(eps),
                                               s.data_ptr(), y.data_ptr(), rstd.data_ptr(), rows,
                                               hidden, _stream(res.device)), "nf4b_rmsnorm_fwd")
        ctx.save_for_backward(s, w32, rstd)
        ctx.shape = res.shape
        return s.view(res.shape), y.view(res.shape)

    @staticmethod
    def backward(ctx, ds, dy):
        s, w32, rstd = ctx.saved_tensors
        rows, hidden = s.shape
        dx = torch.empty_like(s)
        if dy is None:  # only the residual stream is used downstream
            dx.copy_(ds.reshape(rows, hidden))
        else:
            dy2 = _c(dy.reshape(rows, hidden).to(torch.float16))
            ds2 = None if ds is None else _c(ds.reshape(rows, hidden).to(torch.float16))
            _lib.check(_lib.lib().nf4b_rmsnorm_bwd(dy2.data_ptr(), s.data_ptr(), w32.data_ptr(),
                                                   rstd.data_ptr(), None if ds2 is None else ds2.data_ptr(),
                                                   dx.data_ptr(), rows, hidden, _stream(dx.device)),
                       "nf4b_rmsnorm_bwd")
        dxv = dx.view(ctx.shape)
        return dxv, dxv, None, None


class _RopeQK(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, cos, sin):
        q, k = _c(q), _c(k)
        cos32, sin32 = _c(cos.float()), _c(sin.float())
        qo, ko = torch.empty_like(q), torch.empty_like(k)
        _RopeQK._run(q, k, cos32, sin32, qo, ko, 0)
        ctx.save_for_backward(cos32, sin32)
        return qo, ko

    @staticmethod
    def _run(q, k, cos32, sin32, qo, ko, inverse):
        t, hq, d = q.shape
        _lib.check(_lib.lib().nf4b_rope_qk(q.data_ptr(), k.data_ptr(), cos32.data_ptr(), sin32.data_ptr(),
                                           qo.data_ptr(), ko.data_ptr(), t, hq, k.shape[1], d, inverse,
                                           _stream(q.device)), "nf4b_rope_qk")

    @staticmethod
    def backward(ctx, dq, dk):
        cos32, sin32 = ctx.saved_tensors
        dq = _c(dq.to(torch.float16))
        dk = _c(dk.to(torch.float16))
        gq, gk = torch.empty_like(dq), torch.empty_like(dk)
        _RopeQK._run(dq, dk, cos32, sin32, gq, gk, 1)
        return gq, gk, None, None


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gate, up):
        g, u = _c(gate), _c(up)
        m = torch.empty_like(g)
        _lib.check(_lib.lib().nf4b_swiglu_fwd(g.data_ptr(), u.data_ptr(), m.data_ptr(), g.numel(),
                                              _stream(g.device)), "nf4b_swiglu_fwd")
        ctx.save_for_backward(g, u)
        return m

    @staticmethod
    def backward(ctx, dm):
        g, u = ctx.saved_tensors
        dm = _c(dm.to(torch.float16))
        dg, du = torch.empty_like(g), torch.empty_like(u)
        _lib.check(_lib.lib().nf4b_swiglu_bwd(dm.data_ptr(), g.data_ptr(), u.data_ptr(), dg.data_ptr(),
                                              du.data_ptr(), g.numel(), _stream(g.device)),
                   "nf4b_swiglu_bwd")
        return dg, du


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """fp16(w * fp16(x * rsqrt(mean(x^2) + eps))) over the last dimension."""
    return _RMSNorm.apply(x, w, eps)


def add_rms_norm(res: torch.Tensor, delta: torch.Tensor, w: torch.Tensor, eps: float):
    """(s, rms_norm(s)) with s = fp16(res + delta): the residual add and the next norm."""
    return _AddRMSNorm.apply(res, delta, w, eps)


def rope_qk(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """Rotary embedding (rotate-half) of q [T, Hq, D] and k [T, Hk, D]; cos/sin [T, D]."""
    return _RopeQK.apply(q, k, cos, sin)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """fp16(gate * sigmoid(gate) * up), fp32 inside (the reference's SwiGLU kernel)."""
    return _SwiGLU.apply(gate, up)


# The backward's softmax - onehot is written as fp16 times this power of two (exact to divide
# out): a 151,936-entry row's probabilities are ~1e-5 and would otherwise sit in fp16's
# subnormal range.
CE_GRAD_SCALE = 1024.0


class _HeadCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, embed, labels):
        h2 = _c(h)
        logits = h2 @ embed.t()  # [rows, vocab] fp16 (cuBLAS)
        rows, vocab = logits.shape
        lab = _c(labels.to(torch.int64))
        loss = torch.empty(rows, dtype=torch.float32, device=h.device)
        lse = torch.empty(rows, dtype=torch.float32, device=h.device)
        _lib.check(_lib.lib().nf4b_ce_fwd(logits.data_ptr(), lab.data_ptr(), loss.data_ptr(), lse.data_ptr(),
                                          rows, vocab, _stream(h.device)), "nf4b_ce_fwd")
        ctx.save_for_backward(logits, lab, lse, embed)
        return loss.sum()

    @staticmethod
    def backward(ctx, g):
        logits, lab, lse, embed = ctx.saved_tensors
        rows, vocab = logits.shape
        gs = (g.float() * CE_GRAD_SCALE).reshape(1).contiguous()
        # softmax - onehot over the logits' own storage (they are not needed afterwards)
        _lib.check(_lib.lib().nf4b_ce_bwd(logits.data_ptr(), lab.data_ptr(), lse.data_ptr(), gs.data_ptr(),
                                          rows, vocab, _stream(logits.device)), "nf4b_ce_bwd")
        dh = logits @ embed
        dh.mul_(1.0 / CE_GRAD_SCALE)
        return dh, None, None


def head_cross_entropy(h: torch.Tensor, embed: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    """Sum over rows of CE(h @ embed^T, labels): fp16 logits from one GEMM, then the fused
    loss kernel; the gradient of h only (the embedding is frozen).  Labels outside
    [0, vocab) are ignored."""
    return _HeadCrossEntropy.apply(h, embed, labels)
