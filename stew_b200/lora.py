"""NF4 base weight + rank-16 LoRA adapter as one fused autograd op.

peft's lora.Linear computes y = base(x) + lora_B(lora_A(dropout(x))) * scaling; on the
q/v projections of the reference run the base layer is a bitsandbytes Linear4bit NF4
(r = 16, lora_alpha = 32 -> scaling 2; the reference only touches peft's input cast,
solution/rmsnorm.py:137-150, and its dropout modules, solution/unpad.py:77-138).

Here the whole thing is two launches forward (x A^T, then one tensor-core GEMM that
unpacks W and adds the adapter as an extra K=16 slab) and three backward (dY B, the
fused dX GEMM with the adapter slab, and one launch for both weight gradients).
Dropout must be 0 (the configuration this path serves); other adapters use peft's own path.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .nf4 import _qstate, _stream, _supported, _workspace, _workspace_bytes

LORA_RANK = 16


def _lora_c(a16, b16, scale, xa=None) -> _lib.LoraC:
    c = _lib.LoraC()
    c.a = a16.data_ptr()
    c.b = b16.data_ptr()
    c.scale = float(scale)
    c.rank = LORA_RANK
    c.xa = None if xa is None else xa.data_ptr()
    return c


def _fusable(x, st, lora_a, lora_b) -> bool:
    out_f, in_f = int(st.shape[0]), int(st.shape[1])
    return (x.dtype == torch.float16 and in_f % 64 == 0 and out_f % 64 == 0
            and lora_a.shape == (LORA_RANK, in_f) and lora_b.shape == (out_f, LORA_RANK))


def _half_of(p: torch.Tensor) -> torch.Tensor:
    """fp16 form of an adapter matrix: the model's shared fp16 shadow of its adapters (one
    copy kernel per step refreshes all of them) when it keeps one, else a conversion."""
    h = getattr(p, "_stew_half", None)
    return h if h is not None else p.to(torch.float16).contiguous()


class NF4LoraFunction(torch.autograd.Function):
    """y = x W^T (+ bias) + (x A^T) B^T * scaling, W the NF4 weight (packed, st)."""

    @staticmethod
    def forward(ctx, x, packed, st, bias, lora_a, lora_b, scaling):
        out_f, in_f = int(st.shape[0]), int(st.shape[1])
        a16 = _half_of(lora_a)
        b16 = _half_of(lora_b)
        x2 = x.reshape(-1, in_f).contiguous()
        n = x2.shape[0]
        Bv = packed.view(-1, 1)
        y = torch.empty(n, out_f, dtype=torch.float16, device=x.device)
        xa = torch.empty(n, LORA_RANK, dtype=torch.float16, device=x.device)
        with torch.cuda.device(x.device):
            qs = _qstate(st, x.device)
            lc = _lora_c(a16, b16, scaling, xa)
            b = None if bias is None else bias.to(torch.float16).contiguous()
            work, wbytes = _workspace(x.device, n, in_f, out_f, False)
            _lib.check(_lib.lib().nf4b_linear_fwd_ws(
                x2.data_ptr(), Bv.data_ptr(), ctypes.byref(qs), None if b is None else b.data_ptr(),
                ctypes.byref(lc), y.data_ptr(), n, in_f, out_f, work, wbytes, _stream(x.device)),
                "nf4b_linear_fwd_ws")
        ctx.save_for_backward(x2, xa, a16, b16)
        ctx.st, ctx.Bv, ctx.scaling = st, Bv, float(scaling)
        ctx.x_shape = x.shape
        ctx.has_bias = bias is not None
        ctx.param_dtypes = (lora_a.dtype, lora_b.dtype, None if bias is None else bias.dtype)
        return y.reshape(*x.shape[:-1], out_f)

    @staticmethod
    def backward(ctx, grad_y):
        x2, xa, a16, b16 = ctx.saved_tensors
        st = ctx.st
        out_f, in_f = int(st.shape[0]), int(st.shape[1])
        dy = grad_y.reshape(-1, out_f).to(torch.float16).contiguous()
        n = dy.shape[0]
        dev = dy.device
        need_x, need_a, need_b = ctx.needs_input_grad[0], ctx.needs_input_grad[4], ctx.needs_input_grad[5]
        dx = da = db = dbias = None
        dyb = torch.empty(n, LORA_RANK, dtype=torch.float16, device=dev)
        with torch.cuda.device(dev):
            qs = _qstate(st, dev)
            lc = _lora_c(a16, b16, ctx.scaling)
            L = _lib.lib()
            dxt = torch.empty(n, in_f, dtype=torch.float16, device=dev)
            work, wbytes = _workspace(dev, n, in_f, out_f, True)
            _lib.check(L.nf4b_linear_bwd_dx_ws(dy.data_ptr(), ctx.Bv.data_ptr(), ctypes.byref(qs),
                                               ctypes.byref(lc), dyb.data_ptr(), dxt.data_ptr(), n, in_f,
                                               out_f, work, wbytes, _stream(dev)), "nf4b_linear_bwd_dx_ws")
            if need_x:
                dx = dxt.reshape(ctx.x_shape)
            if need_a or need_b:
                da32 = torch.empty(LORA_RANK, in_f, dtype=torch.float32, device=dev)
                db32 = torch.empty(out_f, LORA_RANK, dtype=torch.float32, device=dev)
                # the stream's zeroed workspace (its ticket words are left zero by every call)
                work, _ = _workspace_bytes(dev, max(int(L.nf4b_lora_grads_work_bytes(n, in_f, out_f,
                                                                                    LORA_RANK)), 256))
                _lib.check(L.nf4b_lora_grads(x2.data_ptr(), dy.data_ptr(), xa.data_ptr(), dyb.data_ptr(),
                                             ctx.scaling, da32.data_ptr(), db32.data_ptr(),
                                             work, n, in_f, out_f, LORA_RANK, _stream(dev)),
                           "nf4b_lora_grads")
                da = da32.to(ctx.param_dtypes[0]) if need_a else None
                db = db32.to(ctx.param_dtypes[1]) if need_b else None
        if ctx.has_bias and ctx.needs_input_grad[3]:
            dbias = dy.float().sum(0).to(ctx.param_dtypes[2])
        return dx, None, None, dbias, da, db, None


class GroupedNF4Function(torch.autograd.Function):
    """Several NF4 projections of one input -- q/k/v, or gate/up -- each optionally with a
    rank-16 adapter: ONE forward launch (nf4b_linear_fwd_group; the adapters' x A^T
    projections run just before it).  Backward: ONE dX GEMM over the concatenated out features
    (nf4b_linear_bwd_dx_group, with the adapters' dX terms), and each adapter's weight
    gradients.
    specs: one (packed, quant_state, scaling or None, bias or None) per projection;
    params: (lora_A, lora_B) of the projections whose scaling is not None, in order."""

    @staticmethod
    def forward(ctx, x, specs, *params):
        in_f = int(specs[0][1].shape[1])
        x2 = x.reshape(-1, in_f).contiguous()
        n = x2.shape[0]
        dev = x.device
        items = (_lib.LinearItemC * len(specs))()
        keep, outs, saved, pi = [], [], [], 0
        with torch.cuda.device(dev):
            for i, (packed, st, scaling, bias) in enumerate(specs):
                out_f = int(st.shape[0])
                y = torch.empty(n, out_f, dtype=torch.float16, device=dev)
                qs = _qstate(st, dev)
                b = None if bias is None else bias.to(torch.float16).contiguous()
                lc = None
                if scaling is not None:
                    a16 = _half_of(params[pi])
                    b16 = _half_of(params[pi + 1])
                    xa = torch.empty(n, LORA_RANK, dtype=torch.float16, device=dev)
                    lc = _lora_c(a16, b16, scaling, xa)
                    saved.append((a16, b16, xa))
                    pi += 2
                keep += [y, qs, b, lc]
                items[i].packed = packed.data_ptr()
                items[i].qs = ctypes.pointer(qs)
                items[i].bias = None if b is None else b.data_ptr()
                items[i].lora = None if lc is None else ctypes.pointer(lc)
                items[i].y = y.data_ptr()
                items[i].out_features = out_f
                outs.append(y)
            outs_c = (ctypes.c_int64 * len(specs))(*[int(st.shape[0]) for _, st, _, _ in specs])
            need = int(_lib.lib().nf4b_linear_group_work_bytes(n, in_f, outs_c, len(specs)))
            work, wbytes = _workspace_bytes(dev, need)
            _lib.check(_lib.lib().nf4b_linear_fwd_group(x2.data_ptr(), n, in_f, items, len(specs), work,
                                                        wbytes, _stream(dev)), "nf4b_linear_fwd_group")
        tensors = [x2]
        for a16, b16, xa in saved:
            tensors += [a16, b16, xa]
        ctx.save_for_backward(*tensors)
        ctx.specs = specs
        ctx.x_shape = x.shape
        ctx.param_dtypes = [p.dtype for p in params]
        return tuple(y.reshape(*x.shape[:-1], y.shape[1]) for y in outs)

    @staticmethod
    def backward(ctx, *grads):
        x2, *rest = ctx.saved_tensors
        n, in_f = x2.shape
        dev = x2.device
        L = _lib.lib()
        sel, pgrads, li = [], [], 0
        for (packed, st, scaling, _), gy in zip(ctx.specs, grads):
            lora = None
            if scaling is not None:
                lora = tuple(rest[3 * li:3 * li + 3]) + (scaling,)  # a16, b16, xa, scaling
                li += 1
            sel.append((packed, st, lora, gy))
        live = [x for x in sel if x[3] is not None]
        dx = None
        with torch.cuda.device(dev):
            if live:
                # one GEMM over the concatenated out features: dX = sum_i dY_i W_i (+ adapters)
                items = (_lib.LinearBwdItemC * len(live))()
                keep = []
                for j, (packed, st, lora, gy) in enumerate(live):
                    out_f = int(st.shape[0])
                    dy = gy.reshape(n, out_f).to(torch.float16).contiguous()
                    qs = _qstate(st, dev)
                    lc = dyb = None
                    if lora is not None:
                        dyb = torch.empty(n, LORA_RANK, dtype=torch.float16, device=dev)
                        lc = _lora_c(lora[0], lora[1], lora[3])
                    keep.append((dy, qs, lc, dyb))
                    items[j].dy = dy.data_ptr()
                    items[j].packed = packed.data_ptr()
                    items[j].qs = ctypes.pointer(qs)
                    items[j].lora = None if lc is None else ctypes.pointer(lc)
                    items[j].dyb = None if dyb is None else dyb.data_ptr()
                    items[j].out_features = out_f
                dx = torch.empty(n, in_f, dtype=torch.float16, device=dev)
                outs = (ctypes.c_int64 * len(live))(*[int(st.shape[0]) for _, st, _, _ in live])
                need = int(L.nf4b_linear_bwd_group_work_bytes(n, in_f, outs, len(live)))
                work, wbytes = _workspace_bytes(dev, need)
                _lib.check(L.nf4b_linear_bwd_dx_group(items, len(live), dx.data_ptr(), n, in_f, work,
                                                      wbytes, _stream(dev)), "nf4b_linear_bwd_dx_group")
                kj = 0
            # every adapter's dA, dB in one outer-product launch and one reduction launch
            gitems, slots = [], []
            for packed, st, lora, gy in sel:
                if lora is None:
                    if gy is not None:
                        kj += 1
                    continue
                if gy is None:
                    pgrads += [None, None]
                    continue
                dy, _, _, dyb = keep[kj]
                kj += 1
                out_f = int(st.shape[0])
                da32 = torch.empty(LORA_RANK, in_f, dtype=torch.float32, device=dev)
                db32 = torch.empty(out_f, LORA_RANK, dtype=torch.float32, device=dev)
                it = _lib.LoraGradsItemC()
                it.x, it.dy, it.xa, it.dyb = x2.data_ptr(), dy.data_ptr(), lora[2].data_ptr(), dyb.data_ptr()
                it.scale, it.da, it.db = float(lora[3]), da32.data_ptr(), db32.data_ptr()
                it.in_features, it.out_features = in_f, out_f
                gitems.append(it)
                pgrads += [da32, db32]
            if gitems:
                arr = (_lib.LoraGradsItemC * len(gitems))(*gitems)
                wb = max(int(L.nf4b_lora_grads_group_work_bytes(arr, len(gitems), n)), 256)
                work, wbytes = _workspace_bytes(dev, wb)
                _lib.check(L.nf4b_lora_grads_group(arr, len(gitems), work, wbytes, n, _stream(dev)),
                           "nf4b_lora_grads_group")
        pgrads = [None if gr is None else gr.to(dt) for gr, dt in zip(pgrads, ctx.param_dtypes)]
        return (None if dx is None else dx.reshape(ctx.x_shape), None, *pgrads)


class SwiGLUProjection(torch.autograd.Function):
    """m = fp16(g * sigmoid(g) * u), g = x Wg^T, u = x Wu^T, for the NF4 gate and up weights of an
    MLP, in ONE launch (nf4b_linear_fwd_swiglu: the GEMM's epilogue applies the SwiGLU; gate and up
    are also written, for the backward).  Backward: the SwiGLU backward kernel gives dgate and
    dup, then ONE dX GEMM over the concatenated gate/up out features (nf4b_linear_bwd_dx_group)."""

    @staticmethod
    def forward(ctx, x, gate, up):
        in_f = int(gate[1].shape[1])
        x2 = x.reshape(-1, in_f).contiguous()
        with torch.cuda.device(x.device):
            g, u, m = _swiglu_launch(x2, gate, up)
        ctx.save_for_backward(g, u)
        ctx.weights = (gate, up)
        ctx.x_shape = x.shape
        return m.reshape(*x.shape[:-1], m.shape[1])

    @staticmethod
    def backward(ctx, dm):
        g, u = ctx.saved_tensors
        gate, up = ctx.weights
        n, out_f = g.shape
        dev = g.device
        dm = dm.reshape(n, out_f).to(torch.float16).contiguous()
        dg, du = torch.empty_like(g), torch.empty_like(u)
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().nf4b_swiglu_bwd(dm.data_ptr(), g.data_ptr(), u.data_ptr(), dg.data_ptr(),
                                                  du.data_ptr(), g.numel(), _stream(dev)), "nf4b_swiglu_bwd")
            dx = _gate_up_bwd(dg, du, gate, up, int(gate[1].shape[1]))
        return dx.reshape(ctx.x_shape), None, None


class MLPFunction(torch.autograd.Function):
    """down(fp16(g * sigmoid(g) * u)), g = x Wg^T, u = x Wu^T, of a SwiGLU MLP with NF4 gate, up
    and down weights (no bias, no adapter):
      forward : nf4b_linear_fwd_swiglu (gate, up and the SwiGLU in one launch), then the down
                projection;
      backward: dm = dX of down (nf4b_linear_bwd_dx_ws), dgate/dup from the SwiGLU backward
                kernel (nf4b_swiglu_bwd), then ONE dX GEMM over the concatenated gate/up out
                features.  fused_backward=True applies the SwiGLU backward in down's dX epilogue
                instead (nf4b_linear_bwd_dx_swiglu, bit-identical): one launch and no dm in HBM,
                but on B200 its epilogue -- two loads and two stores per output, bound by load
                latency -- outlasts the tile's MMAs (66 vs 60 us at 1,170 tokens), so it is off
                by default.
    recompute=True keeps only x: the backward runs the forward's gate/up launch again for g and u
    (the reference's MLP memory cap, solution/unpad.py:48-57) -- no torch checkpoint, so the step
    stays capturable in a CUDA graph."""

    @staticmethod
    def forward(ctx, x, gate, up, down, recompute, fused_backward=False):
        (pg, sg), (pu, su), (pd, sd) = gate, up, down
        inter, hidden = int(sg.shape[0]), int(sg.shape[1])
        x2 = x.reshape(-1, hidden).contiguous()
        n = x2.shape[0]
        dev = x.device
        with torch.cuda.device(dev):
            g, u, m = _swiglu_launch(x2, gate, up)
            y = torch.empty(n, hidden, dtype=torch.float16, device=dev)
            qd = _qstate(sd, dev)
            work, wbytes = _workspace(dev, n, inter, hidden, False)
            _lib.check(_lib.lib().nf4b_linear_fwd_ws(m.data_ptr(), pd.view(-1, 1).data_ptr(), ctypes.byref(qd),
                                                     None, None, y.data_ptr(), n, inter, hidden, work, wbytes,
                                                     _stream(dev)), "nf4b_linear_fwd_ws")
        if recompute:
            ctx.save_for_backward(x2)
        else:
            ctx.save_for_backward(x2, g, u)
        ctx.weights = (gate, up, down)
        ctx.x_shape = x.shape
        ctx.fused_backward = fused_backward
        return y.reshape(*x.shape[:-1], hidden)

    @staticmethod
    def backward(ctx, dy):
        saved = ctx.saved_tensors
        (pg, sg), (pu, su), (pd, sd) = ctx.weights
        x2 = saved[0]
        inter, hidden = int(sg.shape[0]), int(sg.shape[1])
        n = x2.shape[0]
        dev = x2.device
        dy = dy.reshape(n, hidden).to(torch.float16).contiguous()
        with torch.cuda.device(dev):
            L = _lib.lib()
            if len(saved) == 3:
                g, u = saved[1], saved[2]
            else:
                g, u, _ = _swiglu_launch(x2, (pg, sg), (pu, su))
            dg, du = torch.empty_like(g), torch.empty_like(u)
            qd = _qstate(sd, dev)
            work, wbytes = _workspace(dev, n, inter, hidden, True)
            st = _stream(dev)
            if ctx.fused_backward:
                _lib.check(L.nf4b_linear_bwd_dx_swiglu(dy.data_ptr(), pd.view(-1, 1).data_ptr(), ctypes.byref(qd),
                                                       g.data_ptr(), u.data_ptr(), dg.data_ptr(), du.data_ptr(), n,
                                                       inter, hidden, work, wbytes, st),
                           "nf4b_linear_bwd_dx_swiglu")
            else:
                dm = torch.empty_like(g)
                _lib.check(L.nf4b_linear_bwd_dx_ws(dy.data_ptr(), pd.view(-1, 1).data_ptr(), ctypes.byref(qd),
                                                   None, None, dm.data_ptr(), n, inter, hidden, work, wbytes, st),
                           "nf4b_linear_bwd_dx_ws")
                _lib.check(L.nf4b_swiglu_bwd(dm.data_ptr(), g.data_ptr(), u.data_ptr(), dg.data_ptr(),
                                             du.data_ptr(), g.numel(), st), "nf4b_swiglu_bwd")
            dx = _gate_up_bwd(dg, du, (pg, sg), (pu, su), hidden)
        return dx.reshape(ctx.x_shape), None, None, None, None, None


def _swiglu_launch(x2, gate, up):
    """(g, u, m) of one nf4b_linear_fwd_swiglu launch."""
    (pg, sg), (pu, su) = gate, up
    out_f, in_f = int(sg.shape[0]), int(sg.shape[1])
    n = x2.shape[0]
    dev = x2.device
    g = torch.empty(n, out_f, dtype=torch.float16, device=dev)
    u = torch.empty_like(g)
    m = torch.empty_like(g)
    L = _lib.lib()
    qg, qu = _qstate(sg, dev), _qstate(su, dev)
    work, wbytes = _workspace_bytes(dev, int(L.nf4b_linear_swiglu_work_bytes(n, in_f, out_f)))
    _lib.check(L.nf4b_linear_fwd_swiglu(x2.data_ptr(), n, in_f, pg.data_ptr(), ctypes.byref(qg), pu.data_ptr(),
                                        ctypes.byref(qu), g.data_ptr(), u.data_ptr(), m.data_ptr(), out_f, work,
                                        wbytes, _stream(dev)), "nf4b_linear_fwd_swiglu")
    return g, u, m


def _gate_up_bwd(dg, du, gate, up, in_f):
    """dX = dg Wg + du Wu as one K-concatenated dX GEMM."""
    (pg, sg), (pu, su) = gate, up
    n, out_f = dg.shape
    dev = dg.device
    L = _lib.lib()
    items = (_lib.LinearBwdItemC * 2)()
    qs = [_qstate(sg, dev), _qstate(su, dev)]
    for j, (packed, dy, q) in enumerate(((pg, dg, qs[0]), (pu, du, qs[1]))):
        items[j].dy, items[j].packed, items[j].qs = dy.data_ptr(), packed.data_ptr(), ctypes.pointer(q)
        items[j].lora, items[j].dyb, items[j].out_features = None, None, out_f
    dx = torch.empty(n, in_f, dtype=torch.float16, device=dev)
    outs = (ctypes.c_int64 * 2)(out_f, out_f)
    work, wbytes = _workspace_bytes(dev, int(L.nf4b_linear_bwd_group_work_bytes(n, in_f, outs, 2)))
    _lib.check(L.nf4b_linear_bwd_dx_group(items, 2, dx.data_ptr(), n, in_f, work, wbytes, _stream(dev)),
               "nf4b_linear_bwd_dx_group")
    return dx


def nf4_mlp(x, gate, up, down, recompute: bool = False, fused_backward: bool = False):
    """down(SwiGLU(gate(x), up(x))) for three NF4Linear modules without bias (MLPFunction): two
    launches forward, three backward (four with recompute=True, which keeps only x);
    fused_backward=True puts the SwiGLU backward in down's dX epilogue (one launch fewer)."""
    return MLPFunction.apply(x, (gate.packed, gate.quant_state), (up.packed, up.quant_state),
                             (down.packed, down.quant_state), bool(recompute), bool(fused_backward))


def swiglu_projection(x, gate, up):
    """fp16(g * sigmoid(g) * u) of g = gate(x), u = up(x) for two NF4Linear modules without bias (an MLP's gate
    and up projections), fused into one launch forward."""
    return SwiGLUProjection.apply(x, (gate.packed, gate.quant_state), (up.packed, up.quant_state))


def grouped_projection(x, modules):
    """The outputs of several NF4Linear / NF4LoraLinear modules that read the same input x,
    computed by one grouped forward launch (up to 3 modules)."""
    specs, params = [], []
    for m in modules:
        if isinstance(m, NF4LoraLinear):
            specs.append((m.packed, m.quant_state, m.scaling, m.bias))
            params += [m.lora_A, m.lora_B]
        else:
            specs.append((m.packed, m.quant_state, None, m.bias))
    return GroupedNF4Function.apply(x, tuple(specs), *params)


def nf4_lora_linear(x, packed, st, lora_a, lora_b, scaling, bias=None):
    """Functional entry: the fused op inside its envelope (fp16 x, feature counts that are
    multiples of 64, a rank-16 adapter); outside it the base projection (MatMul4Bit, which
    warns when it is not fused either) plus the adapter in torch, as peft composes it, with a
    one-time warning."""
    if _supported(packed, st) and _fusable(x, st, lora_a, lora_b):
        return NF4LoraFunction.apply(x, packed, st, bias, lora_a, lora_b, scaling)
    from .nf4 import _warn_once, matmul_4bit
    _warn_once(f"lora:{x.dtype}:{tuple(lora_a.shape)}",
               f"adapter {tuple(lora_a.shape)} on {x.dtype} input is outside the fused envelope: "
               "base projection + torch adapter")
    y = matmul_4bit(x, packed.t(), st, bias=bias)
    return y + (x @ lora_a.to(x.dtype).t()) @ lora_b.to(x.dtype).t() * scaling


class NF4LoraLinear(torch.nn.Module):
    """A frozen NF4 Linear with a trainable rank-16 LoRA adapter (peft layout:
    lora_A.weight [16, in], lora_B.weight [out, 16], scaling = alpha / r)."""

    def __init__(self, packed, quant_state, lora_alpha: float = 32.0, bias=None,
                 lora_init: str = "kaiming", device=None):
        super().__init__()
        out_f, in_f = int(quant_state.shape[0]), int(quant_state.shape[1])
        self.register_buffer("packed", packed)
        self.quant_state = quant_state
        self.bias = bias
        self.scaling = lora_alpha / LORA_RANK
        dev = device or packed.device
        self.lora_A = torch.nn.Parameter(torch.empty(LORA_RANK, in_f, dtype=torch.float32, device=dev))
        self.lora_B = torch.nn.Parameter(torch.zeros(out_f, LORA_RANK, dtype=torch.float32, device=dev))
        torch.nn.init.kaiming_uniform_(self.lora_A, a=5 ** 0.5)
        self.in_features, self.out_features = in_f, out_f

    def forward(self, x):
        return nf4_lora_linear(x, self.packed, self.quant_state, self.lora_A, self.lora_B,
                               self.scaling, self.bias)


class NF4Linear(torch.nn.Module):
    """A frozen NF4 Linear without adapter (bitsandbytes Linear4bit.forward contract)."""

    def __init__(self, packed, quant_state, bias=None):
        super().__init__()
        self.register_buffer("packed", packed)
        self.quant_state = quant_state
        self.bias = bias
        self.out_features, self.in_features = int(quant_state.shape[0]), int(quant_state.shape[1])

    def forward(self, x):
        from .nf4 import matmul_4bit
        return matmul_4bit(x, self.packed.t(), self.quant_state, bias=self.bias)


def patch_peft_lora():
    """Route peft lora.Linear.forward through the fused op for adapters it fits: base layer a
    bitsandbytes Linear4bit NF4, one active adapter of rank 16, dropout 0 (or identity),
    not merged.  Everything else keeps peft's forward."""
    from peft.tuners.lora import layer as L

    cls = L.Linear
    orig = cls.forward
    if getattr(orig, "_stew_b200", False):
        return

    def forward(self, x, *args, **kwargs):
        try:
            base = self.get_base_layer()
            names = list(self.active_adapters)
        except Exception:  # noqa: BLE001
            return orig(self, x, *args, **kwargs)
        if (not args and not kwargs and len(names) == 1 and not getattr(self, "merged", False)
                and not getattr(self, "disable_adapters", False)):
            name = names[0]
            w = getattr(base, "weight", None)
            st = getattr(w, "quant_state", None)
            drop = self.lora_dropout[name] if name in self.lora_dropout else None
            p = getattr(drop, "p", 0.0)
            if (st is not None and self.r.get(name) == LORA_RANK and p == 0.0
                    and x.is_cuda and _supported(w, st) and x.dtype == torch.float16):
                la = self.lora_A[name].weight
                lb = self.lora_B[name].weight
                if _fusable(x, st, la, lb):
                    return NF4LoraFunction.apply(x, w.t(), st, getattr(base, "bias", None), la, lb,
                                                 self.scaling[name])
        return orig(self, x, *args, **kwargs)

    forward._stew_b200 = True
    cls.forward = forward

