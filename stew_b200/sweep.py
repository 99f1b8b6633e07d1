"""Whole-model NF4 unpack sweep: every packed projection of the model unpacked in ONE
launch (C ABI nf4b_dequant_plan + nf4b_dequant_batched).

The reference unpacks each of the 7 projections x 28 layers separately, forward and
backward (196 `_nf4_unpack` launches per direction per step, tools/bench_nf4.py:47);
on a B200 a k/v projection (0.39 M weights, ~0.6 us of HBM time) is far shorter than a
kernel launch, so the sweep is planned once and issued as one grid.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .nf4 import _qstate, _stream, _supported
from .quant_state import quantize_4bit

# Qwen2.5-1.5B projection shapes [out, in] (config: hidden 1536, MLP 8960, 12 q / 2 kv heads
# of dim 128): q, k, v, o, gate, up, down.
QWEN_PROJ = (("q", (1536, 1536)), ("k", (256, 1536)), ("v", (256, 1536)), ("o", (1536, 1536)),
             ("gate", (8960, 1536)), ("up", (8960, 1536)), ("down", (1536, 8960)))


@torch.no_grad()
def qwen_model_weights(layers: int = 28, device="cuda", seed: int = 0, blocksize: int = 64,
                       nested: bool = True, projections=QWEN_PROJ):
    """Seeded synthetic NF4 weights of the Qwen2.5-1.5B decoder: for layer l and
    projection p the fp16 weight is N(0, 0.02) from seed 1000*l + p (+ seed), quantized
    with blocksize 64 and double quantization.  Returns [(packed, QuantState)] in
    layer-major order."""
    out = []
    for layer in range(layers):
        for p, (_, shape) in enumerate(projections):
            g = torch.Generator(device=device).manual_seed(seed + 1000 * layer + p)
            w = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * 0.02
            out.append(quantize_4bit(w.to(torch.float16), blocksize=blocksize,
                                     compress_statistics=nested))
            del w
    return out


class DequantSweep:
    """Unpacks a fixed list of (packed, quant_state) in one launch into preallocated outputs."""

    def __init__(self, weights, outputs=None):
        if not weights:
            raise ValueError("empty sweep")
        self.weights = list(weights)
        dev = self.weights[0][0].device
        self.device = dev
        if outputs is None:
            outputs = [torch.empty(st.shape, dtype=st.dtype, device=dev) for _, st in self.weights]
        self.outputs = outputs
        n = len(self.weights)
        jobs = (_lib.DequantJobC * n)()
        L = _lib.lib()
        with torch.cuda.device(dev):
            for i, ((q, st), o) in enumerate(zip(self.weights, self.outputs)):
                if not _supported(q, st):
                    raise ValueError(f"weight {i} outside the NF4 envelope")
                jobs[i].packed = q.data_ptr()
                jobs[i].out = o.data_ptr()
                jobs[i].qs = _qstate(st, dev)
                jobs[i].numel = o.numel()
                jobs[i].out_dtype = _lib.NF4B_F16 if st.dtype == torch.float16 else _lib.NF4B_F32
            nbytes = int(L.nf4b_dequant_plan_bytes(n))
            self.plan = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            ctas = ctypes.c_int64(0)
            _lib.check(L.nf4b_dequant_plan(jobs, n, self.plan.data_ptr(), ctypes.byref(ctas),
                                           _stream(dev)), "nf4b_dequant_plan")
        self.n_jobs = n
        self.n_ctas = int(ctas.value)
        self.numel = sum(o.numel() for o in self.outputs)
        self.packed_bytes = sum(q.numel() for q, _ in self.weights)

    def run(self):
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().nf4b_dequant_batched(self.plan.data_ptr(), self.n_jobs, self.n_ctas,
                                                       _stream(self.device)), "nf4b_dequant_batched")
        return self.outputs

    def algorithmic_bytes(self) -> int:
        """Bytes the unpack must move: packed nibbles + absmax (8-bit or fp32) + second-level
        absmax in, values out."""
        total = 0
        for (q, st), o in zip(self.weights, self.outputs):
            total += q.numel() + st.absmax.numel() * st.absmax.element_size()
            if st.nested:
                total += st.state2.absmax.numel() * 4
            total += o.numel() * o.element_size()
        return total


class PipelinedSweep:
    """The sweep end to end from host memory: the weights in `chunks` groups of consecutive
    matrices, each group's packed bytes and scales copied host -> device on one stream, unpacked
    on a second (one batched launch per group) and its fp16 output copied device -> host on a
    third, so the two copy directions (separate copy engines) and the kernels overlap across
    groups instead of running one after the other.  Host buffers are pinned; every copy is one
    cudaMemcpyAsync per tensor."""

    def __init__(self, weights, host_inputs, host_outputs, chunks: int = 7):
        self.device = weights[0][0].device
        n = len(weights)
        per = (n + chunks - 1) // chunks
        self.groups = []
        for c in range(0, n, per):
            ws = weights[c:c + per]
            sweep = DequantSweep(ws)
            self.groups.append((sweep, host_inputs[c:c + per], host_outputs[c:c + per]))
        self.streams = [torch.cuda.Stream(self.device) for _ in range(3)]
        self.h2d_bytes = sum(h.numel() * h.element_size() for _, ins, _ in self.groups
                             for parts in ins for _, h in parts)
        self.d2h_bytes = sum(h.numel() * h.element_size() for _, _, outs in self.groups for h in outs)

    def run(self):
        main = torch.cuda.current_stream(self.device)
        up, work, down = self.streams
        for s in self.streams:
            s.wait_stream(main)
        for sweep, ins, outs in self.groups:
            with torch.cuda.stream(up):
                for parts in ins:
                    for dev_t, host_t in parts:
                        dev_t.copy_(host_t, non_blocking=True)
            work.wait_stream(up)
            with torch.cuda.stream(work):
                sweep.run()
            down.wait_stream(work)
            with torch.cuda.stream(down):
                for dev_t, host_t in zip(sweep.outputs, outs):
                    host_t.copy_(dev_t, non_blocking=True)
        for s in self.streams:
            main.wait_stream(s)

    def algorithmic_bytes(self) -> int:
        return sum(g[0].algorithmic_bytes() for g in self.groups)
