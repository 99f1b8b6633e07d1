"""The full QLoRA training step the NF4 path serves: Qwen2.5-1.5B (28 layers, hidden 1536,
SwiGLU MLP 8960, 12 query / 2 key-value heads of dim 128, RMSNorm, RoPE theta 1e6, vocabulary
151936, tied fp16 embedding / LM head) with every projection an NF4 weight and a rank-16
LoRA adapter on q and v, run on packed token rows.

Scope: the reference patches this model (transformers' Qwen2 under peft/bitsandbytes) and runs
it on packed real tokens (solution/unpad.py:278-345).  The NF4 projections and the LoRA
adapters are this library's kernels (fused unpack + tcgen05 GEMMs, forward and backward), and
so are the layer's RMSNorm (fused with the residual add), RoPE and SwiGLU (step_ops, the
counterparts of solution/rmsnorm.py, rope.py, swiglu.py); attention is torch's variable-length
flash attention over the packed rows, and the tied LM head + cross-entropy are torch.  Weights
are random (seeded) and NF4-quantized on the GPU: no checkpoint is used.

`train_step` = forward on the packed rows, backward (LoRA grads only: base weights, norms and
embedding are frozen), one all-reduce of the LoRA grads across data-parallel ranks
(stew_b200.dp), AdamW on the adapters.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import dp
from .lora import LORA_RANK, NF4Linear, NF4LoraLinear, grouped_projection, nf4_mlp
from .step_ops import add_rms_norm, head_cross_entropy, rms_norm, rope_qk
from .sweep import QWEN_PROJ, qwen_model_weights


@dataclass
class QwenConfig:
    layers: int = 28
    hidden: int = 1536
    intermediate: int = 8960
    heads: int = 12
    kv_heads: int = 2
    head_dim: int = 128
    vocab: int = 151936
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    lora_alpha: float = 32.0
    # MLP memory cap (the reference's unpad path, solution/unpad.py:48-57): with more than this
    # many real tokens, the first layers keep only the MLP input and run their gate/up + SwiGLU
    # launch again in the backward.  None: never (a B200's 180 GB holds every layer's activations).
    mlp_token_budget: int | None = None


# Fraction of one layer's kept activations that belong to the MLP's gate/up/SwiGLU block,
# i.e. what a layer that recomputes that block in its backward stops keeping.
MLP_SAVED_SHARE = 0.63


def mlp_recompute_layers(n_tokens: int, layers: int, budget: int | None) -> int:
    """How many of `layers` layers recompute their MLP's gate/up for a batch of n real tokens
    so the activations kept stay within `budget` tokens' worth per layer at the peak (the
    reference's rule, solution/unpad.py:52-57)."""
    if budget is None or n_tokens <= budget:
        return 0
    return min(layers, math.ceil(layers * (n_tokens - budget) / (n_tokens * MLP_SAVED_SHARE)))


def rope_tables(positions: torch.Tensor, head_dim: int, theta: float):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=positions.device, dtype=torch.float32) / head_dim))
    ang = positions.float()[:, None] * inv[None, :]
    emb = torch.cat([ang, ang], dim=-1)
    return emb.cos(), emb.sin()


def packed_causal_attention(q, k, v, rows):
    """Causal attention inside each packed row: q [N, H, D], k/v [N, KH, D] (grouped-query
    heads, H a multiple of KH), rows = (cu_seqlens int32 [B+1], longest row).  The
    variable-length flash kernel sees only the real tokens, no [N, N] mask, and reads the
    shared k/v heads directly (no expanded copies, no head-sum in the backward)."""
    from torch.nn.attention.varlen import varlen_attn
    cu, longest = rows
    return varlen_attn(q, k, v, cu, cu, longest, longest, window_size=(-1, 0))


class Layer(torch.nn.Module):
    def __init__(self, cfg: QwenConfig, weights, device):
        super().__init__()
        self.cfg = cfg
        mods = {}
        for (name, _), (packed, st) in zip(QWEN_PROJ, weights):
            # Qwen2 has biases on q/k/v only (frozen, fp16)
            bias = ((torch.randn(int(st.shape[0]), device=device) * 0.02).to(torch.float16)
                    if name in ("q", "k", "v") else None)
            if name in ("q", "v"):
                m = NF4LoraLinear(packed, st, lora_alpha=cfg.lora_alpha, bias=bias, device=device)
                torch.nn.init.normal_(m.lora_B, std=0.01)
            else:
                m = NF4Linear(packed, st, bias=bias)
            mods[name] = m
        self.proj = torch.nn.ModuleDict(mods)
        self.register_buffer("ln1", torch.ones(cfg.hidden, device=device))
        self.register_buffer("ln2", torch.ones(cfg.hidden, device=device))

    def attention(self, h, cos, sin, rows):
        """o(attn(rope(q(h)), rope(k(h)), v(h))) for the normed input h [N, hidden]."""
        c, p = self.cfg, self.proj
        n = h.shape[0]
        q, k, v = grouped_projection(h, [p["q"], p["k"], p["v"]])  # one launch
        q, k = rope_qk(q.view(n, c.heads, c.head_dim), k.view(n, c.kv_heads, c.head_dim), cos, sin)
        v = v.view(n, c.kv_heads, c.head_dim)
        a = packed_causal_attention(q, k, v, rows)
        return p["o"](a.reshape(n, c.heads * c.head_dim))

    def mlp(self, h, recompute: bool = False):
        """down(SwiGLU(gate(h), up(h))) in two launches each way (lora.MLPFunction: the SwiGLU runs
        in the gate/up GEMM's epilogue forward and in down's dX epilogue backward); recompute:
        keep only h and run the gate/up launch again in the backward."""
        p = self.proj
        return nf4_mlp(h, p["gate"], p["up"], p["down"], recompute=recompute and torch.is_grad_enabled())


@dataclass
class PackedBatch:
    ids: torch.Tensor        # [N] token ids of the real tokens, row after row
    positions: torch.Tensor  # [N] position inside the row
    cu: torch.Tensor         # [B+1] int32 row starts (cumulative lengths)
    longest: int             # longest row
    lab_idx: torch.Tensor    # [M] packed index of every token that has a next-token label
    labels: torch.Tensor     # [M] the label (the next token of the same row)

    @property
    def n_labels(self) -> int:
        return int(self.lab_idx.numel())

    def shape_key(self):
        return (int(self.ids.numel()), int(self.cu.numel()), self.longest, self.n_labels)


class QwenQLoRA(torch.nn.Module):
    def __init__(self, cfg: QwenConfig = QwenConfig(), device="cuda", seed: int = 0, weights=None):
        super().__init__()
        self.cfg = cfg
        ws = weights if weights is not None else qwen_model_weights(layers=cfg.layers, device=device,
                                                                     seed=seed)
        g = torch.Generator(device=device).manual_seed(seed + 7)
        self.register_buffer("embed", (torch.randn(cfg.vocab, cfg.hidden, generator=g, device=device)
                                       * 0.02).to(torch.float16))
        torch.manual_seed(seed)
        self.layers = torch.nn.ModuleList(
            [Layer(cfg, ws[7 * i:7 * i + 7], device) for i in range(cfg.layers)])
        self.register_buffer("ln_f", torch.ones(cfg.hidden, device=device))
        # The adapters live in one fp32 buffer (each parameter a view of it) with an fp16
        # shadow of the same layout: one copy kernel per step gives every projection its fp16
        # A and B, instead of one conversion per matrix (112 launches a step).
        params = self.lora_parameters()
        total = sum(p.numel() for p in params)
        self._lora_flat = torch.empty(total, dtype=torch.float32, device=device)
        self._lora_half = torch.empty(total, dtype=torch.float16, device=device)
        off = 0
        for p in params:
            n = p.numel()
            self._lora_flat[off:off + n].copy_(p.detach().reshape(-1))
            p.data = self._lora_flat[off:off + n].view_as(p)
            p._stew_half = self._lora_half[off:off + n].view_as(p)
            off += n

    def lora_parameters(self):
        return [p for p in self.parameters() if p.requires_grad]

    def refresh_lora_half(self):
        """The fp16 shadow of the adapters from their current fp32 values."""
        self._lora_half.copy_(self._lora_flat)

    @staticmethod
    def pack(tokens: torch.Tensor, lengths: torch.Tensor) -> "PackedBatch":
        """Right-padded rows -> the packed real tokens and their metadata.  The row lengths are
        read on the host (a host tensor is used as is; a device one costs one read, as the
        reference's unpad path does), the index arrays are built there and sent in one copy,
        and the tokens are gathered with one index_select: no data-dependent device
        synchronisation, so the host can queue the next step while the GPU runs this one."""
        B, T = tokens.shape
        dev = tokens.device
        lens_t = lengths.detach().to("cpu", torch.int64) if lengths.is_cuda else lengths.to(torch.int64)
        lens = [int(v) for v in lens_t.tolist()]
        starts = [0]
        for L in lens:
            starts.append(starts[-1] + L)
        n = starts[-1]
        gather = torch.cat([torch.arange(L, dtype=torch.int64) + b * T for b, L in enumerate(lens)]
                           or [torch.zeros(0, dtype=torch.int64)])
        positions = torch.cat([torch.arange(L, dtype=torch.int64) for L in lens]
                              or [torch.zeros(0, dtype=torch.int64)])
        # next-token labels inside each row; a row's last token has none
        lab_idx = torch.cat([torch.arange(a, b - 1, dtype=torch.int64) for a, b in zip(starts[:-1], starts[1:])
                             if b - a > 1] or [torch.zeros(0, dtype=torch.int64)])
        m = int(lab_idx.numel())
        host = torch.cat([gather, positions, lab_idx, torch.tensor(starts, dtype=torch.int64)])
        dv = host.to(dev, non_blocking=True)
        gather_d, positions_d, lab_d = dv[:n], dv[n:2 * n], dv[2 * n:2 * n + m]
        cu = dv[2 * n + m:].to(torch.int32)
        ids = tokens.reshape(-1).index_select(0, gather_d)
        labels = ids.index_select(0, lab_d + 1)
        return PackedBatch(ids, positions_d, cu, max(lens) if lens else 0, lab_d, labels)

    def forward(self, tokens: torch.Tensor, lengths: torch.Tensor):
        """tokens [B, T] right-padded, lengths [B].  Returns (sum of next-token CE over the
        labelled tokens, number of labelled tokens)."""
        pb = self.pack(tokens, lengths)
        return self.forward_packed(pb), pb.n_labels

    def forward_packed(self, pb: "PackedBatch") -> torch.Tensor:
        """Sum of next-token CE over the labelled tokens of a packed batch.  Fixed shapes and
        no host synchronisation, so a step can be captured in a CUDA graph."""
        rows = (pb.cu, pb.longest)
        self.refresh_lora_half()
        cos, sin = rope_tables(pb.positions, self.cfg.head_dim, self.cfg.rope_theta)
        x = self.embed.index_select(0, pb.ids)
        eps = self.cfg.rms_eps
        h = rms_norm(x, self.layers[0].ln1, eps)
        n_rec = mlp_recompute_layers(int(pb.ids.numel()), len(self.layers), self.cfg.mlp_token_budget)
        for i, layer in enumerate(self.layers):
            # residual adds fused into the following norm: x += attn; h = norm(x); x += mlp; h = ...
            x, h = add_rms_norm(x, layer.attention(h, cos, sin, rows), layer.ln2, eps)
            nxt = self.layers[i + 1].ln1 if i + 1 < len(self.layers) else self.ln_f
            x, h = add_rms_norm(x, layer.mlp(h, recompute=i < n_rec), nxt, eps)
        # LM head + summed next-token CE, fused (the reference's solution/head_loss.py)
        return head_cross_entropy(h.index_select(0, pb.lab_idx), self.embed, pb.labels)


def synthetic_batch(batch: int = 4, seq: int = 512, vocab: int = 151936, mean_frac: float = 0.57,
                    seed: int = 0, device="cuda", total: int | None = None):
    """4 right-padded rows of 512 with uniform-random real lengths averaging 57% of the row
    (about 1170 real tokens), token ids uniform over the vocabulary.  `total`: the drawn
    lengths are then shifted, row by row and within [lo, seq], until they sum to exactly
    `total` real tokens (so every data-parallel rank can get the same amount of work)."""
    g = torch.Generator().manual_seed(seed)
    lo, hi = int(seq * (2 * mean_frac - 1.0)), seq
    lengths = torch.randint(lo, hi + 1, (batch,), generator=g)
    if total is not None:
        if not batch * lo <= total <= batch * hi:
            raise ValueError(f"total {total} outside [{batch * lo}, {batch * hi}]")
        lens = [int(v) for v in lengths]
        while sum(lens) != total:
            diff = total - sum(lens)
            step = 1 if diff > 0 else -1
            share = max(1, abs(diff) // batch)
            for i in range(batch):
                room = (hi - lens[i]) if step > 0 else (lens[i] - lo)
                d = min(share, room, abs(total - sum(lens)))
                lens[i] += step * d
        lengths = torch.tensor(lens, dtype=lengths.dtype)
    tokens = torch.randint(0, vocab, (batch, seq), generator=g)
    tokens[torch.arange(seq)[None, :] >= lengths[:, None]] = 0
    return tokens.to(device), lengths.to(device)


class QLoRATrainer:
    """One QLoRA step per call: forward, backward, LoRA-grad all-reduce, AdamW.

    cuda_graph=True captures the whole step (forward, backward, the all-reduce and AdamW) in
    one CUDA graph per packed-batch shape and replays it: the step's ~3,000 kernel launches
    cost one graph launch on the host.  The packed batch is copied into the graph's static
    input buffers each step; a new shape (token count, rows, longest row, labels) re-captures.
    The capture's warm-up steps are undone (adapters and optimizer state restored), so every
    call is exactly one optimizer step."""

    def __init__(self, model: QwenQLoRA, lr: float = 2e-4, group=None, cuda_graph: bool = False,
                 buckets: int = 4, buckets_on_one_rank: bool = False):
        self.model = model
        self.params = model.lora_parameters()
        self.cuda_graph = cuda_graph
        # data parallel: the LoRA-grad all-reduce in `buckets` groups of layers, each launched
        # from the backward as soon as its layers' gradients are complete (dp.BucketedGradAllReduce);
        # buckets_on_one_rank runs that machinery (hooks, side stream, normalisation) with no
        # collective on a single rank
        self._reducer = None
        if buckets > 0 and (dp._world(group) > 1 or buckets_on_one_rank):
            layer_params = [[p for p in layer.parameters() if p.requires_grad] for layer in model.layers]
            self._reducer = dp.BucketedGradAllReduce(layer_params, group, n_buckets=buckets)
        self.buckets = len(self._reducer) if self._reducer is not None else 0
        # fused: one kernel for all adapters (the multi-tensor form was ~0.9 ms per step)
        self.opt = torch.optim.AdamW(self.params, lr=lr, weight_decay=0.0, capturable=cuda_graph,
                                     fused=True)
        self.group = group
        self._graph = None
        self._key = None
        # one side stream for every capture's warm-up: per-stream state keyed by the stream
        # (the GEMMs' split-K workspace) is then created once, not once per re-capture
        self._side = None

    def _eager(self, pb):
        loss_sum = self.model.forward_packed(pb)
        if self._reducer is not None:
            self._reducer.count = torch.full((1,), float(pb.n_labels), device=pb.ids.device)
            loss_sum.backward()
            total = float(self._reducer.finish())
        else:
            loss_sum.backward()
            total = dp.allreduce_lora_grads(self.params, pb.n_labels, self.group)
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return loss_sum.detach(), total

    def _graph_body(self):
        loss = self.model.forward_packed(self._pb)
        if self._reducer is not None:
            self._reducer.count = self._n_lab
        loss.backward()
        # keep no reference to this autograd graph: a later capture must not reuse its nodes
        self._loss = loss.detach()
        if self._reducer is not None:
            self._total = self._reducer.finish()
        else:
            self._total = dp.allreduce_lora_grads_device(self.params, self._n_lab, self.group)
        self.opt.step()

    def _capture(self, pb):
        dev = pb.ids.device
        self._graph = None
        self._pb = PackedBatch(pb.ids.clone(), pb.positions.clone(), pb.cu.clone(), pb.longest,
                               pb.lab_idx.clone(), pb.labels.clone())
        self._n_lab = torch.full((1,), float(pb.n_labels), device=dev)
        saved_p = [p.detach().clone() for p in self.params]
        saved_s = {p: {k: v.clone() for k, v in st.items() if torch.is_tensor(v)}
                   for p, st in self.opt.state.items()}
        if self._side is None:
            self._side = torch.cuda.Stream(dev)
        side = self._side
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):  # lazy state (optimizer moments, library handles) before capture
                self.opt.zero_grad(set_to_none=True)
                self._graph_body()
        torch.cuda.current_stream(dev).wait_stream(side)
        # undo the warm-up steps: adapters and optimizer state as before them (state that the
        # warm-up created starts from zero, as a fresh optimizer's would)
        with torch.no_grad():
            for p, sp in zip(self.params, saved_p):
                p.copy_(sp)
            for p, st in self.opt.state.items():
                old = saved_s.get(p, {})
                for k, v in st.items():
                    if torch.is_tensor(v):
                        if k in old:
                            v.copy_(old[k])
                        else:
                            v.zero_()
        self.opt.zero_grad(set_to_none=True)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._graph_body()
        self._graph = g
        self._key = pb.shape_key()

    def step(self, tokens, lengths):
        """Returns (mean loss of this rank's labelled tokens as a 0-d device tensor,
        labelled tokens of this rank, labelled tokens over all ranks).  Steps whose MLP memory
        cap recomputes activations are captured as well (the recompute is the MLP op's own
        launch, not torch's checkpoint)."""
        pb = self.model.pack(tokens, lengths)
        n_lab = pb.n_labels
        if not self.cuda_graph:
            loss_sum, total = self._eager(pb)
            return loss_sum / max(n_lab, 1), n_lab, total
        if self._graph is None or self._key != pb.shape_key():
            self._capture(pb)
        for dst, src in ((self._pb.ids, pb.ids), (self._pb.positions, pb.positions), (self._pb.cu, pb.cu),
                         (self._pb.lab_idx, pb.lab_idx), (self._pb.labels, pb.labels)):
            dst.copy_(src)
        self._graph.replay()
        return self._loss.detach() / max(n_lab, 1), n_lab, self._total

    def release(self):
        """Drop the captured graph (it holds NCCL work: release before destroying the group)."""
        self._graph = None
        self._pb = None

    def lora_grad_bytes(self) -> int:
        return dp.lora_grad_bytes(self.params)


def step_flops(cfg: QwenConfig, n_tokens: int) -> dict:
    """Algorithmic FLOPs of the NF4 projections in one step (forward + input-gradient
    backward) plus the LoRA terms on q/v."""
    nf4 = 0
    lora = 0
    for name, (out_f, in_f) in QWEN_PROJ:
        nf4 += 2 * 2 * n_tokens * in_f * out_f  # forward + backward dX
        if name in ("q", "v"):
            lora += 6 * n_tokens * LORA_RANK * (in_f + out_f)
    return {"nf4_gemm": nf4 * cfg.layers, "lora": lora * cfg.layers}
