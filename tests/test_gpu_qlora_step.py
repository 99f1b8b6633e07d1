"""GPU: the QLoRA step on the Qwen2.5-1.5B layer architecture (2 layers, small vocabulary)
against an fp32 torch reference of the same model whose projections use the
oracle-dequantised NF4 weights; and a few AdamW steps lower the loss.
Tolerances (written here): loss relative 5e-3; LoRA gradients max |g - ref| / max |ref| 5e-2
(fp16 activations between layers on both sides, fp32 accumulation order differs)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import nf4_oracle as O
from tests.helpers import to_oracle_state

pytestmark = pytest.mark.gpu


def _small_model(layers=2, vocab=4096):
    from stew_b200.qlora_step import QwenConfig, QwenQLoRA
    cfg = QwenConfig(layers=layers, vocab=vocab)
    return QwenQLoRA(cfg, device="cuda", seed=3)


def rms_norm(x, w, eps):
    """Qwen2 RMSNorm: fp32 statistics, normalised value rounded to fp16, then the weight."""
    xf = x.float()
    xn = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(torch.float16)
    return (w * xn.float()).to(torch.float16)


def apply_rope(x, cos, sin):
    """x [N, heads, d]; rotate-half convention of Qwen2, fp32 math."""
    xf = x.float()
    d = xf.shape[-1] // 2
    rot = torch.cat([-xf[..., d:], xf[..., :d]], dim=-1)
    return (xf * cos[:, None, :] + rot * sin[:, None, :]).to(x.dtype)


def _ref_loss(model, tokens, lengths):
    """fp32 reference forward with the oracle-dequantised weights: torch attention with a
    dense block-diagonal causal mask, torch RMSNorm / RoPE / SwiGLU."""
    from stew_b200.qlora_step import rope_tables
    cfg = model.cfg
    dev = tokens.device
    lens = lengths.tolist()
    T = tokens.shape[1]
    keep = torch.arange(T, device=dev)[None, :] < lengths[:, None]
    ids = tokens[keep]
    positions = torch.cat([torch.arange(L, device=dev) for L in lens])
    seg = torch.cat([torch.full((L,), i, device=dev) for i, L in enumerate(lens)])
    mask = (seg[:, None] == seg[None, :]) & (positions[None, :] <= positions[:, None])
    cos, sin = rope_tables(positions, cfg.head_dim, cfg.rope_theta)
    x = model.embed[ids]
    params = {}

    def lin(mod, h, name, li):
        W = torch.from_numpy(O.dequant_nf4(mod.packed.cpu().numpy(),
                                           to_oracle_state(mod.quant_state, mod.packed)).astype(np.float32)).cuda()
        y = h.float() @ W.t()
        if mod.bias is not None:
            y = y + mod.bias.float()
        if hasattr(mod, "lora_A"):
            a = mod.lora_A.detach().clone().requires_grad_(True)
            b = mod.lora_B.detach().clone().requires_grad_(True)
            params[(li, name)] = (a, b)
            y = y + (h.float() @ a.t()) @ b.t() * mod.scaling
        return y.to(torch.float16)

    n = x.shape[0]
    for li, layer in enumerate(model.layers):
        p = layer.proj
        h = rms_norm(x, layer.ln1, cfg.rms_eps)
        q = apply_rope(lin(p["q"], h, "q", li).view(n, cfg.heads, cfg.head_dim), cos, sin)
        k = apply_rope(lin(p["k"], h, "k", li).view(n, cfg.kv_heads, cfg.head_dim), cos, sin)
        v = lin(p["v"], h, "v", li).view(n, cfg.kv_heads, cfg.head_dim)
        a = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                           v.transpose(0, 1)[None], attn_mask=mask, enable_gqa=True)
        x = x + lin(p["o"], a[0].transpose(0, 1).reshape(n, -1), "o", li)
        h = rms_norm(x, layer.ln2, cfg.rms_eps)
        gg = lin(p["gate"], h, "gate", li).float()
        m = (gg * torch.sigmoid(gg) * lin(p["up"], h, "up", li).float()).to(torch.float16)
        x = x + lin(p["down"], m, "down", li)
    h = rms_norm(x, model.ln_f, cfg.rms_eps)
    nxt = torch.roll(ids, -1)
    has = torch.roll(seg, -1) == seg
    has[-1] = False
    logits = h[has] @ model.embed.t()
    return F.cross_entropy(logits.float(), nxt[has], reduction="sum"), int(has.sum()), params


def test_step_matches_fp32_reference(cuda_lib):
    from stew_b200.qlora_step import synthetic_batch
    model = _small_model()
    tokens, lengths = synthetic_batch(batch=2, seq=96, vocab=model.cfg.vocab, seed=1)
    loss, n = model(tokens, lengths)
    loss.backward()
    ref, n_ref, params = _ref_loss(model, tokens, lengths)
    ref.backward()
    assert n == n_ref
    assert abs(loss.item() - ref.item()) <= 5e-3 * abs(ref.item())
    for li, layer in enumerate(model.layers):
        for name in ("q", "v"):
            mod = layer.proj[name]
            a, b = params[(li, name)]
            for got, want in ((mod.lora_A.grad, a.grad), (mod.lora_B.grad, b.grad)):
                err = (got.double() - want.double()).abs().max() / want.double().abs().max()
                assert err <= 5e-2, (li, name, float(err))


def test_graphed_step_matches_eager_step(cuda_lib):
    """The CUDA-graph trainer (capture, warm-up undone, replay) takes the same optimizer
    steps as the eager one, including after a batch of another shape forces a re-capture.
    Two eager runs already differ slightly: the flash-attention backward sums dq with
    atomics, and Adam's first steps move an element by about +-lr whatever the size of its
    gradient, so a near-zero gradient whose sign differs flips that element.  Measured
    between two eager runs: relative L2 of the adapters <= 2e-2, elements apart by more
    than lr/2 <= 0.1 %.  Tolerances here: loss 1e-3 relative, adapters 5e-2 relative L2 and
    0.5 % of elements."""
    from stew_b200.qlora_step import QLoRATrainer, synthetic_batch
    eager_model, graph_model = _small_model(), _small_model()
    eager = QLoRATrainer(eager_model, lr=5e-3)
    graphed = QLoRATrainer(graph_model, lr=5e-3, cuda_graph=True)
    batches = [synthetic_batch(batch=2, seq=96, vocab=4096, seed=s) for s in (2, 2, 5, 2)]
    for tokens, lengths in batches:
        le, ne, _ = eager.step(tokens, lengths)
        lg, ng, _ = graphed.step(tokens, lengths)
        assert ne == ng
        assert abs(float(le) - float(lg)) <= 1e-3 * abs(float(le))
    for pe, pg in zip(eager.params, graphed.params):
        d = pe.detach().double() - pg.detach().double()
        assert float(d.norm() / pe.detach().double().norm()) <= 5e-2
        assert float((d.abs() > 2.5e-3).double().mean()) <= 5e-3
    graphed.release()


def test_bucketed_exchange_in_the_graph_matches_the_flat_path(cuda_lib):
    """The data-parallel step's bucketed LoRA-grad exchange -- post-accumulate-grad hooks, a side
    stream, one flat buffer per bucket, the normalisation after the backward -- captured in the
    step's CUDA graph, on one rank (no collective): the same labelled-token counts and the same
    optimizer steps as the flat path, to the run-to-run spread of the test above."""
    from stew_b200.qlora_step import QLoRATrainer, synthetic_batch
    flat_model, bucket_model = _small_model(), _small_model()
    flat = QLoRATrainer(flat_model, lr=5e-3, cuda_graph=True)
    bucketed = QLoRATrainer(bucket_model, lr=5e-3, cuda_graph=True, buckets=2, buckets_on_one_rank=True)
    assert bucketed.buckets == 2 and flat.buckets == 0
    for seed in (2, 2, 5):
        tokens, lengths = synthetic_batch(batch=2, seq=96, vocab=4096, seed=seed)
        lf, nf, _ = flat.step(tokens, lengths)
        lb, nb, _ = bucketed.step(tokens, lengths)
        assert nf == nb
        assert abs(float(lf) - float(lb)) <= 1e-3 * abs(float(lf))
    for pf, pb in zip(flat.params, bucketed.params):
        d = pf.detach().double() - pb.detach().double()
        assert float(d.norm() / pf.detach().double().norm()) <= 5e-2
        assert float((d.abs() > 2.5e-3).double().mean()) <= 5e-3
    flat.release()
    bucketed.release()


def test_training_steps_lower_the_loss(cuda_lib):
    from stew_b200.qlora_step import QLoRATrainer, synthetic_batch
    model = _small_model()
    trainer = QLoRATrainer(model, lr=5e-3)
    tokens, lengths = synthetic_batch(batch=2, seq=96, vocab=model.cfg.vocab, seed=2)
    losses = [float(trainer.step(tokens, lengths)[0]) for _ in range(4)]
    assert losses[-1] < losses[0]
    assert trainer.lora_grad_bytes() == 4 * (2 * (16 * 1536 + 1536 * 16 + 16 * 1536 + 256 * 16) + 1)


def test_adapter_fp16_shadow_follows_the_optimizer(cuda_lib):
    """The adapters are views of one fp32 buffer with one fp16 shadow; every forward refreshes
    the shadow, so the projections always see the current (optimizer-updated) adapters."""
    from stew_b200.qlora_step import QLoRATrainer, synthetic_batch
    model = _small_model()
    trainer = QLoRATrainer(model, lr=5e-3)
    tokens, lengths = synthetic_batch(batch=2, seq=96, vocab=model.cfg.vocab, seed=4)
    before = [p.detach().clone() for p in trainer.params]
    trainer.step(tokens, lengths)
    assert any(not torch.equal(b, p.detach()) for b, p in zip(before, trainer.params))
    model(tokens, lengths)
    for p in trainer.params:
        assert p.data_ptr() >= model._lora_flat.data_ptr()
        assert torch.equal(p._stew_half, p.detach().to(torch.float16))


def test_mlp_recompute_matches_kept_activations(cuda_lib):
    """The MLP memory cap (gate/up + SwiGLU recomputed in the backward for the first layers,
    the reference's solution/unpad.py:48-57 rule) changes no result: the same loss, and LoRA
    gradients equal up to the run-to-run spread of the flash-attention backward (relative L2
    <= 1e-2); and a graph trainer captures such a step too (the recompute is the MLP op's own
    gate/up launch, not torch's checkpoint), with the eager step's loss."""
    import dataclasses
    from stew_b200.qlora_step import QLoRATrainer, mlp_recompute_layers, synthetic_batch
    tokens, lengths = synthetic_batch(batch=2, seq=96, vocab=4096, seed=6)
    n = int(lengths.sum())
    kept, rec = _small_model(), _small_model()
    rec.cfg = dataclasses.replace(rec.cfg, mlp_token_budget=n // 2)
    assert mlp_recompute_layers(n, 2, n // 2) == 2
    l0, _ = kept(tokens, lengths)
    l1, _ = rec(tokens, lengths)
    l0.backward()
    l1.backward()
    assert float(l0) == float(l1)
    for pa, pb in zip(kept.lora_parameters(), rec.lora_parameters()):
        d = (pa.grad.double() - pb.grad.double()).norm() / pa.grad.double().norm()
        assert float(d) <= 1e-2
    # the eager losses keep their autograd graphs -- and the AccumulateGrad nodes, bound to the
    # stream they ran on -- alive; the graph trainer gets models those graphs never touched
    del l0, l1
    rec2, rec3 = _small_model(), _small_model()
    for m in (rec2, rec3):
        m.cfg = dataclasses.replace(m.cfg, mlp_token_budget=n // 2)
    eager = QLoRATrainer(rec2, lr=1e-3)
    tr = QLoRATrainer(rec3, lr=1e-3, cuda_graph=True)
    le, _, _ = eager.step(tokens, lengths)
    lg, _, _ = tr.step(tokens, lengths)
    assert tr._graph is not None, "the recompute step is captured"
    assert torch.isfinite(lg) and abs(float(lg) - float(le)) <= 1e-5 * abs(float(le))
    tr.release()
