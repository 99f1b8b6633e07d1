"""Data parallelism of the QLoRA step: one process per GPU, each with a full replica of the
packed NF4 weights and the LoRA adapters, each running its own batch of packed token rows.
The only exchange is ONE all-reduce per step of a flat fp32 buffer holding every LoRA
gradient plus the rank's labelled-token count, after which the gradients are divided by the
global count -- the loss normalisation of the reference's head loss (sum of per-token CE
over the batch divided by the number of labelled tokens, solution/head_loss.py:164-169),
taken over all ranks' batches.

With a process group of size 1 (or no group) the same code runs without communication, so a
G-rank step equals a 1-rank step over the concatenated batches.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _world(group) -> int:
    if not (dist.is_available() and dist.is_initialized()):
        return 1
    return dist.get_world_size(group)


def flatten_grads(params, extra: float) -> torch.Tensor:
    """One fp32 buffer: every parameter's gradient (zeros where it has none), then `extra`."""
    parts = []
    dev = None
    for p in params:
        dev = p.device
        g = p.grad if p.grad is not None else torch.zeros_like(p)
        parts.append(g.reshape(-1).float())
    parts.append(torch.tensor([float(extra)], dtype=torch.float32, device=dev))
    return torch.cat(parts)


def unflatten_into_grads(params, flat: torch.Tensor) -> None:
    off = 0
    for p in params:
        n = p.numel()
        g = flat[off:off + n].view_as(p).to(p.dtype)
        if p.grad is None:
            p.grad = g.clone()
        else:
            p.grad.copy_(g)
        off += n


def allreduce_lora_grads(params, local_labels: float, group=None) -> float:
    """Sum the LoRA gradients and the labelled-token counts over the ranks in one
    all-reduce, then divide the gradients by the global count.  The gradients on entry
    are of the rank's summed (not averaged) loss.  Returns the global count."""
    params = list(params)
    flat = flatten_grads(params, local_labels)
    if _world(group) > 1:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    total = float(flat[-1].item())
    if total <= 0:
        total = 1.0
    unflatten_into_grads(params, flat[:-1] / total)
    return total


def allreduce_lora_grads_device(params, local_labels: torch.Tensor, group=None) -> torch.Tensor:
    """allreduce_lora_grads with the count as a device tensor and no host synchronisation,
    so the exchange can be captured in a CUDA graph.  Returns the global count (device).

    The gradients are gathered into the flat buffer with one concatenation and written back
    and normalised with multi-tensor (foreach) kernels, so the step's ~100 adapter tensors
    cost a handful of launches instead of one copy each; a single rank skips the buffer and
    only divides."""
    params = list(params)
    for p in params:
        if p.grad is None:
            p.grad = torch.zeros_like(p)
    grads = [p.grad for p in params]
    count = local_labels.reshape(1).float()
    if _world(group) > 1:
        flat = torch.cat([g.reshape(-1).float() for g in grads] + [count])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        total = flat[-1:].clamp_min(1.0)
        body = flat[:-1]
        body.div_(total)
        sizes = [g.numel() for g in grads]
        torch._foreach_copy_(grads, [v.view_as(g) for v, g in zip(body.split(sizes), grads)])
        return total
    total = count.clamp_min(1.0)
    torch._foreach_div_(grads, total.reshape(()))
    return total


def balanced_shards(lengths, world: int, rows_per_rank: int):
    """Length-balanced assignment of a global batch of `world * rows_per_rank` rows to the
    ranks, `rows_per_rank` rows each: rows are dealt longest first to the rank with the fewest
    tokens that still has room (greedy longest-processing-time).  A data-parallel step ends
    with the slowest rank, so dealing rows by length instead of in order keeps the ranks'
    token counts close (the per-rank spread is at most one row's length).  The gradients do
    not depend on the assignment: they are summed over all rows and divided by the global
    labelled-token count.  Returns the row indices of each rank, in ascending order."""
    lengths = [int(v) for v in lengths]
    assert len(lengths) == world * rows_per_rank, "global batch must have world * rows_per_rank rows"
    order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
    load = [0] * world
    shards = [[] for _ in range(world)]
    for i in order:
        r = min((k for k in range(world) if len(shards[k]) < rows_per_rank), key=lambda k: (load[k], k))
        shards[r].append(i)
        load[r] += lengths[i]
    return [sorted(s) for s in shards]


def lora_grad_bytes(params) -> int:
    return 4 * (sum(p.numel() for p in params) + 1)
