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

import math

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


class BucketedGradAllReduce:
    """The LoRA-gradient all-reduce in buckets of consecutive layers, each launched from the
    backward as soon as its gradients are complete -- layers finish in reverse order (27 ... 0),
    so the exchange of the later layers' bucket overlaps the backward of the earlier layers.

    Each bucket is one flat fp32 buffer (allocated once, so a CUDA graph replays the same
    memory); a post-accumulate-grad hook on every adapter parameter counts the bucket's
    gradients and, with the last one, copies them into the buffer and all-reduces it on a
    side stream (which waits for the backward's stream up to that point).  The bucket that
    completes last (the one holding layer 0) also carries this rank's labelled-token count.
    `finish()` joins the side stream, divides every gradient by the global count (the loss
    normalisation of solution/head_loss.py:164-169, taken over all ranks) and writes the
    results back into .grad -- the same values as allreduce_lora_grads_device.

    param_groups: the adapter parameters layer by layer (layer 0 first)."""

    def __init__(self, param_groups, group=None, n_buckets: int = 4):
        self.group = group
        groups = [list(g) for g in param_groups if len(g)]
        per = max(1, math.ceil(len(groups) / max(1, n_buckets)))
        self.buckets = [[p for g in groups[i:i + per] for p in g] for i in range(0, len(groups), per)]
        dev = self.buckets[0][0].device
        # layer 0's bucket is the last to complete: it carries the count
        self.flat = [torch.zeros(sum(p.numel() for p in b) + (1 if i == 0 else 0), dtype=torch.float32,
                                 device=dev) for i, b in enumerate(self.buckets)]
        self._where = {}
        for i, b in enumerate(self.buckets):
            for p in b:
                self._where[p] = i
        self._ready = [0] * len(self.buckets)
        self._launched = [False] * len(self.buckets)
        self.count = None
        self.stream = torch.cuda.Stream(dev) if dev.type == "cuda" else None
        self._handles = [p.register_post_accumulate_grad_hook(self._hook) for b in self.buckets for p in b]

    def __len__(self):
        return len(self.buckets)

    def _hook(self, p):
        i = self._where[p]
        if self._launched[i]:
            # the bucket was exchanged already: a second backward before finish() would
            # accumulate gradients that no all-reduce carries
            raise RuntimeError("BucketedGradAllReduce: a second backward before finish(); call finish() "
                               "after each backward")
        self._ready[i] += 1
        if self._ready[i] == len(self.buckets[i]):
            self._launch(i)

    def _launch(self, i):
        b, flat = self.buckets[i], self.flat[i]
        n = flat.numel() - (1 if i == 0 else 0)
        if self.stream is not None:
            self.stream.wait_stream(torch.cuda.current_stream(flat.device))
            ctx = torch.cuda.stream(self.stream)
        else:
            ctx = _NullCtx()
        with ctx:
            torch.cat([p.grad.reshape(-1).float() for p in b], out=flat[:n])
            if i == 0:
                if self.count is None:
                    raise RuntimeError("BucketedGradAllReduce: set .count before the backward")
                flat[n:].copy_(self.count.reshape(1))
            if _world(self.group) > 1:
                dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group)
        self._launched[i] = True

    def finish(self) -> torch.Tensor:
        """Join the exchange, normalise by the global labelled-token count, write the grads.
        Returns the global count (device tensor)."""
        for i, b in enumerate(self.buckets):  # a bucket whose grads never came: zeros
            if not self._launched[i]:
                for p in b:
                    if p.grad is None:
                        p.grad = torch.zeros_like(p)
                self._launch(i)
        if self.stream is not None:
            torch.cuda.current_stream(self.flat[0].device).wait_stream(self.stream)
        total = self.flat[0][-1:].clamp_min(1.0)
        grads, views = [], []
        for i, b in enumerate(self.buckets):
            n = self.flat[i].numel() - (1 if i == 0 else 0)
            body = self.flat[i][:n]
            body.div_(total)
            for p, v in zip(b, body.split([p.numel() for p in b])):
                grads.append(p.grad)
                views.append(v.view_as(p))
        torch._foreach_copy_(grads, views)
        self._ready = [0] * len(self.buckets)
        self._launched = [False] * len(self.buckets)
        return total

    def remove(self):
        for h in self._handles:
            h.remove()
        self._handles = []


class _NullCtx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


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
