"""CPU, 2 gloo ranks: the data-parallel LoRA-gradient exchange of the QLoRA step
(stew_b200.dp) -- G ranks x their own rows give the same normalised gradients as one rank
over all rows; and a rank that fails before the all-reduce makes the other rank's
collective end with an error within the process-group timeout instead of hanging."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from stew_b200 import dp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class TinyLoRA(torch.nn.Module):
    """A frozen base projection with a rank-4 adapter and a per-token CE head: enough
    structure for summed-loss / global-count normalisation to matter."""

    def __init__(self):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        self.register_buffer("w", torch.randn(24, 16, generator=g) * 0.2)
        self.a = torch.nn.Parameter(torch.randn(4, 16, generator=g) * 0.3)
        self.b = torch.nn.Parameter(torch.randn(24, 4, generator=g) * 0.3)

    def forward(self, x, labels):
        y = x @ self.w.t() + (x @ self.a.t()) @ self.b.t() * 2.0
        keep = labels >= 0
        return torch.nn.functional.cross_entropy(y[keep], labels[keep], reduction="sum"), int(keep.sum())


def _rows(seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(13 + seed, 16, generator=g)
    labels = torch.randint(0, 24, (13 + seed,), generator=g)
    labels[::5] = -100
    return x, labels


def _worker(rank, world, port, q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the all-reduce")
        m = TinyLoRA()
        loss, n = m(*_rows(rank))
        loss.backward()
        # the graph-capturable form (count as a tensor, no host sync) on a copy of the grads
        m2 = TinyLoRA()
        m2.a.grad, m2.b.grad = m.a.grad.clone(), m.b.grad.clone()
        total_dev = dp.allreduce_lora_grads_device([m2.a, m2.b], torch.tensor(float(n)))
        total = dp.allreduce_lora_grads([m.a, m.b], n)
        assert float(total_dev) == total
        assert torch.equal(m2.a.grad, m.a.grad) and torch.equal(m2.b.grad, m.b.grad)
        q.put((rank, "ok", total, m.a.grad.clone(), m.b.grad.clone()))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), None, None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, status, a, ga, gb = q.get(timeout=120)
        out[r] = (status, a, ga, gb)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_two_ranks_equal_one_rank_over_all_rows():
    out = _run(2)
    m = TinyLoRA()
    loss0, n0 = m(*_rows(0))
    loss1, n1 = m(*_rows(1))
    ((loss0 + loss1) / (n0 + n1)).backward()
    for r in (0, 1):
        status, total, ga, gb = out[r]
        assert status == "ok"
        assert total == n0 + n1
        torch.testing.assert_close(ga, m.a.grad, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(gb, m.b.grad, rtol=1e-5, atol=1e-6)


def test_single_process_needs_no_group():
    m = TinyLoRA()
    loss, n = m(*_rows(3))
    loss.backward()
    ga = m.a.grad.clone()
    gb = m.b.grad.clone()
    total = dp.allreduce_lora_grads([m.a, m.b], n)
    assert total == n
    torch.testing.assert_close(m.a.grad, ga / n)
    # the capturable form divides in place without the flat buffer when there is no group
    m.a.grad, m.b.grad = ga.clone(), gb.clone()
    total_dev = dp.allreduce_lora_grads_device([m.a, m.b], torch.tensor(float(n)))
    assert float(total_dev) == n
    assert torch.equal(m.a.grad, ga / n) and torch.equal(m.b.grad, gb / n)


@pytest.mark.timeout(180)
def test_failed_rank_ends_peer_collective_with_error():
    out = _run(2, fail_rank=1)
    assert out[1][0] == "error" and "injected failure" in out[1][1]
    assert out[0][0] == "error", "the surviving rank must not hang or succeed"


def test_balanced_shards_partition_and_spread():
    """Every row goes to exactly one rank, each rank gets its rows_per_rank rows, and the
    ranks' token counts differ by at most the longest row (greedy longest-first bound)."""
    import random
    rng = random.Random(0)
    for world in (1, 2, 4, 8):
        lengths = [rng.randint(58, 512) for _ in range(4 * world)]
        shards = dp.balanced_shards(lengths, world, 4)
        assert sorted(i for s in shards for i in s) == list(range(4 * world))
        assert all(len(s) == 4 for s in shards)
        loads = [sum(lengths[i] for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(lengths)
    # the bench's 4-rank global batch: in-order shards spread 787..1585 tokens
    lengths = [442, 232, 206, 431, 78, 276, 360, 425, 410, 508, 198, 469, 110, 400, 138, 139]
    loads = [sum(lengths[i] for i in s) for s in dp.balanced_shards(lengths, 4, 4)]
    assert max(loads) - min(loads) <= 60


def test_mlp_recompute_layer_count_follows_the_reference_rule():
    """min(layers, ceil(layers * (n - budget) / (n * 0.63))) above the budget, 0 at or below it
    (solution/unpad.py:52-57); no budget never recomputes."""
    from stew_b200.qlora_step import mlp_recompute_layers
    assert mlp_recompute_layers(1000, 28, 1000) == 0
    assert mlp_recompute_layers(1170, 28, 1000) == 7      # ceil(28 * 170 / 737.1) = ceil(6.46)
    assert mlp_recompute_layers(2048, 28, 1000) == 23     # ceil(28 * 1048 / 1290.24) = ceil(22.7)
    assert mlp_recompute_layers(100000, 28, 1000) == 28
    assert mlp_recompute_layers(5000, 28, None) == 0


class LayeredLoRA(torch.nn.Module):
    """Five 'layers', each a frozen projection with a rank-4 adapter, applied in sequence:
    their gradients complete in reverse layer order, as in the QLoRA step's backward."""

    def __init__(self):
        super().__init__()
        g = torch.Generator().manual_seed(1)
        self.w = [torch.randn(16, 16, generator=g) * 0.3 for _ in range(5)]
        self.a = torch.nn.ParameterList([torch.nn.Parameter(torch.randn(4, 16, generator=g) * 0.3)
                                         for _ in range(5)])
        self.b = torch.nn.ParameterList([torch.nn.Parameter(torch.randn(16, 4, generator=g) * 0.3)
                                         for _ in range(5)])
        self.head = torch.randn(24, 16, generator=g) * 0.3

    def layer_params(self):
        return [[self.a[i], self.b[i]] for i in range(5)]

    def forward(self, x, labels):
        for w, a, b in zip(self.w, self.a, self.b):
            x = torch.tanh(x @ w.t() + (x @ a.t()) @ b.t() * 2.0)
        y = x @ self.head.t()
        keep = labels >= 0
        return torch.nn.functional.cross_entropy(y[keep], labels[keep], reduction="sum"), int(keep.sum())


def _bucket_worker(rank, world, port, q, n_buckets):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        x, labels = _rows(rank)
        m = LayeredLoRA()
        red = dp.BucketedGradAllReduce(m.layer_params(), n_buckets=n_buckets)
        res = []
        for step in range(2):  # the hooks re-arm after finish(): a second step is exchanged too
            for p in m.parameters():
                p.grad = None
            loss, n = m(x * (1 + step), labels)
            red.count = torch.tensor([float(n)])
            loss.backward()
            total = red.finish()
            ref = LayeredLoRA()
            lr, nr = ref(x * (1 + step), labels)
            lr.backward()
            flat_total = dp.allreduce_lora_grads(list(ref.parameters()), nr)
            assert float(total) == flat_total
            for p, r in zip(m.parameters(), ref.parameters()):
                assert torch.equal(p.grad, r.grad), "bucketed != one flat all-reduce"
            res.append(float(total))
        red.remove()
        q.put((rank, "ok", res, len(red.buckets), None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), None, None))
    finally:
        dist.destroy_process_group()


def test_bucketed_allreduce_refuses_a_second_backward_before_finish():
    """Buckets are exchanged as the backward completes them; a second backward before finish()
    would add gradients that no exchange carries, so it raises (single process, no group)."""
    x, labels = _rows(0)
    m = LayeredLoRA()
    red = dp.BucketedGradAllReduce(m.layer_params(), n_buckets=2)
    loss, n = m(x, labels)
    red.count = torch.tensor([float(n)])
    loss.backward()
    loss2, _ = m(x, labels)
    with pytest.raises(RuntimeError, match="second backward before finish"):
        loss2.backward()
    red.remove()


@pytest.mark.parametrize("n_buckets", [1, 2, 5])
def test_bucketed_allreduce_equals_one_flat_allreduce(n_buckets):
    """dp.BucketedGradAllReduce (buckets launched from post-accumulate-grad hooks as the
    backward completes them, layer 4 ... 0) gives bit-identical gradients and the same global
    count as one flat all-reduce after the backward, on 2 gloo ranks, for two steps."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bucket_worker, args=(r, 2, port, q, n_buckets)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        r, status, res, nb, _ = q.get(timeout=120)
        out[r] = (status, res, nb)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in (0, 1):
        assert out[r][0] == "ok", out[r]
        assert out[r][2] == min(n_buckets, 5)
    assert out[0][1] == out[1][1]
