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
