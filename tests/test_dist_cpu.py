"""Data-parallel host logic on CPU ranks (gloo, world size 2): per-layer
buckets of the flat gradient buffer are all-reduced as their `grad ready`
hooks fire (in reverse layer order, head last), blocks whose hook never fired
are reduced by finish(), and every rank ends with the average."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class FakeModel:
    def __init__(self, rank, n_layers=3, per=5, head=4):
        self.flat_grads = torch.zeros(head + n_layers * per)
        self.layer_offsets = [(head + l * per, head + (l + 1) * per) for l in range(n_layers)]
        for i in range(self.flat_grads.numel()):
            self.flat_grads[i] = float((rank + 1) * (i + 1))
        self.grad_ready_hook = None


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                        "forge-llm_b200"))
        from forgellm.dist import DataParallel, shard_rows
        m = FakeModel(rank)
        dp = DataParallel(m)
        assert m.grad_ready_hook is not None
        m.grad_ready_hook(2)          # backward reaches the last layer first
        m.grad_ready_hook(1)
        m.grad_ready_hook(1)          # a repeated hook is ignored
        dp.finish()                   # layer 0 and head were never signalled
        want = [sum((r + 1) * (i + 1) for r in range(world)) / world
                for i in range(m.flat_grads.numel())]
        ok = torch.allclose(m.flat_grads, torch.tensor(want))
        rows = shard_rows(torch.arange(8 * 3).reshape(8, 3), rank, world)
        ok = ok and rows.shape == (4, 3) and int(rows[0, 0]) == rank * 12
        dp.detach()
        ok = ok and m.grad_ready_hook is None
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_bucketed_allreduce_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)


def test_shard_rows_rejects_uneven_split():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "forge-llm_b200"))
    from forgellm.dist import shard_rows
    with pytest.raises(ValueError):
        shard_rows(torch.zeros(6, 2), 0, 4)


def _worker_shard(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                        "forge-llm_b200"))
        from forgellm.dist import DataParallel
        m = FakeModel(rank, n_layers=3, per=6, head=4)
        dp = DataParallel(m, shard=True)
        sl = dp.slices()
        ok = sl == [(rank * 2, rank * 2 + 2)] + [(4 + l * 6 + rank * 3, 4 + l * 6 + rank * 3 + 3) for l in range(3)]
        m.grad_ready_hook(2)
        dp.finish()
        want = torch.tensor([sum((r + 1) * (i + 1) for r in range(world)) / world
                             for i in range(m.flat_grads.numel())])
        ok = ok and all(torch.allclose(m.flat_grads[a:b], want[a:b]) for a, b in sl)
        try:
            DataParallel(FakeModel(rank, n_layers=1, per=5, head=4), shard=True)
            ok = False                  # a bucket of 5 cannot split over 2 ranks
        except ValueError:
            pass
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_sharded_slices_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_shard, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
