"""The data-parallel exchange on one GPU.

- A one-rank NCCL communicator driven entirely through the C-ABI
  (fcu_comm_unique_id, fcu_comm_init, fcu_allreduce_grads,
  fcu_reduce_scatter_grads, fcu_allgather_params, fcu_allreduce_sum_f64,
  fcu_comm_join, fcu_comm_poll, fcu_comm_destroy): every collective of one
  rank is the identity, ordered after the kernels queued before it and before
  those queued after the join, eagerly and replayed from a CUDA graph.
- ZeRO-1 (DataParallel(shard=True) + ShardedAdam) against replicated Adam with
  two ranks that share one GPU and exchange through the host (gloo): the
  sharded update kernels (per-slice Adam with the global gradient norm) give
  the replicated step's parameters on every rank.  The NCCL transport itself
  is covered by the one-rank test above and, on 2 GPUs, by test_gpu_dp.py.
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _comm1():
    from forgellm import _lib
    uid = C.create_string_buffer(_lib.FCU_COMM_ID_BYTES)
    _lib.call("fcu_comm_unique_id", uid)
    h = C.c_void_p()
    _lib.call("fcu_comm_init", torch.cuda.current_device(), uid, 1, 0, 60.0, C.byref(h))
    return h


def test_one_rank_communicator_through_the_c_abi():
    from forgellm import _lib
    from forgellm.autograd import ctx
    L = _lib.lib()
    h = ctx().handle
    comm = _comm1()
    try:
        n, r, d = C.c_int(), C.c_int(), C.c_int()
        _lib.call("fcu_comm_info", comm, C.byref(n), C.byref(r), C.byref(d))
        assert (n.value, r.value, d.value) == (1, 0, torch.cuda.current_device())
        g = torch.Generator(device="cuda").manual_seed(1)
        x = torch.randn(1 << 20, device="cuda", generator=g)
        want = x * 3.0
        # scale then average: the collective must see the scaled values
        _lib.call("fcu_scale", h, x.data_ptr(), x.numel(), C.c_float(3.0))
        _lib.call("fcu_allreduce_grads", h, comm, x.data_ptr(), x.numel())
        _lib.call("fcu_reduce_scatter_grads", h, comm, x.data_ptr(), x.numel())
        _lib.call("fcu_allgather_params", h, comm, x.data_ptr(), x.numel(), 4)
        xb = want.to(torch.bfloat16)
        _lib.call("fcu_allgather_params", h, comm, xb.data_ptr(), xb.numel(), 2)
        s = torch.tensor([2.5, -1.0], dtype=torch.float64, device="cuda")
        _lib.call("fcu_allreduce_sum_f64", h, comm, s.data_ptr(), 2)
        _lib.call("fcu_comm_join", h, comm)
        y = x * 0.5            # queued after the join on the same stream
        _lib.call("fcu_comm_poll", comm, 60.0)
        torch.cuda.synchronize()
        assert torch.equal(x, want)
        assert torch.equal(y, want * 0.5)
        assert torch.equal(xb, want.to(torch.bfloat16))
        assert s.tolist() == [2.5, -1.0]
        assert L.fcu_check_device_error(h) == 0
        # misuse is rejected before NCCL is called
        assert L.fcu_allgather_params(h, comm, x.data_ptr(), x.numel(), 3) == _lib.FCU_ERR_ARG
    finally:
        _lib.call("fcu_comm_destroy", comm)


def test_one_rank_collectives_replay_from_a_cuda_graph():
    from forgellm import _lib
    from forgellm.autograd import ctx
    comm = _comm1()
    try:
        x = torch.ones(4096, device="cuda")
        s = torch.zeros(1, dtype=torch.float64, device="cuda")
        # one eager call first: the context's scratch (fcu_sumsq's partials) is
        # allocated on first use, which stream capture does not allow
        _lib.call("fcu_sumsq", ctx().handle, x.data_ptr(), x.numel(), s.data_ptr(), 0)
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            h = ctx().handle              # the context follows the capturing stream
            with torch.cuda.graph(graph, stream=side):
                _lib.call("fcu_scale", h, x.data_ptr(), x.numel(), C.c_float(2.0))
                _lib.call("fcu_allreduce_grads", h, comm, x.data_ptr(), x.numel())
                _lib.call("fcu_sumsq", h, x.data_ptr(), x.numel(), s.data_ptr(), 0)
                _lib.call("fcu_allreduce_sum_f64", h, comm, s.data_ptr(), 1)
                _lib.call("fcu_comm_join", h, comm)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        for k in range(1, 4):
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(x, torch.full_like(x, 2.0 ** k))
            assert float(s.item()) == 4096 * 4.0 ** k
        graph.reset()
        _lib.call("fcu_comm_poll", comm, 60.0)
    finally:
        ctx().bind_stream(torch.cuda.current_stream().cuda_stream)
        _lib.call("fcu_comm_destroy", comm)


# ------------------------------------------------------------------ ZeRO-1, two ranks on one GPU
class HostComm:
    """The NcclComm surface over gloo on host copies (two processes that share
    one GPU cannot form an NCCL communicator).  Synchronous: eager steps only."""

    def __init__(self, dist):
        self.dist = dist
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()

    def allreduce_avg(self, t):
        h = t.cpu()
        self.dist.all_reduce(h)
        t.copy_(h / self.world)

    def reduce_scatter_avg(self, t):
        self.allreduce_avg(t)          # a superset of slice r

    def allgather(self, t):
        n = t.numel() // self.world
        parts = [torch.empty(n, dtype=t.dtype) for _ in range(self.world)]
        self.dist.all_gather(parts, t[self.rank * n:(self.rank + 1) * n].cpu())
        t.copy_(torch.cat(parts))

    def allreduce_sum_f64(self, t):
        h = t.cpu()
        self.dist.all_reduce(h)
        t.copy_(h)

    def join(self):
        pass


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _zero_rank(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "forge-llm_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import forgellm as F
        from forgellm.dist import DataParallel, ShardedAdam, shard_rows
        F.set_precision("bf16")
        kw = dict(dim=128, hidden=256, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=256)
        batches = [shard_rows(torch.from_numpy(F.RNG(60 + s).ints(4 * 65, 256).reshape(4, 65)),
                              rank, world).numpy() for s in range(3)]
        out = []
        for zero in (False, True):
            m = F.TrainableTransformer(F.Config(**kw), seed=8)
            dp = DataParallel(m, shard=zero, comm=HostComm(dist))
            opt = (ShardedAdam(m, dp, lr=3e-3, totalSteps=20) if zero
                   else F.Adam(m.paramList, lr=3e-3, totalSteps=20))
            for b in batches:
                F.resetTape()
                m.zeroGrad()
                F.backward(m.lossBatch(b))
                dp.finish()
                opt.step()
            torch.cuda.synchronize()
            if zero:
                assert opt.m_flat.numel() * world == m.flat_params.numel()
            out.append(m.flat_params.cpu().numpy().copy())
            dp.detach()
        q.put((rank, out))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_zero1_two_ranks_sharing_one_gpu_match_replicated_adam():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_zero_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    for r in range(2):
        rep, zero = res[r]
        assert np.abs(rep - zero).max() <= 1e-5 * max(1.0, float(np.abs(rep).max()))
    assert np.array_equal(res[0][1], res[1][1])        # the gathers leave identical replicas
    assert np.array_equal(res[0][0], res[1][0])


def test_one_rank_collective_profile():
    """fcu_comm_profile / fcu_comm_profile_read: each collective and join
    issued after profiling starts is recorded with its kind and byte count,
    ready <= start <= end, the collectives run in issue order on the
    communicator's stream, and a record limit drops the calls beyond it."""
    from forgellm import _lib
    from forgellm.autograd import ctx
    from forgellm.dist import NcclComm
    h = ctx().handle
    comm = _comm1()
    try:
        x = torch.randn(1 << 22, device="cuda")
        xb = x.to(torch.bfloat16)
        _lib.call("fcu_allreduce_grads", h, comm, x.data_ptr(), x.numel())   # binds the device
        torch.cuda.synchronize()
        _lib.call("fcu_comm_profile", comm, 4)
        _lib.call("fcu_allreduce_grads", h, comm, x.data_ptr(), x.numel())
        _lib.call("fcu_reduce_scatter_grads", h, comm, x.data_ptr(), x.numel())
        _lib.call("fcu_allgather_params", h, comm, xb.data_ptr(), xb.numel(), 2)
        _lib.call("fcu_comm_join", h, comm)
        _lib.call("fcu_allreduce_grads", h, comm, x.data_ptr(), x.numel())   # beyond the limit
        torch.cuda.synchronize()
        nc = NcclComm.__new__(NcclComm)
        nc.handle = comm
        recs = nc.profile_read(16)
        assert [r["kind"] for r in recs] == ["allreduce", "reduce_scatter", "allgather", "join"]
        assert [r["bytes"] for r in recs] == [4 * x.numel(), 4 * x.numel(), 2 * xb.numel(), 0]
        for r in recs:
            assert 0.0 <= r["ready"] <= r["start"] + 1e-3 and r["start"] <= r["end"] + 1e-3
        for a, b in zip(recs[:2], recs[1:3]):
            assert b["start"] >= a["end"] - 1e-3
        _lib.call("fcu_comm_profile", comm, 0)
    finally:
        _lib.lib().fcu_comm_destroy(comm)
