"""Data parallelism on 2 GPUs (skipped with fewer), through the C-ABI NCCL
communicator (fcu_comm_init / fcu_allreduce_grads / fcu_reduce_scatter_grads /
fcu_allgather_params): the averaged gradients of a batch split over two ranks
equal the full-batch gradients of one process (fp32 parity mode, relL2 <=
1e-5), and after one Adam step the two replicas hold bit-identical
parameters; ZeRO-1 matches replicated Adam, eager and graph-captured."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KW = dict(dim=64, hidden=128, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=96)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import sys
    from datetime import timedelta
    sys.path.insert(0, os.path.join(ROOT, "forge-llm_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import forgellm as F
        from forgellm.dist import DataParallel, shard_rows
        F.set_precision("fp32")
        rows = F.RNG(9).ints(4 * 33, KW["vocabSize"]).reshape(4, 33)
        m = F.TrainableTransformer(F.Config(**KW), seed=3)
        dp = DataParallel(m)
        F.resetTape()
        loss = m.lossBatch(shard_rows(torch.from_numpy(rows), rank, world).numpy())
        F.backward(loss)
        dp.finish()
        opt = F.Adam(m.paramList, lr=1e-3)
        g = m.flat_grads.cpu().numpy().copy()
        opt.step()
        p = m.flat_params.cpu().numpy()
        torch.cuda.synchronize()
        dp.check(60.0)             # the C-ABI communicator saw no failure
        q.put((rank, g, p))
        dp.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_two_rank_gradients_equal_full_batch():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        r, g, p = q.get(timeout=300)
        out[r] = (g, p)
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    ocfg = O.Config(**KW)
    P = O.init_weights(ocfg, 3)
    G = np.zeros_like(P)
    rows = O.RNG(9).ints(4 * 33, KW["vocabSize"]).reshape(4, 33)
    O.model_step(ocfg, P, rows[:, :-1].ravel(), rows[:, 1:].ravel(), 4, 32, G)
    assert O.rel_l2(G, out[0][0]) <= 1e-5
    assert np.array_equal(out[0][0], out[1][0])
    assert np.array_equal(out[0][1], out[1][1])


def _rank_zero(rank, world, port, q, graph):
    """Replicated Adam and ZeRO-1 ShardedAdam on the same 2-rank data-parallel
    run (bf16 fused path): the parameters after three steps agree."""
    import sys
    from datetime import timedelta
    sys.path.insert(0, os.path.join(ROOT, "forge-llm_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import forgellm as F
        from forgellm.dist import DataParallel, ShardedAdam, shard_rows
        from forgellm.graph import CapturedStep
        F.set_precision("bf16")
        kw = dict(dim=128, hidden=256, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=256)
        batches = [torch.from_numpy(shard_rows(torch.from_numpy(F.RNG(40 + s).ints(4 * 65, 256).reshape(4, 65)),
                                               rank, world).numpy()) for s in range(3)]
        out = []
        for zero in (False, True):
            m = F.TrainableTransformer(F.Config(**kw), seed=8)
            if zero:
                dp = DataParallel(m, shard=True)
                opt = ShardedAdam(m, dp, lr=3e-3, totalSteps=20)
            else:
                dp = DataParallel(m)
                opt = F.Adam(m.paramList, lr=3e-3, totalSteps=20)
            cs = CapturedStep(m, opt, 2, 64, dp=dp) if graph else None
            for b in batches:
                if graph:
                    cs(b)
                else:
                    F.resetTape()
                    m.zeroGrad()
                    F.backward(m.lossBatch(b.numpy()))
                    dp.finish()
                    opt.step()
            torch.cuda.synchronize()
            out.append((m.flat_params.cpu().numpy().copy(), int(opt.t)))
            if graph:
                cs.graph.reset()
                del cs
            dp.check(60.0)
            dp.close()
        q.put((rank, out))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("graph", [False, True])
def test_sharded_adam_matches_replicated(graph):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_zero, args=(r, 2, port, q, graph)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    for r in range(2):
        (rep, t_rep), (zero, t_zero) = res[r]
        assert t_rep == t_zero == 3
        # the same update up to the summation order of the gradient norm and
        # of the NCCL reductions (reduce-scatter vs all-reduce)
        assert np.abs(rep - zero).max() <= 1e-5 * max(1.0, float(np.abs(rep).max()))
    assert np.array_equal(res[0][1][0], res[1][1][0])       # replicas identical after the gathers
