"""Data parallelism on 2 GPUs (skipped with fewer): the averaged gradients of
a batch split over two NCCL ranks equal the full-batch gradients of one
process (fp32 parity mode, relL2 <= 1e-5), and after one Adam step the two
replicas hold bit-identical parameters."""
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
        q.put((rank, g, p))
        dp.detach()
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
