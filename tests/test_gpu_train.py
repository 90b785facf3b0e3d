"""train() with device-resident tokens: the window gather reproduces the JS
windows (train.js:256-262) exactly, and the graph-replayed loop follows the
op-by-op loop."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KW = dict(dim=64, hidden=128, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=96)


def test_gather_windows_matches_js_windows():
    import forgellm as F
    from forgellm import _lib
    from forgellm.autograd import ctx
    n, B, T1 = 1000, 6, 33
    data = F.RNG(3).ints(n, 50).astype(np.int32)
    rng = F.RNG(11)
    starts = np.array([rng.int(max(1, n - T1)) for _ in range(B - 2)] + [n - 5, n - 1], np.int32)
    want = np.array([[data[s + i] if s + i < n else data[-1] for i in range(T1)] for s in starts], np.int32)
    d, st = torch.from_numpy(data).cuda(), torch.from_numpy(starts).cuda()
    out = torch.full((B, T1), -7, dtype=torch.int32, device="cuda")
    _lib.call("fcu_gather_windows", ctx().handle, d.data_ptr(), n, st.data_ptr(), B, T1, out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), want)


@pytest.mark.parametrize("precision", ["bf16"])
def test_train_graph_follows_op_by_op(precision):
    import forgellm as F
    F.set_precision(precision)
    try:
        data = F.RNG(5).ints(5000, KW["vocabSize"])
        hist = {}
        for graph in (False, True):
            m = F.TrainableTransformer(F.Config(**KW), seed=2)
            hist[graph] = (F.train(m, data, steps=6, batchSize=2, seqLen=64, lr=3e-3, logEvery=1,
                                   graph=graph), m.flat_params.cpu().numpy())
        (he, pe), (hg, pg) = hist[False], hist[True]
        assert [h["step"] for h in he] == [h["step"] for h in hg] == list(range(6))
        for a, b in zip(he, hg):
            assert abs(a["loss"] - b["loss"]) <= 1e-4 * abs(a["loss"]), (a, b)
            assert abs(a["lr"] - b["lr"]) <= 1e-12
        assert np.abs(pe - pg).max() <= 1e-4 * max(1.0, float(np.abs(pe).max()))
    finally:
        F.set_precision("fp32")


@pytest.mark.parametrize("graph", [False, True])
def test_train_batches_are_the_js_windows_without_per_step_sync(graph):
    """train() at its default logEvery (10) over 13 steps: the host never
    waits between steps 1-9, so a host buffer rewritten per step would be
    read late.  The batches the device used (cloned in stream order) must be
    the windows train.js:256-264 draws from RNG(seed)."""
    import forgellm as F
    F.set_precision("bf16")
    try:
        n, B, seqLen, steps, seed = 3000, 3, 64, 13, 7
        data = F.RNG(9).ints(n, KW["vocabSize"])
        rng = F.RNG(seed)
        want = []
        for _ in range(steps):
            rows = []
            for _ in range(B):
                s = rng.int(max(1, n - seqLen - 1))
                rows.append([data[s + i] if s + i < n else data[-1] for i in range(seqLen + 1)])
            want.append(np.array(rows, np.int32))
        got = []
        m = F.TrainableTransformer(F.Config(**KW), seed=2)
        hist = F.train(m, data, steps=steps, batchSize=B, seqLen=seqLen, lr=3e-3, seed=seed,
                       graph=graph, onBatch=lambda k, b: got.append(b.clone()))
        torch.cuda.synchronize()
        assert [h["step"] for h in hist] == [0, 10, 12]
        assert len(got) == steps
        for k in range(steps):
            assert np.array_equal(got[k].cpu().numpy(), want[k]), k
    finally:
        F.set_precision("fp32")
