"""GPU-path invariants and full training steps against the oracle, in the
fp32 mode (CUDA cores) and the fp32 tensor-core mode (every matmulT / linear
contraction on tcgen05 through the three-way bf16 split).

* verify.js I-30, I-33a, I-33b, I-33c, I-33d, I-34, I-35, I-36 with every
  forward and backward on the GPU, at the reference's thresholds.
* BASELINE config 1 (tiny char-LM, one fwd+bwd+Adam step): loss, every
  parameter gradient and the post-Adam parameters against the oracle.
* test/l2-l6.test.js batch == per-sample mean, and I-71 overfit, on the GPU.
"""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module", autouse=True, params=["fp32", "fp32tc"])
def fp32_mode(request):
    """Every test of this module runs in both fp32-parity modes: the CUDA
    cores, and the tensor cores (matmulT as a three-way bf16 split with six
    products), at the same thresholds."""
    import forgellm as F
    F.set_precision(request.param)
    yield request.param
    F.set_precision("fp32")


def F():
    import forgellm
    return forgellm


def host(t):
    return t.detach().float().cpu().numpy().ravel()


def gpu_num_grad(loss_fn, params, eps=2e-3):
    """verify.js:141-162 numGrad with the loss computed on the GPU."""
    f = F()
    f.resetTape()
    base = loss_fn()
    f.backward(base)
    worst = 0.0
    for name, p in params.items():
        ana = host(p.grad) if p.grad is not None else np.zeros(p.n, np.float32)
        floor = max(float(np.max(np.abs(ana))) if ana.size else 0.0, 1e-3)
        data = p.data
        for i in range(p.n):
            o = float(data[i].item())
            data[i] = float(np.float32(o + eps))
            lp = float(loss_fn().data[0].item())
            data[i] = float(np.float32(o - eps))
            lm = float(loss_fn().data[0].item())
            data[i] = float(np.float32(o))
            num = (lp - lm) / (2 * eps)
            worst = max(worst, abs(num - float(ana[i])) / floor)
    return worst


@pytest.fixture(scope="module")
def verify_inputs():
    """The exact verify.js draws (RNG(12345), same order as the oracle pins)."""
    rng = O.RNG(12345)
    rng.normals(8 * 12)
    rng.normals(16 * 12)
    rng.normals(12)
    rng.normals(7)
    rng.normals(8)
    for _ in range(16):
        rng.normal()
    d = {}
    d["33a"] = (rng.normals(15, 0.5), rng.normals(20, 0.5), rng.normals(12))
    d["33b"] = (rng.normals(12, 0.5), rng.normals(12))
    d["33c"] = (rng.normals(24, 0.5), rng.normals(24))
    d["33d"] = (rng.normals(64, 0.5), rng.normals(32, 0.5), rng.normals(32, 0.5), rng.normals(64))
    d["34"] = rng.normals(15, 0.5)
    d["35"] = (rng.normals(10, 0.5), rng.normals(10, 0.5), rng.normals(10))
    d["36"] = rng.normals(15, 0.5)
    return d


def test_I30_gradcheck_gpu():
    f = F()
    W = f.param(np.array([0.3, -0.2, 0.1, 0.4, 0.0, 0.2, -0.1, 0.5, 0.3, -0.4, 0.1, 0.2, 0.6, -0.3,
                          0.2, 0.4, -0.5, 0.1, 0.3, 0.2], np.float32))
    x = f.leaf(np.array([1, 0.5, -0.3, 0.2, 0.4], np.float32))

    def lf():
        f.resetTape()
        return f.softmaxCE(f.linear(W, x, 4, 5), 2)

    gc = f.gradCheck(lf, {"W": W})
    assert gc["maxRelErr"] < 1e-4


def test_I33a_matmulT_gpu(verify_inputs):
    f = F()
    X0, W0, t = verify_inputs["33a"]
    X, W = f.param(X0.copy()), f.param(W0.copy())
    w = gpu_num_grad(lambda: (f.resetTape(), f.weightedSum(f.matmulT(X, W, 3, 5, 4), t))[1],
                     {"X": X, "W": W})
    assert w < 2e-3


def test_I33b_rmsnorm_gpu(verify_inputs):
    f = F()
    X0, t = verify_inputs["33b"]
    X, Wt = f.param(X0.copy()), f.param(np.ones(6, np.float32))
    w = gpu_num_grad(lambda: (f.resetTape(), f.weightedSum(f.rmsNorm(X, Wt, 2, 6, 1e-5), t))[1],
                     {"X": X, "Wt": Wt})
    assert w < 2e-3


def test_I33c_rope_gpu(verify_inputs):
    f = F()
    X0, t = verify_inputs["33c"]
    X = f.param(X0.copy())
    w = gpu_num_grad(lambda: (f.resetTape(), f.weightedSum(f.ropeRows(X, 3, 2, 4, 0, 10000), t))[1],
                     {"X": X})
    assert w < 2e-3


def test_I33d_attention_gpu(verify_inputs):
    f = F()
    Q0, K0, V0, t = verify_inputs["33d"]
    Q, K, V = f.param(Q0.copy()), f.param(K0.copy()), f.param(V0.copy())
    w = gpu_num_grad(lambda: (f.resetTape(),
                              f.weightedSum(f.causalAttn(Q, K, V, 4, 4, 2, 4), t))[1],
                     {"Q": Q, "K": K, "V": V})
    assert w < 2e-3


def test_I34_ce_grad_gpu(verify_inputs):
    f = F()
    L0 = verify_inputs["34"]
    targets = [1, 3, 0]
    f.resetTape()
    L = f.param(L0.copy())
    f.backward(f.crossEntropyMean(L, targets, 3, 5))
    g = host(L.grad)
    worst = 0.0
    for ti in range(3):
        row = L0[ti * 5:(ti + 1) * 5].astype(np.float64)
        p = np.exp(row - row.max())
        p /= p.sum()
        for i in range(5):
            want = (p[i] - (1.0 if i == targets[ti] else 0.0)) / 3
            worst = max(worst, abs(float(g[ti * 5 + i]) - want))
    assert worst < 1e-6


def test_I35_swiglu_gpu(verify_inputs):
    f = F()
    G0, U0, t = verify_inputs["35"]
    G, U = f.param(G0.copy()), f.param(U0.copy())
    w = gpu_num_grad(lambda: (f.resetTape(), f.weightedSum(f.swigluRows(G, U, 2, 5), t))[1],
                     {"G": G, "U": U})
    assert w < 2e-3


def test_I36_embed_gpu(verify_inputs):
    f = F()
    E0 = verify_inputs["36"]
    ids = [0, 3, 3]
    f.resetTape()
    E = f.param(E0.copy())
    X = f.embedLookup(E, ids, 5, 3)
    f.backward(f.weightedSum(X, np.arange(1, 10, dtype=np.float32)))
    g = host(E.grad)
    for v in range(5):
        for d in range(3):
            want = sum(ti * 3 + d + 1 for ti in range(3) if ids[ti] == v)
            assert abs(g[v * 3 + d] - want) <= 1e-5


# ------------------------------------------------------------------ full steps
C1 = dict(vocabSize=64, dim=64, nLayers=2, nHeads=4, nKvHeads=4, hidden=176, normEps=1e-5,
          ropeTheta=10000)


def _c1_inputs():
    ids = O.RNG(1).ints(65, 64)      # a separate RNG(1) instance draws the tokens
    return ids[:64].copy(), ids[1:].copy()


def test_config1_train_step_matches_oracle():
    """initWeights(cfg, 1), one loss() + backward() + Adam
    (lr 3e-3) step.  Loss and every gradient within relL2 1e-5; Adam given the
    same gradients reproduces the oracle's parameters."""
    f = F()
    ocfg = O.Config(**{k: v for k, v in C1.items()})
    P = O.init_weights(ocfg, 1)
    ids, tg = _c1_inputs()
    G = np.zeros_like(P)
    lo = O.model_step(ocfg, P, ids, tg, 1, 64, G)

    m = f.TrainableTransformer(f.Config(**C1), seed=1)
    assert np.array_equal(host(m.flat_params), P)
    f.resetTape()
    m.zeroGrad()
    lg = m.backward(m.loss(list(ids) + [int(tg[-1])], tg))
    assert abs(lg - float(lo)) <= TOL * abs(float(lo))
    grads = host(m.flat_grads)
    assert O.rel_l2(G, grads) <= TOL
    # per-parameter check so a wrong small tensor cannot hide in the total
    from forgellm.train import param_shapes
    off = 0
    for name, n in param_shapes(m.cfg):
        assert O.rel_l2(G[off:off + n], grads[off:off + n]) <= 1e-4, name
        off += n
    opt = f.Adam(m.paramList, lr=3e-3)
    opt.step()
    po = P.copy()
    O.adam_step(po, grads, np.zeros_like(P), np.zeros_like(P), 1, lr=3e-3)
    assert np.abs(host(m.flat_params) - po).max() <= 1e-6


def test_batch_equals_per_sample_mean_gpu():
    """test/l2-l6.test.js:175-187 on the GPU (tolerance 1e-5)."""
    f = F()
    cfg = f.Config(dim=32, hidden=64, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=20, maxSeq=32)
    m = f.TrainableTransformer(cfg, f.initWeights(cfg, 11))
    rows = [[1, 2, 3, 4, 5, 6], [7, 8, 9, 10, 11, 12]]
    f.resetTape()
    batch = m.backward(m.lossBatch(rows))
    s = 0.0
    for r in rows:
        f.resetTape()
        s += m.backward(m.loss(r[:-1], r[1:]))
    assert abs(batch - s / 2) < 1e-5


def test_batch_step_matches_oracle():
    f = F()
    kw = dict(dim=48, hidden=96, nLayers=2, nHeads=6, nKvHeads=2, vocabSize=50)
    ocfg = O.Config(**kw)
    P = O.init_weights(ocfg, 21)
    rows = O.RNG(22).ints(3 * 17, 50).reshape(3, 17)
    G = np.zeros_like(P)
    lo = O.model_step(ocfg, P, rows[:, :-1].ravel(), rows[:, 1:].ravel(), 3, 16, G)
    m = f.TrainableTransformer(f.Config(**kw), seed=21)
    f.resetTape()
    lg = m.backward(m.lossBatch(rows))
    assert abs(lg - float(lo)) <= TOL * abs(float(lo))
    assert O.rel_l2(G, host(m.flat_grads)) <= TOL


def test_I71_overfit_gpu():
    """verify.js:313-325 on the GPU: reported 'loss 2.9805 -> 0.0006'."""
    f = F()
    cfg = f.Config(dim=32, hidden=64, nLayers=1, nHeads=4, nKvHeads=4, vocabSize=20, maxSeq=16)
    m = f.TrainableTransformer(cfg, f.initWeights(cfg, 777))
    data = [1, 2, 3, 4, 5, 6, 7, 8]
    f.resetTape()
    first = m.backward(m.loss(data, data[1:]))
    opt = f.Adam(m.paramList, lr=0.05, totalSteps=60, clip=1.0)
    last = first
    for _ in range(60):
        f.resetTape()
        m.zeroGrad()
        last = m.backward(m.loss(data, data[1:]))
        opt.step()
    assert "%.4f" % first == "2.9805"
    assert last < first * 0.6
    assert last < 0.01
