"""The bf16 fused TrainableTransformer step (FCU_PREC_BF16) against the CPU
oracle and against its own invariants.

Stated bound: bf16 operands everywhere (weights, activations, P, dS and the
activation gradients), fp32 accumulation, fp32 master weights and gradients.
Against the fp32 oracle the loss agrees to 1e-2 relative and the flat
gradient to relL2 <= 5e-2 (bf16 keeps 8 mantissa bits and rounds once per
stored activation, so errors compound over layers)."""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

LOSS_TOL = 1e-2
GRAD_TOL = 5e-2


@pytest.fixture(autouse=True)
def bf16_mode():
    import forgellm as F
    F.set_precision("bf16")
    yield
    F.set_precision("fp32")


def host(t):
    return t.detach().float().cpu().numpy().ravel()


def _step(kw, seed, rows, threads=8):
    import forgellm as F
    m = F.TrainableTransformer(F.Config(**kw), seed=seed)
    assert m._use_fused()
    F.resetTape()
    loss = m.backward(m.lossBatch(rows))
    ocfg = O.Config(**kw)
    P = O.init_weights(ocfg, seed)
    G = np.zeros_like(P)
    O.set_threads(threads)
    try:
        lo = O.model_step(ocfg, P, rows[:, :-1].ravel(), rows[:, 1:].ravel(), rows.shape[0],
                          rows.shape[1] - 1, G)
    finally:
        O.set_threads(1)
    return m, loss, float(lo), G


@pytest.mark.parametrize("kw,B,T", [
    (dict(dim=64, hidden=128, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=96), 2, 70),
    (dict(dim=128, hidden=256, nLayers=3, nHeads=4, nKvHeads=4, vocabSize=512), 3, 64),
    (dict(dim=768, hidden=2048, nLayers=2, nHeads=12, nKvHeads=4, vocabSize=32000), 1, 128),
])
def test_fused_step_matches_oracle(kw, B, T):
    rows = O.RNG(40 + B + T).ints(B * (T + 1), kw["vocabSize"]).reshape(B, T + 1)
    m, loss, lo, G = _step(kw, 7, rows)
    assert abs(loss - lo) <= LOSS_TOL * abs(lo), (loss, lo)
    g = host(m.flat_grads)
    assert O.rel_l2(G, g) <= GRAD_TOL, O.rel_l2(G, g)
    from forgellm.train import param_shapes
    off = 0
    for name, n in param_shapes(m.cfg):   # no tensor may be wrong on its own
        r = O.rel_l2(G[off:off + n], g[off:off + n])
        assert r <= 1e-1, (name, r)
        off += n


def test_fused_step_is_deterministic_and_accumulates():
    import forgellm as F
    kw = dict(dim=64, hidden=128, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=96)
    rows = O.RNG(3).ints(2 * 33, 96).reshape(2, 33)
    m = F.TrainableTransformer(F.Config(**kw), seed=5)
    F.resetTape()
    m.backward(m.lossBatch(rows))
    g1 = host(m.flat_grads).copy()
    F.resetTape()
    m.backward(m.lossBatch(rows))              # no zeroGrad: JS `+=` doubles the grads
    g2 = host(m.flat_grads)
    assert np.allclose(g2, 2 * g1, rtol=1e-5, atol=1e-7)
    m.zeroGrad()
    F.resetTape()
    m.backward(m.lossBatch(rows))
    assert np.array_equal(host(m.flat_grads), g1)


@pytest.mark.parametrize("kw,B,T", [
    (dict(dim=64, hidden=128, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=96), 2, 70),
    (dict(dim=256, hidden=768, nLayers=1, nHeads=4, nKvHeads=2, vocabSize=256), 1, 200),
])
def test_swiglu_epilogue_fusion_changes_no_bit(kw, B, T):
    """The step with SwiGLU in the GEMM epilogues gives bit-identical loss and
    gradients to the step with the standalone SwiGLU kernels."""
    import forgellm as F
    rows = O.RNG(11).ints(B * (T + 1), kw["vocabSize"]).reshape(B, T + 1)
    m = F.TrainableTransformer(F.Config(**kw), seed=4)
    out = []
    for fuse in (True, False):
        m.zeroGrad()
        F.resetTape()
        loss = m.lossBatch(rows)
        fs = m._fused_steps[(B, T)]
        assert fs.can_fuse_swiglu
        if fs.fuse_swiglu != fuse:          # rerun the forward on the other path
            fs.fuse_swiglu = fuse
            F.resetTape()
            loss = m.lossBatch(rows)
        lv = m.backward(loss)
        out.append((float(lv), host(m.flat_grads).copy()))
    assert out[0][0] == out[1][0]
    assert np.array_equal(out[0][1], out[1][1])


def test_bf16_weight_copy_follows_adam_and_host_writes():
    import forgellm as F
    kw = dict(dim=64, hidden=128, nLayers=1, nHeads=4, nKvHeads=4, vocabSize=64)
    rows = O.RNG(8).ints(2 * 17, 64).reshape(2, 17)
    m = F.TrainableTransformer(F.Config(**kw), seed=2)
    opt = F.Adam(m.paramList, lr=1e-2)
    for _ in range(2):
        F.resetTape()
        m.zeroGrad()
        m.backward(m.lossBatch(rows))
        opt.step()
    want = m.flat_params.to(torch.bfloat16)
    assert torch.equal(m.flat_params_bf16, want)
    m.params["layers"][0]["wo"].data[3] = 0.5            # host write (numGrad style)
    m.bf16_weights()
    assert float(m.flat_params_bf16[m.offsets["layer.0.wo"][0] + 3]) == 0.5


def test_fused_overfit_I71():
    """verify.js:313-325's overfit check through the fused bf16 step (at the
    smallest widths the fused kernels take: head dim 16, vocab a multiple of 8)."""
    import forgellm as F
    cfg = F.Config(dim=64, hidden=64, nLayers=1, nHeads=4, nKvHeads=4, vocabSize=24, maxSeq=16)
    m = F.TrainableTransformer(cfg, F.initWeights(cfg, 777))
    assert m._use_fused()
    data = [1, 2, 3, 4, 5, 6, 7, 8]
    F.resetTape()
    first = m.backward(m.loss(data, data[1:]))
    opt = F.Adam(m.paramList, lr=0.05, totalSteps=60, clip=1.0)
    last = first
    for _ in range(60):
        F.resetTape()
        m.zeroGrad()
        last = m.backward(m.loss(data, data[1:]))
        opt.step()
    assert last < first * 0.6 and last < 0.05, (first, last)


@pytest.mark.parametrize("T,D", [(1000, 768), (257, 100), (64, 1024)])
def test_rmsnorm_fwd_bf16_add(T, D):
    """Residual add fused into the normalisation: Xout is exactly X + A
    (fp32), inv and the bf16 output follow from Xout."""
    from forgellm import _lib
    from forgellm.autograd import ctx
    g = torch.Generator(device="cuda").manual_seed(T + D)
    X = torch.randn(T, D, device="cuda", generator=g)
    A = torch.randn(T, D, device="cuda", generator=g)
    w = torch.randn(D, device="cuda", generator=g)
    Xout = torch.empty(T, D, device="cuda")
    out = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
    inv = torch.empty(T, device="cuda")
    _lib.call("fcu_rmsnorm_fwd_bf16_add", ctx().handle, X.data_ptr(), A.data_ptr(), w.data_ptr(), T, D,
              1e-5, Xout.data_ptr(), out.data_ptr(), inv.data_ptr())
    torch.cuda.synchronize()
    assert torch.equal(Xout, X + A)
    x = Xout.double()
    iv = 1.0 / torch.sqrt((x * x).mean(1) + 1e-5)
    assert float(((inv.double() - iv).abs() / iv).max()) <= 1e-5
    ref = x * iv[:, None] * w.double()[None, :]
    assert float(((out.double() - ref).abs() - 2 ** -8 * ref.abs()).max()) <= 1e-6


@pytest.mark.parametrize("T,V", [(8192, 32000), (300, 1000), (7, 1001)])
def test_ce_fwd_bf16grad(T, V):
    """Fused-path cross-entropy: mean loss against float64 to 1e-5 relative,
    dLogits = (softmax - onehot) / T within bf16 rounding (plus 2^-20 of the
    row's largest probability for the fast exp)."""
    from forgellm import _lib
    from forgellm.autograd import ctx
    g = torch.Generator(device="cuda").manual_seed(T + V)
    logits = torch.randn(T, V, device="cuda", generator=g) * 2.0
    targets = torch.randint(0, V, (T,), device="cuda", generator=g, dtype=torch.int32)
    loss = torch.empty(1, device="cuda")
    d = torch.empty(T, V, device="cuda", dtype=torch.bfloat16)
    _lib.call("fcu_ce_fwd_bf16grad", ctx().handle, logits.data_ptr(), targets.data_ptr(), T, V,
              loss.data_ptr(), d.data_ptr())
    torch.cuda.synchronize()
    x = logits.double()
    lse = torch.logsumexp(x, 1)
    ref_loss = float((lse - x.gather(1, targets.long()[:, None])[:, 0]).mean())
    assert abs(float(loss) - ref_loss) <= 1e-5 * abs(ref_loss)
    ref = torch.softmax(x, 1)
    ref[torch.arange(T), targets.long()] -= 1.0
    ref /= T
    err = (d.double() - ref).abs() - 2 ** -8 * ref.abs()
    assert float(err.max()) <= 2 ** -20 / T
