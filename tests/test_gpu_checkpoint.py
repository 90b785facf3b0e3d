"""Checkpoint / resume: a run that saves, reloads into fresh objects and
continues reproduces the uninterrupted run bit for bit (eager and as a
captured CUDA graph), and a checkpoint of another configuration is refused."""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KW = dict(dim=128, hidden=256, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=256)
B, T = 2, 64


@pytest.fixture(autouse=True)
def bf16_mode():
    import forgellm as F
    F.set_precision("bf16")
    yield
    F.set_precision("fp32")


def _batches(n):
    return [O.RNG(90 + s).ints(B * (T + 1), KW["vocabSize"]).reshape(B, T + 1) for s in range(n)]


def _eager_steps(m, opt, batches):
    import forgellm as F
    out = []
    for b in batches:
        F.resetTape()
        m.zeroGrad()
        out.append(m.backward(m.lossBatch(b)))
        opt.step()
    return out


def test_resume_eager_bit_exact(tmp_path):
    import forgellm as F
    bs = _batches(5)
    ref = F.TrainableTransformer(F.Config(**KW), seed=3)
    opt_r = F.Adam(ref.paramList, lr=3e-3, totalSteps=20)
    losses_ref = _eager_steps(ref, opt_r, bs)

    a = F.TrainableTransformer(F.Config(**KW), seed=3)
    opt_a = F.Adam(a.paramList, lr=3e-3, totalSteps=20)
    _eager_steps(a, opt_a, bs[:3])
    path = str(tmp_path / "run.ck")
    F.save_checkpoint(path, a, opt_a, extra={"step": 3})

    b = F.TrainableTransformer(F.Config(**KW), seed=999)        # different initial weights
    opt_b = F.Adam(b.paramList, lr=3e-3, totalSteps=20)
    hdr = F.load_checkpoint(path, b, opt_b)
    assert hdr["extra"]["step"] == 3 and opt_b.t == 3
    losses_b = _eager_steps(b, opt_b, bs[3:])
    assert losses_b == losses_ref[3:]
    assert torch.equal(b.flat_params, ref.flat_params)
    assert torch.equal(opt_b.m_flat, opt_r.m_flat) and torch.equal(opt_b.v_flat, opt_r.v_flat)


def test_resume_captured_graph_bit_exact(tmp_path):
    import forgellm as F
    from forgellm.graph import CapturedStep
    bs = [torch.from_numpy(x) for x in _batches(5)]
    ref = F.TrainableTransformer(F.Config(**KW), seed=5)
    opt_r = F.Adam(ref.paramList, lr=3e-3, totalSteps=20)
    cs_r = CapturedStep(ref, opt_r, B, T)
    losses_ref = [float(cs_r(x).item()) for x in bs]

    a = F.TrainableTransformer(F.Config(**KW), seed=5)
    opt_a = F.Adam(a.paramList, lr=3e-3, totalSteps=20)
    cs_a = CapturedStep(a, opt_a, B, T)
    for x in bs[:2]:
        cs_a(x)
    path = str(tmp_path / "g.ck")
    F.save_checkpoint(path, a, opt_a)

    b = F.TrainableTransformer(F.Config(**KW), seed=77)
    opt_b = F.Adam(b.paramList, lr=3e-3, totalSteps=20)
    cs_b = CapturedStep(b, opt_b, B, T)
    F.load_checkpoint(path, b, opt_b)
    assert int(opt_b._t_dev.item()) == 2
    losses_b = [float(cs_b(x).item()) for x in bs[2:]]
    assert losses_b == losses_ref[2:]
    assert torch.equal(b.flat_params, ref.flat_params)


def test_wrong_config_or_missing_state_is_refused(tmp_path):
    import forgellm as F
    m = F.TrainableTransformer(F.Config(**KW), seed=1)
    path = str(tmp_path / "w.ck")
    F.save_checkpoint(path, m)                     # weights only
    other = F.TrainableTransformer(F.Config(**dict(KW, hidden=384)), seed=1)
    before = other.flat_params.clone()
    with pytest.raises(ValueError, match="configuration"):
        F.load_checkpoint(path, other)
    assert torch.equal(other.flat_params, before)
    with pytest.raises(ValueError, match="optimizer"):
        F.load_checkpoint(path, F.TrainableTransformer(F.Config(**KW), seed=2),
                          F.Adam(m.paramList, lr=1e-3))
    exp = m.exportWeights()                          # weights-only export of the JS API
    hdr, sec = __import__("forgellm").checkpoint.read_file(path)
    assert np.array_equal(sec["params"][:exp["tok_emb"].size], exp["tok_emb"])
