"""CapturedStep (the whole fused training step replayed as one CUDA graph)
against the same step launched op by op: the same losses and parameters over
several steps, with Adam's cosine schedule advancing on the device."""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KW = dict(dim=128, hidden=256, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=256)


@pytest.fixture(autouse=True)
def bf16_mode():
    import forgellm as F
    F.set_precision("bf16")
    yield
    F.set_precision("fp32")


def test_captured_step_matches_eager_steps():
    import forgellm as F
    from forgellm.graph import CapturedStep
    B, T = 2, 96
    batches = [O.RNG(60 + s).ints(B * (T + 1), KW["vocabSize"]).reshape(B, T + 1) for s in range(4)]
    eager = F.TrainableTransformer(F.Config(**KW), seed=4)
    opt_e = F.Adam(eager.paramList, lr=3e-3, totalSteps=10)
    losses_e = []
    for b in batches:
        F.resetTape()
        eager.zeroGrad()
        losses_e.append(eager.backward(eager.lossBatch(b)))
        opt_e.step()

    graphed = F.TrainableTransformer(F.Config(**KW), seed=4)
    opt_g = F.Adam(graphed.paramList, lr=3e-3, totalSteps=10)
    cs = CapturedStep(graphed, opt_g, B, T)
    assert opt_g.t == 0
    losses_g = [float(cs(torch.from_numpy(b)).item()) for b in batches]
    assert opt_g.t == len(batches)
    assert np.allclose(losses_g, losses_e, rtol=1e-5, atol=1e-6), (losses_g, losses_e)
    pe, pg = eager.flat_params.cpu().numpy(), graphed.flat_params.cpu().numpy()
    assert np.abs(pe - pg).max() <= 1e-5 * max(1.0, float(np.abs(pe).max()))
    info = cs.info.cpu().numpy()                   # {gnorm, scale, lr} of the last step
    import math
    want_lr = 3e-3 * 0.5 * (1 + math.cos(math.pi * len(batches) / 10))
    assert abs(info[2] - want_lr) <= 1e-15


def test_captured_step_restores_state_after_capture():
    import forgellm as F
    from forgellm.graph import CapturedStep
    m = F.TrainableTransformer(F.Config(**KW), seed=9)
    before = m.flat_params.clone()
    opt = F.Adam(m.paramList, lr=1e-2)
    CapturedStep(m, opt, 1, 64)
    assert torch.equal(m.flat_params, before)
    assert opt.t == 0 and int(opt._t_dev.item()) == 0
    assert float(opt.m_flat.abs().max()) == 0.0
