"""Token sampling downstream of the GPU forward: the logits that
TrainableTransformer.forward (train.js:101-158) computes on the GPU, fed to
forge-llm's unchanged host sampler (src/L8/sampling.js:28-96, restated in
oracle/sampling.py), give the same tokens as the reference arithmetic's
logits, for greedy, temperature, top-k, top-p, min-p and penalty settings."""
import numpy as np
import pytest

import oracle as O
from sampling import sample

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

OPTS = [
    {"temperature": 0},
    {"temperature": 1.0},
    {"temperature": 0.7, "top_k": 8},
    {"temperature": 1.3, "top_p": 0.9},
    {"temperature": 1.0, "min_p": 0.05},
    {"temperature": 0.9, "top_k": 20, "top_p": 0.8, "min_p": 0.02},
]


@pytest.mark.parametrize("kw,T", [
    (dict(vocabSize=96, dim=64, nLayers=2, nHeads=4, nKvHeads=2, hidden=176), 40),
    (dict(vocabSize=512, dim=128, nLayers=2, nHeads=4, nKvHeads=4, hidden=256), 24),
])
def test_tokens_from_gpu_logits_match_the_reference_arithmetic(kw, T):
    import forgellm as F
    F.set_precision("fp32")
    V = kw["vocabSize"]
    m = F.TrainableTransformer(F.Config(**kw), seed=21)
    ids = O.RNG(77).ints(T, V)
    F.resetTape()
    got = m.forward(ids).data.detach().cpu().numpy().reshape(T, V).astype(np.float32)
    ocfg = O.Config(**kw)
    _, want = O.model_step(ocfg, O.init_weights(ocfg, 21), ids, ids, 1, T, want_logits=True)
    want = want.reshape(T, V)
    assert O.rel_l2(want, got) <= 1e-5
    n, same = 0, 0
    for t in range(T):
        for j, opt in enumerate(OPTS):
            o = dict(opt, seed=1000 * t + j)
            counts = O.RNG(t + 5).ints(V, 3)
            for extra in ({}, {"freqPenalty": 0.3, "presPenalty": 0.1, "counts": counts}):
                a = sample(got[t].copy(), dict(o, **extra))
                b = sample(want[t].copy(), dict(o, **extra))
                n += 1
                same += a == b
    # the logits agree to ~1e-6 relative, so a draw can only differ when it
    # lands within that distance of a cumulative-probability boundary
    assert same == n, f"{n - same} of {n} draws differ"
