"""The host-side sampler restatement (oracle/sampling.py) against the
reference's own sampler tests (test/l7-l10.test.js:46-75): greedy at
temperature 0 and at top_k 1, same seed -> same token, min-p keeps only the
high-probability head, top-p concentrates the draws."""
import numpy as np

import oracle as O
from sampling import sample


def test_temperature_zero_is_greedy():
    logits = np.array([0.1, 5.0, 0.2], np.float32)
    for _ in range(20):
        assert sample(logits.copy(), {"temperature": 0}) == 1


def test_top_k_one_is_greedy():
    assert sample(np.array([0.1, 5.0, 0.2], np.float32), {"temperature": 1, "top_k": 1}) == 1


def test_same_seed_same_token():
    rng = O.RNG(3)
    logits = np.array([rng.normal() for _ in range(50)], np.float32)
    a = sample(logits.copy(), {"temperature": 1, "seed": 42})
    b = sample(logits.copy(), {"temperature": 1, "seed": 42})
    assert a == b


def test_min_p_keeps_the_head():
    logits = np.array([10, 9, -20, -20], np.float32)
    picked = {sample(logits.copy(), {"temperature": 1, "min_p": 0.5, "seed": s}) for s in range(200)}
    assert len(picked) <= 2, picked


def test_top_p_concentrates_on_the_head():
    logits = np.array([10, 9.9, 0, -1, -2], np.float32)
    counts = [0] * 5
    for s in range(500):
        counts[sample(logits.copy(), {"temperature": 1, "top_p": 0.5, "seed": s})] += 1
    assert counts[0] + counts[1] >= 490, counts


def test_penalties_and_forbid_follow_the_js():
    """Frequency / presence penalties rewrite the logits in place (fp32
    stores); a forbidden id is never drawn."""
    logits = np.array([3.0, 2.9, 2.8, -1.0], np.float32)
    counts = np.array([2, 0, 0, 0])
    lg = logits.copy()
    sample(lg, {"temperature": 1, "seed": 1, "freqPenalty": 0.5, "presPenalty": 0.25, "counts": counts})
    assert lg[0] == np.float32(3.0 - (0.5 * 2 + 0.25)) and lg[1] == logits[1]
    forbid = [1, 0, 0, 0]
    for s in range(100):
        assert sample(logits.copy(), {"temperature": 1, "seed": s, "forbid": forbid}) != 0
