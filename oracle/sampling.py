"""CPU restatement of forge-llm's host-side token sampler -- TEST INFRASTRUCTURE.

`sample` follows src/L8/sampling.js:28-96 (and `softmax` of
src/L1/special.js:66-74) step for step, with the JS numerics: scalar locals
and sums are double, every Float32Array store rounds to float32, the sort is
stable (V8's Array.prototype.sort), and the uniform draw comes from the same
xorshift128+ RNG (src/L0/numeric.js:27-49).  Plain Python loops, so the
summation order is the JS one; meant for test-sized vocabularies.

The sampler itself is not part of the training hot path: forge-llm calls it
on the host with the logits the forward produced.  The tests use this
restatement to show that the tokens drawn from the GPU path's logits are the
tokens drawn from the reference arithmetic's logits.
"""
from __future__ import annotations

import math

import numpy as np

from oracle import RNG


def _f32(x: float) -> float:
    return float(np.float32(x))


def _argmax(a) -> int:
    """argmax of sampling.js:91: the first index of the largest value."""
    bi, bv = 0, -math.inf
    for i, v in enumerate(a):
        if v > bv:
            bv, bi = v, i
    return bi


def _argsort_desc(arr) -> list[int]:
    """sampling.js:92-96: indices by descending value, ties in index order."""
    return sorted(range(len(arr)), key=lambda i: -arr[i])


def _softmax(x: list[float]) -> list[float]:
    """special.js:66-74 into a Float32Array."""
    m = -math.inf
    for v in x:
        if v > m:
            m = v
    out, s = [], 0.0
    for v in x:
        e = math.exp(v - m)
        out.append(_f32(e))
        s += e
    inv = 1.0 / s
    return [_f32(v * inv) for v in out]


def sample(logits, opt: dict | None = None, rng: RNG | None = None) -> int:
    """sampling.js:28-86.  `logits` is a float32 array (modified in place by
    the frequency / presence penalties, as the JS does)."""
    opt = dict(opt or {})
    if rng is None:
        rng = RNG(opt.get("seed", 0x9E3779B9))
    logits = np.asarray(logits)
    assert logits.dtype == np.float32
    n = logits.shape[0]
    temperature = opt.get("temperature", 1.0)
    k = opt.get("top_k", 0)
    top_p = opt.get("top_p", 1.0)
    min_p = opt.get("min_p", 0.0)
    t = max(temperature, 1e-6)
    fp, pp = opt.get("freqPenalty", 0), opt.get("presPenalty", 0)
    if (fp or pp) and opt.get("counts") is not None:
        counts = opt["counts"]
        for i in range(n):
            c = int(counts[i])
            if c > 0:
                logits[i] = np.float32(float(logits[i]) - (fp * c + pp * (1 if c > 0 else 0)))
    scaled = [_f32(float(v) / t) for v in logits]
    if temperature == 0 or (k == 1 and top_p >= 1):
        return _argmax(scaled)
    probs = _softmax(scaled)
    if min_p > 0:
        pmax = 0.0
        for v in probs:
            if v > pmax:
                pmax = v
        thr = min_p * pmax
        s = 0.0
        for i in range(n):
            if probs[i] < thr:
                probs[i] = 0.0
            else:
                s += probs[i]
        if s > 0:
            probs = [_f32(v / s) for v in probs]
    allow = [1] * n
    if k > 1:
        order = _argsort_desc(probs)
        allow = [0] * n
        for i in range(min(k, n)):
            allow[order[i]] = 1
    if top_p < 1:
        order = _argsort_desc(probs)
        cum = 0.0
        for i in range(n):
            idx = order[i]
            if not allow[idx]:
                continue
            cum += probs[idx]
            if cum >= top_p:
                for j in range(i + 1, n):
                    allow[order[j]] = 0
                break
    forbid = opt.get("forbid")
    s = 0.0
    for i in range(n):
        if allow[i]:
            s += 0.0 if (forbid is not None and forbid[i]) else probs[i]
    r = rng.next() * s
    acc = 0.0
    for i in range(n):
        if not allow[i]:
            continue
        if forbid is not None and forbid[i]:
            continue
        acc += probs[i]
        if r <= acc:
            return i
    return _argmax(probs)
