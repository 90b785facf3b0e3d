"""GPU parity: every hot-path kernel, called through the C-ABI (via the
forgellm host layer), against the CPU oracle on identical seeded inputs.

Tolerances (FCU_PREC_FP32, the parity mode): relL2 <= 1e-5 on every output
and gradient (relL2 as src/L0/numeric.js:152-156); index/copy work
(embedding, sliceCols) bit-exact.  The reference's own gradient invariants
(verify.js I-30, I-33a-d, I-34, I-35, I-36) run with the GPU computing every
forward and backward, at the reference's thresholds.
"""
import math

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def fp32_mode():
    import forgellm as F
    F.set_precision("fp32")
    yield


def F():
    import forgellm
    return forgellm


def dev(a, dtype=None):
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a).cuda()
    return t if dtype is None else t.to(dtype)


def host(t):
    return t.detach().float().cpu().numpy().ravel()


def rel(ref, got):
    """relL2 (numeric.js:152-156); a reference that is zero up to fp32
    rounding noise (|ref| <= 1e-6 per element, e.g. dQ of a 1-token sequence)
    is compared in absolute terms instead."""
    ref = np.asarray(ref, np.float32).ravel()
    got = np.asarray(got, np.float32).ravel()
    if ref.size and float(np.max(np.abs(ref))) <= 1e-6:
        return float(np.max(np.abs(ref - got))) / 1e-1
    return O.rel_l2(ref, got)


# ------------------------------------------------------------------ matmulT
@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (3, 5, 4), (4, 5, 3), (7, 13, 9), (130, 70, 260),
                                   (64, 768, 1280)])
def test_matmulT_matches_oracle(M, K, N):
    f = F()
    rng = O.RNG(1000 + M + K + N)
    X, W, g = rng.normals(M * K), rng.normals(N * K), rng.normals(M * N)
    gX0, gW0 = rng.normals(M * K), rng.normals(N * K)   # pre-existing grads: JS `+=`
    f.resetTape()
    Xn, Wn = f.param(X), f.param(W)
    Xn.grad, Wn.grad = gX0.copy(), gW0.copy()
    Y = f.matmulT(Xn, Wn, M, K, N)
    Y.grad = g
    Y._b(Y.grad)
    Yo = O.matmulT_fwd(X, W, M, K, N)
    gXo, gWo = O.matmulT_bwd(g, X, W, M, K, N, gX0.copy(), gW0.copy())
    assert rel(Yo, host(Y.data)) <= TOL
    assert rel(gXo, host(Xn.grad)) <= TOL
    assert rel(gWo, host(Wn.grad)) <= TOL


def test_matmulT_config2_full_size():
    """X[4096x2048] . W[8192x2048]^T, dX, dW; all fp32
    N(0,1) from RNG(2).  The oracle checks 24 rows of Y, dX and dW."""
    f = F()
    M, K, N = 4096, 2048, 8192
    rng = O.RNG(2)
    X, W, dY = rng.normals(M * K), rng.normals(N * K), rng.normals(M * N)
    f.resetTape()
    Xn, Wn = f.param(X), f.param(W)
    Y = f.matmulT(Xn, Wn, M, K, N)
    Y.grad = dY
    Y._b(Y.grad)
    torch.cuda.synchronize()
    Yg, dXg, dWg = host(Y.data), host(Xn.grad), host(Wn.grad)
    sel = np.random.default_rng(0).choice(M, 24, replace=False)
    seln = np.random.default_rng(1).choice(N, 24, replace=False)
    O.set_threads(8)
    try:
        Xs = X.reshape(M, K)[sel].ravel()
        dYs = dY.reshape(M, N)[sel].ravel()
        Yo = O.matmulT_fwd(Xs, W, 24, K, N)
        assert rel(Yo, Yg.reshape(M, N)[sel]) <= TOL
        dXo = O.matmulT_bwd_dx(dYs, W, 24, K, N)
        assert rel(dXo, dXg.reshape(M, K)[sel]) <= TOL
        for n in seln[:8]:
            dWo = O.matmulT_bwd_dw_rows(dY, X, M, K, N, int(n), int(n) + 1)
            assert rel(dWo, dWg.reshape(N, K)[n]) <= TOL
    finally:
        O.set_threads(1)
    # size-independent property: Y . 1 == X . (W^T 1) (linearity)
    ones = np.ones(N, np.float32)
    lhs = Yg.reshape(M, N).astype(np.float64) @ ones
    rhs = X.reshape(M, K).astype(np.float64) @ (W.reshape(N, K).astype(np.float64).T @ ones)
    assert np.linalg.norm(lhs - rhs) / np.linalg.norm(rhs) < 1e-4


# ------------------------------------------------------------------ embedding
def test_embed_bit_exact_with_duplicates():
    f = F()
    V, D = 37, 24
    rng = O.RNG(3)
    E = rng.normals(V * D)
    ids = rng.ints(300, V)
    ids[:50] = 5                                     # a heavy id
    g = rng.normals(ids.size * D)
    gE0 = rng.normals(V * D)
    f.resetTape()
    En = f.param(E)
    En.grad = gE0.copy()
    X = f.embedLookup(En, ids, V, D)
    assert np.array_equal(host(X.data), O.embed_fwd(E, ids, V, D))
    X.grad = g
    X._b(X.grad)
    assert np.array_equal(host(En.grad), O.embed_bwd(g, ids, V, D, gE0.copy()))


def test_embed_large_and_out_of_range():
    f = F()
    V, D, T = 32000, 64, 5000
    rng = O.RNG(4)
    E = rng.normals(V * D)
    ids = rng.ints(T, V)
    ids[7] = -1
    ids[9] = V           # out of range: NaN row forward, skipped backward (JS semantics)
    g = rng.normals(T * D)
    f.resetTape()
    En = f.param(E)
    X = f.embedLookup(En, ids, V, D)
    out = host(X.data).reshape(T, D)
    assert np.isnan(out[7]).all() and np.isnan(out[9]).all()
    ok = np.ones(T, bool)
    ok[[7, 9]] = False
    assert np.array_equal(out[ok], O.embed_fwd(E, ids[ok], V, D).reshape(-1, D))
    X.grad = g
    X._b(X.grad)
    want = O.embed_bwd(g.reshape(T, D)[ok].ravel(), ids[ok], V, D)
    assert np.array_equal(host(En.grad), want)


def test_empty_inputs():
    f = F()
    f.resetTape()
    En = f.param(np.ones(4 * 3, np.float32))
    X = f.embedLookup(En, np.zeros(0, np.int32), 4, 3)
    assert X.n == 0


# ------------------------------------------------------------------ rmsNorm
@pytest.mark.parametrize("T,D", [(2, 6), (3, 8), (65, 768), (1, 1), (300, 100)])
def test_rmsnorm_matches_oracle(T, D):
    f = F()
    rng = O.RNG(5 + T + D)
    X, w, g = rng.normals(T * D), rng.normals(D), rng.normals(T * D)
    gX0 = rng.normals(T * D)
    f.resetTape()
    Xn, wn = f.param(X), f.param(w)
    Xn.grad = gX0.copy()
    Y = f.rmsNorm(Xn, wn, T, D, 1e-5)
    Yo, inv = O.rmsnorm_fwd(X, w, T, D, 1e-5)
    assert rel(Yo, host(Y.data)) <= TOL
    Y.grad = g
    Y._b(Y.grad)
    gXo, gwo = O.rmsnorm_bwd(g, X, w, inv, T, D, gX0.copy())
    assert rel(gXo, host(Xn.grad)) <= TOL
    assert rel(gwo, host(wn.grad)) <= TOL


# ------------------------------------------------------------------ ropeRows
@pytest.mark.parametrize("T,nH,dH,pos0,stride", [(3, 2, 4, 0, 0), (64, 4, 16, 0, 64),
                                                  (50, 3, 8, 7, 0), (96, 2, 64, 0, 32),
                                                  (2048, 1, 64, 0, 2048)])
def test_rope_matches_oracle(T, nH, dH, pos0, stride):
    f = F()
    rng = O.RNG(6 + T)
    X, g = rng.normals(T * nH * dH), rng.normals(T * nH * dH)
    f.resetTape()
    Xn = f.param(X)
    Y = f.ropeRows(Xn, T, nH, dH, pos0, 10000, stride)
    assert rel(O.rope_fwd(X, T, nH, dH, pos0, 10000.0, stride), host(Y.data)) <= TOL
    Y.grad = g
    Y._b(Y.grad)
    assert rel(O.rope_bwd(g, T, nH, dH, pos0, 10000.0, stride), host(Xn.grad)) <= TOL


def test_slicecols_bit_exact():
    f = F()
    M, K = 17, 40
    rng = O.RNG(8)
    X, g = rng.normals(M * K), rng.normals(M * 11)
    f.resetTape()
    Xn = f.param(X)
    Y = f.sliceCols(Xn, M, K, 13, 11)
    assert np.array_equal(host(Y.data), O.slicecols_fwd(X, M, K, 13, 11))
    Y.grad = g
    Y._b(Y.grad)
    assert np.array_equal(host(Xn.grad), O.slicecols_bwd(g, M, K, 13, 11))


# ------------------------------------------------------------------ attention
@pytest.mark.parametrize("B,T,nH,nKV,dH", [(1, 4, 4, 2, 4), (1, 64, 4, 4, 16), (3, 37, 6, 2, 8),
                                          (2, 130, 4, 1, 64), (1, 1, 2, 2, 4), (2, 70, 2, 2, 128),
                                          (1, 33, 3, 3, 24)])
def test_attention_matches_oracle(B, T, nH, nKV, dH):
    f = F()
    rng = O.RNG(9 + B * T + dH)
    Q = rng.normals(B * T * nH * dH)
    K = rng.normals(B * T * nKV * dH)
    V = rng.normals(B * T * nKV * dH)
    g = rng.normals(B * T * nH * dH)
    f.resetTape()
    Qn, Kn, Vn = f.param(Q), f.param(K), f.param(V)
    Out = (f.causalAttn(Qn, Kn, Vn, T, nH, nKV, dH) if B == 1 else
           f.causalAttnBatch(Qn, Kn, Vn, B, T, nH, nKV, dH))
    Oo, P = O.attn_fwd(Q, K, V, B, T, nH, nKV, dH)
    assert rel(Oo, host(Out.data)) <= TOL
    Out.grad = g
    Out._b(Out.grad)
    gQ, gK, gV = O.attn_bwd(g, Q, K, V, P, B, T, nH, nKV, dH)
    assert rel(gQ, host(Qn.grad)) <= TOL
    assert rel(gK, host(Kn.grad)) <= TOL
    assert rel(gV, host(Vn.grad)) <= TOL


def test_attention_config4_slices():
    """B=8, Hq=32, Hkv=8, T=2048, dH=64, RoPE on Q and K,
    Q/K/V/dO ~N(0,1) from RNG(4).  GPU runs the full op; the oracle checks two
    (sequence, kv-group) slices of O, dQ, dK, dV."""
    f = F()
    B, T, nH, nKV, dH = 8, 2048, 32, 8, 64
    rng = O.RNG(4)
    Q = rng.normals(B * T * nH * dH)
    K = rng.normals(B * T * nKV * dH)
    V = rng.normals(B * T * nKV * dH)
    dO = rng.normals(B * T * nH * dH)
    f.resetTape()
    Qn, Kn, Vn = f.param(Q), f.param(K), f.param(V)
    Qr = f.ropeRows(Qn, B * T, nH, dH, 0, 10000, T)
    Kr = f.ropeRows(Kn, B * T, nKV, dH, 0, 10000, T)
    Out = f.causalAttnBatch(Qr, Kr, Vn, B, T, nH, nKV, dH)
    Out.grad = dO
    for nd in reversed(f.tape().nodes):
        if nd._b is not None and nd._grad is not None:
            nd._b(nd.grad)
    torch.cuda.synchronize()
    Og = host(Out.data).reshape(B, T, nH, dH)
    dQg = host(Qn.grad).reshape(B, T, nH, dH)
    dKg = host(Kn.grad).reshape(B, T, nKV, dH)
    dVg = host(Vn.grad).reshape(B, T, nKV, dH)
    group = nH // nKV
    O.set_threads(8)
    try:
        for b, kvh in [(0, 0), (5, 7)]:
            hs = slice(kvh * group, (kvh + 1) * group)
            q = Q.reshape(B, T, nH, dH)[b, :, hs].ravel()
            k = K.reshape(B, T, nKV, dH)[b, :, kvh].ravel()
            v = V.reshape(B, T, nKV, dH)[b, :, kvh].ravel()
            go = dO.reshape(B, T, nH, dH)[b, :, hs].ravel()
            qr = O.rope_fwd(q, T, group, dH, 0, 10000.0, T)
            kr = O.rope_fwd(k, T, 1, dH, 0, 10000.0, T)
            o, P = O.attn_fwd(qr, kr, v, 1, T, group, 1, dH)
            assert rel(o, Og[b, :, hs]) <= TOL
            gqr, gkr, gv = O.attn_bwd(go, qr, kr, v, P, 1, T, group, 1, dH)
            assert rel(O.rope_bwd(gqr, T, group, dH, 0, 10000.0, T), dQg[b, :, hs]) <= TOL
            assert rel(O.rope_bwd(gkr, T, 1, dH, 0, 10000.0, T), dKg[b, :, kvh]) <= TOL
            assert rel(gv, dVg[b, :, kvh]) <= TOL
    finally:
        O.set_threads(1)


# ------------------------------------------------------------------ swiglu / add / wsum
@pytest.mark.parametrize("n", [10, 176 * 64, 1 << 20])
def test_swiglu_matches_oracle(n):
    f = F()
    rng = O.RNG(10 + n)
    G, U, g = rng.normals(n), rng.normals(n), rng.normals(n)
    f.resetTape()
    Gn, Un = f.param(G), f.param(U)
    Y = f.swigluRows(Gn, Un, 1, n)
    Yo, sig = O.swiglu_fwd(G, U)
    assert rel(Yo, host(Y.data)) <= TOL
    Y.grad = g
    Y._b(Y.grad)
    gG, gU = O.swiglu_bwd(g, G, U, sig)
    assert rel(gG, host(Gn.grad)) <= TOL
    assert rel(gU, host(Un.grad)) <= TOL


def test_weighted_sum():
    f = F()
    rng = O.RNG(11)
    Y, t = rng.normals(1000), rng.normals(1000)
    f.resetTape()
    Yn = f.param(Y)
    s = f.weightedSum(Yn, t)
    assert abs(float(host(s.data)[0]) - float(O.wsum_fwd(Y, t))) <= 1e-5 * max(1.0, abs(float(O.wsum_fwd(Y, t))))


# ------------------------------------------------------------------ cross-entropy
@pytest.mark.parametrize("T,V", [(3, 5), (3, 6), (64, 64), (17, 1003), (9, 32000)])
def test_ce_matches_oracle(T, V):
    f = F()
    rng = O.RNG(12 + T + V)
    L = (rng.normals(T * V) * 2).astype(np.float32)
    tg = rng.ints(T, V)
    f.resetTape()
    Ln = f.param(L)
    loss = f.crossEntropyMean(Ln, tg, T, V)
    lo, probs = O.ce_fwd(L, tg, T, V)
    assert abs(float(host(loss.data)[0]) - float(lo)) <= TOL * max(1.0, abs(float(lo)))
    f.backward(loss)
    assert rel(O.ce_bwd(1.0, probs, tg, T, V), host(Ln.grad)) <= TOL


def test_ce_config3_full_size():
    """logits[8192x32000] ~N(0,2), targets U[0,32000), RNG(3)."""
    f = F()
    T, V = 8192, 32000
    rng = O.RNG(3)
    L = rng.normals(T * V, 2.0)
    tg = rng.ints(T, V)
    f.resetTape()
    Ln = f.param(L)
    loss = f.crossEntropyMean(Ln, tg, T, V)
    f.backward(loss)
    lo, probs = O.ce_fwd(L, tg, T, V)
    assert abs(float(host(loss.data)[0]) - float(lo)) <= TOL * abs(float(lo))
    gL = host(Ln.grad)
    assert rel(O.ce_bwd(1.0, probs, tg, T, V), gL) <= TOL
    # property: every gradient row sums to zero (softmax minus one-hot)
    assert np.abs(gL.reshape(T, V).astype(np.float64).sum(1)).max() < 1e-6


# ------------------------------------------------------------------ Adam
def test_adam_matches_oracle_given_same_grads():
    f = F()
    rng = O.RNG(13)
    n = 100003
    p0, g = rng.normals(n, 0.02), rng.normals(n, 1e-3)
    f.resetTape()
    P = f.param(p0.copy())
    opt = f.Adam([P], lr=3e-3, wd=0.01, totalSteps=50)
    po, m, v = p0.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    for t in range(1, 4):
        P.grad = g * t
        info = opt.step()
        io = O.adam_step(po, (g * t).astype(np.float32), m, v, t, lr=3e-3, wd=0.01, total=50)
        assert abs(info["lr"] - io["lr"]) < 1e-15
        assert abs(info["gnorm"] - io["gnorm"]) <= 1e-12 * io["gnorm"]
        got = host(P.data)
        assert np.abs(got - po).max() <= 1e-7 + 1e-6 * np.abs(po).max()


def test_adam_first_step_is_lr_on_gpu():
    """test/l2-l6.test.js:205-211 on the GPU path."""
    f = F()
    f.resetTape()
    p = f.param(np.array([1.0], np.float32))
    p.grad = np.array([1.0], np.float32)
    opt = f.Adam([p], lr=0.1, totalSteps=100)
    opt.step()
    dw = 1.0 - float(host(p.data)[0])
    assert abs(dw - 0.1) < 1e-4
    assert abs(dw - 0.1 * 0.5 * (1 + math.cos(math.pi / 100))) < 1e-6


def test_adam_clips_global_norm():
    f = F()
    f.resetTape()
    a, b = f.param(np.zeros(3, np.float32)), f.param(np.zeros(2, np.float32))
    a.grad = np.array([3.0, 0, 0], np.float32)
    b.grad = np.array([0, 4.0], np.float32)
    info = f.Adam([a, b], lr=0.1).step()
    assert abs(info["gnorm"] - 5.0) < 1e-12 and abs(info["scale"] - 0.2) < 1e-12


@pytest.mark.parametrize("V,D,T", [(50, 128, 700), (3000, 768, 4096)])
def test_embed_bwd_vectorized_bit_exact(V, D, T):
    """Widths that take the register-cached segmented sum (D a multiple of
    128): still bit-exact against the oracle's token-order scatter-add, with
    a heavy id, accumulation into an existing gradient and out-of-range ids."""
    f = F()
    rng = O.RNG(V + D)
    E = rng.normals(V * D)
    ids = rng.ints(T, V)
    ids[: T // 5] = 7
    ids[3] = -1
    ids[11] = V
    g = rng.normals(T * D)
    gE0 = rng.normals(V * D)
    f.resetTape()
    En = f.param(E)
    En.grad = gE0.copy()
    X = f.embedLookup(En, ids, V, D)
    X.grad = g
    X._b(X.grad)
    assert np.array_equal(host(En.grad), O.embed_bwd(g, ids, V, D, gE0.copy()))
