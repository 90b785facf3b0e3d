"""Tensor-core (tcgen05) matmulT in FCU_PREC_BF16 mode.

Two bars:
  * exactness of the kernel: against a float64 product of the SAME
    bf16-rounded operands, so only the fp32 accumulation order differs --
    relL2 <= 1e-5;
  * the stated bf16-mode bound against the fp32 oracle: relL2 <= 1e-2
    (bf16 keeps 8 mantissa bits; random-sign inputs land near 3e-3).
"""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

EXACT = 1e-5
BF16_BOUND = 1e-2


@pytest.fixture(autouse=True)
def bf16_mode():
    import forgellm as F
    F.set_precision("bf16")
    yield
    F.set_precision("fp32")


def bf16_round(a):
    """Round float32 to the nearest bf16 (ties to even), kept as float32."""
    u = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def host(t):
    return t.detach().float().cpu().numpy().ravel()


def relf(ref, got):
    ref = np.asarray(ref, np.float64).ravel()
    got = np.asarray(got, np.float64).ravel()
    return float(np.linalg.norm(ref - got) / max(np.linalg.norm(ref), 1e-30))


def device_ok():
    from forgellm import _lib
    from forgellm.autograd import ctx
    assert _lib.lib().fcu_check_device_error(ctx().handle) == 0, _lib.lib().fcu_last_error()


@pytest.mark.parametrize("M,K,N", [(128, 64, 256), (300, 200, 520), (1, 8, 8), (129, 1024, 257),
                                   (1024, 768, 1280), (4096, 2048, 8192)])
def test_tc_matmulT_fwd_bwd(M, K, N):
    import forgellm as F
    rng = np.random.default_rng(M * 7 + K * 3 + N)
    X = rng.standard_normal(M * K).astype(np.float32)
    W = rng.standard_normal(N * K).astype(np.float32)
    g = rng.standard_normal(M * N).astype(np.float32)
    gX0 = rng.standard_normal(M * K).astype(np.float32)
    F.resetTape()
    Xn, Wn = F.param(X), F.param(W)
    Xn.grad = gX0.copy()                      # dX accumulates, dW overwrites
    Y = F.matmulT(Xn, Wn, M, K, N)
    Y.grad = g
    Y._b(Y.grad)
    torch.cuda.synchronize()
    device_ok()
    # Which contractions the tensor cores take (16-byte TMA row strides);
    # the others run the fp32 CUDA-core kernel on unrounded operands.
    tc_fwd, tc_dx, tc_dw = K % 8 == 0, K % 8 == 0 and N % 8 == 0, N % 8 == 0 and K % 8 == 0
    r = lambda a, on: bf16_round(a).astype(np.float64) if on else a.astype(np.float64)  # noqa: E731
    rows = np.arange(M) if M <= 1024 else np.random.default_rng(0).choice(M, 64, replace=False)
    cols = np.arange(N) if N <= 1024 else np.random.default_rng(1).choice(N, 64, replace=False)
    Yg = host(Y.data).reshape(M, N)
    Xb, Wb = r(X, tc_fwd).reshape(M, K), r(W, tc_fwd).reshape(N, K)
    assert relf(Xb[rows] @ Wb.T, Yg[rows]) <= EXACT
    dXg = host(Xn.grad).reshape(M, K)
    gb, Wb = r(g, tc_dx).reshape(M, N), r(W, tc_dx).reshape(N, K)
    assert relf(gX0.reshape(M, K)[rows] + gb[rows] @ Wb, dXg[rows]) <= EXACT
    dWg = host(Wn.grad).reshape(N, K)
    gb, Xb = r(g, tc_dw).reshape(M, N), r(X, tc_dw).reshape(M, K)
    assert relf(gb[:, cols].T @ Xb, dWg[cols]) <= EXACT
    # stated bf16 bound against the unrounded fp32 product
    Xf, Wf = X.reshape(M, K).astype(np.float64), W.reshape(N, K).astype(np.float64)
    assert relf(Xf[rows] @ Wf.T, Yg[rows]) <= BF16_BOUND


def test_tc_fallback_for_unaligned_shapes():
    """Row lengths that are not multiples of 8 elements cannot be TMA tiled;
    they take the CUDA-core kernel (fp32 exact) instead."""
    import forgellm as F
    M, K, N = 33, 5, 7
    rng = O.RNG(77)
    X, W = rng.normals(M * K), rng.normals(N * K)
    F.resetTape()
    Y = F.matmulT(F.param(X), F.param(W), M, K, N)
    assert O.rel_l2(O.matmulT_fwd(X, W, M, K, N), host(Y.data)) <= 1e-5


def test_tc_repeated_calls_are_deterministic():
    import forgellm as F
    M, K, N = 512, 768, 2048
    rng = np.random.default_rng(5)
    X = rng.standard_normal(M * K).astype(np.float32)
    W = rng.standard_normal(N * K).astype(np.float32)
    outs = []
    for _ in range(3):
        F.resetTape()
        outs.append(host(F.matmulT(F.param(X), F.param(W), M, K, N).data))
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])
    device_ok()


# ------------------------------------------------------------------ fcu_gemm_bf16 output modes
@pytest.mark.parametrize("op,M,N,K", [(0, 128, 256, 4096),     # 1 tile, K long: split-K
                                      (0, 300, 520, 768),      # no split, ragged tiles
                                      (2, 256, 128, 8192),     # dW layout, split-K
                                      (1, 200, 256, 4096)])    # dX layout, split-K
@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4])
def test_gemm_bf16_output_modes(op, M, N, K, mode):
    """Every epilogue (fp32 / fp32 + residual / bf16 / bf16 + RoPE, and fp32
    accumulating into the output as mode 4), with and without split-K,
    against a float64 product of the same bf16 operands."""
    accumulate = 1 if mode == 4 else 0
    mode = 0 if mode == 4 else mode
    import ctypes
    from forgellm import _lib
    from forgellm.autograd import ctx
    g = torch.Generator(device="cuda").manual_seed(op * 100 + mode)
    na = M * K if op != 2 else K * M
    nb = N * K if op == 0 else K * N
    A = torch.randn(na, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(nb, device="cuda", generator=g).to(torch.bfloat16)
    Ad, Bd = A.double().cpu(), B.double().cpu()
    if op == 0:
        ref = Ad.view(M, K) @ Bd.view(N, K).T
    elif op == 1:
        ref = Ad.view(M, K) @ Bd.view(K, N)
    else:
        ref = Ad.view(K, M).T @ Bd.view(K, N)
    R = torch.randn(M * N, device="cuda", generator=g)
    out = torch.zeros(M * N, device="cuda", dtype=torch.float32 if mode < 2 else torch.bfloat16)
    if accumulate:
        out.normal_(generator=g)
    out0 = out.double().cpu().view(M, N)
    T_rope, hd, rc = 64, 64, 128
    o = _lib.GemmOut(mode, out.data_ptr(), accumulate, R.data_ptr() if mode == 1 else None,
                     T_rope if mode == 3 else 0, rc if mode == 3 else 0, hd if mode == 3 else 0,
                     10000.0 if mode == 3 else 0.0)
    _lib.call("fcu_gemm_bf16", ctx().handle, op, A.data_ptr(), B.data_ptr(), M, N, K, ctypes.byref(o))
    torch.cuda.synchronize()
    device_ok()
    want = ref.clone()
    if accumulate:
        want += out0
    if mode == 1:
        want += R.double().cpu().view(M, N)
    if mode == 3:
        import math
        w = want.numpy()
        for m in range(M):
            pos = m % T_rope
            for c in range(0, min(rc, N), 2):
                i = (c % hd) // 2
                ang = pos / math.pow(10000.0, 2 * i / hd)
                cs, sn = math.cos(ang), math.sin(ang)
                a, b = w[m, c], w[m, c + 1]
                w[m, c], w[m, c + 1] = a * cs - b * sn, a * sn + b * cs
        want = torch.from_numpy(w)
    got = out.double().cpu().view(M, N)
    tol = EXACT if mode < 2 else 5e-3          # bf16 outputs carry their own rounding
    assert relf(want.numpy(), got.numpy()) <= tol


@pytest.mark.parametrize("op,M,N,K", [(2, 768, 768, 8192), (2, 4096, 768, 8192), (1, 8192, 768, 32000)])
def test_gemm_split_k_repeats_bit_exactly(op, M, N, K):
    """Split-K products (the weight-gradient and LM-head input-gradient shapes
    of a batch-8 step): five launches in a row give the same bits, the output
    matches float64 of the same bf16 operands, and an accumulating launch
    adds exactly the product once more."""
    import ctypes
    from forgellm import _lib
    from forgellm.autograd import ctx
    g = torch.Generator(device="cuda").manual_seed(M + N)
    A = (torch.randn(M * K, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    B = (torch.randn(N * K, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    out = torch.empty(M * N, device="cuda")
    h = ctx().handle
    outs = []
    for _ in range(5):
        out.fill_(float("nan"))
        o = _lib.GemmOut(0, out.data_ptr(), 0, None, 0, 0, 0, 0.0)
        _lib.call("fcu_gemm_bf16", h, op, A.data_ptr(), B.data_ptr(), M, N, K, ctypes.byref(o))
        torch.cuda.synchronize()
        outs.append(out.clone())
    device_ok()
    for x in outs[1:]:
        assert torch.equal(x, outs[0])
    Ad, Bd = A.double(), B.double()
    if op == 1:
        ref = Ad.view(M, K) @ Bd.view(K, N)
    else:
        ref = Ad.view(K, M).T @ Bd.view(K, N)
    # the tensor cores' fp32 accumulation is not round-to-nearest: 1.8e-5
    # relL2 measured over the 32,000-term contraction, within 1e-5 at 8,192
    tol = EXACT if K <= 8192 else 4e-5
    assert relf(ref.cpu().numpy(), out.double().view(M, N).cpu().numpy()) <= tol
    o = _lib.GemmOut(0, out.data_ptr(), 1, None, 0, 0, 0, 0.0)
    _lib.call("fcu_gemm_bf16", h, op, A.data_ptr(), B.data_ptr(), M, N, K, ctypes.byref(o))
    torch.cuda.synchronize()
    assert torch.equal(out, outs[0] + outs[0])


def _gemm_out(mode, out, out2=None, aux=None):
    from forgellm import _lib
    return _lib.GemmOut(mode, out.data_ptr(), 0, None, 0, 0, 0, 0.0,
                        out2.data_ptr() if out2 is not None else None,
                        aux.data_ptr() if aux is not None else None)


@pytest.mark.parametrize("M,H,K", [(256, 128, 64), (333, 384, 96), (1000, 2048, 768)])
def test_gemm_swiglu_epilogue_is_bit_identical(M, H, K):
    """FCU_OUT_BF16_SWIGLU (gate|up GEMM with swigluRows in the epilogue)
    writes exactly what the bf16 GEMM followed by fcu_swiglu_fwd_bf16 writes,
    ragged row counts included."""
    import ctypes
    from forgellm import _lib
    from forgellm.autograd import ctx
    h = ctx().handle
    g = torch.Generator(device="cuda").manual_seed(M + H + K)
    A = torch.randn(M * K, device="cuda", generator=g).to(torch.bfloat16)
    B = (0.3 * torch.randn(2 * H * K, device="cuda", generator=g)).to(torch.bfloat16)
    gu = torch.zeros(M * 2 * H, device="cuda", dtype=torch.bfloat16)
    act = torch.zeros(M * H, device="cuda", dtype=torch.bfloat16)
    _lib.call("fcu_gemm_bf16", h, 0, A.data_ptr(), B.data_ptr(), M, 2 * H, K,
              ctypes.byref(_gemm_out(_lib.OUT_BF16, gu)))
    _lib.call("fcu_swiglu_fwd_bf16", h, gu.data_ptr(), M, H, act.data_ptr())
    gu2 = torch.full_like(gu, 7.0)
    act2 = torch.full_like(act, 7.0)
    _lib.call("fcu_gemm_bf16", h, 0, A.data_ptr(), B.data_ptr(), M, 2 * H, K,
              ctypes.byref(_gemm_out(_lib.OUT_BF16_SWIGLU, gu2, out2=act2)))
    torch.cuda.synchronize()
    device_ok()
    assert torch.equal(gu, gu2)
    assert torch.equal(act, act2)
    # and the product itself is right
    ref = A.double().view(M, K) @ B.double().view(2 * H, K).T
    assert relf(ref.cpu().numpy(), gu.double().cpu().view(M, 2 * H).numpy()) <= 5e-3


@pytest.mark.parametrize("M,H,K", [(256, 128, 64), (333, 192, 96), (1000, 2048, 768)])
def test_gemm_swiglu_bwd_epilogue_is_bit_identical(M, H, K):
    """FCU_OUT_BF16_SWIGLU_BWD (down-projection input gradient with the
    swigluRows backward in the epilogue) writes exactly what the bf16 dX GEMM
    followed by fcu_swiglu_bwd_bf16 writes."""
    import ctypes
    from forgellm import _lib
    from forgellm.autograd import ctx
    h = ctx().handle
    g = torch.Generator(device="cuda").manual_seed(7 * M + H + K)
    dY = torch.randn(M * K, device="cuda", generator=g).to(torch.bfloat16)
    W = (0.3 * torch.randn(K * H, device="cuda", generator=g)).to(torch.bfloat16)
    gu = (2 * torch.randn(M * 2 * H, device="cuda", generator=g)).to(torch.bfloat16)
    dact = torch.zeros(M * H, device="cuda", dtype=torch.bfloat16)
    dgu = torch.zeros(M * 2 * H, device="cuda", dtype=torch.bfloat16)
    _lib.call("fcu_gemm_bf16", h, 1, dY.data_ptr(), W.data_ptr(), M, H, K,
              ctypes.byref(_gemm_out(_lib.OUT_BF16, dact)))
    _lib.call("fcu_swiglu_bwd_bf16", h, dact.data_ptr(), gu.data_ptr(), M, H, dgu.data_ptr())
    dgu2 = torch.full_like(dgu, 7.0)
    _lib.call("fcu_gemm_bf16", h, 1, dY.data_ptr(), W.data_ptr(), M, H, K,
              ctypes.byref(_gemm_out(_lib.OUT_BF16_SWIGLU_BWD, dgu2, aux=gu)))
    torch.cuda.synchronize()
    device_ok()
    assert torch.equal(dgu, dgu2)
    assert bool(torch.isfinite(dgu2.float()).all())


def test_gemm_swiglu_modes_reject_bad_shapes():
    import ctypes
    from forgellm import _lib
    from forgellm.autograd import ctx
    h = ctx().handle
    A = torch.zeros(128 * 64, device="cuda", dtype=torch.bfloat16)
    B = torch.zeros(192 * 64, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(128 * 192, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(F_error()):   # N = 2H = 192: H is not a multiple of 128
        _lib.call("fcu_gemm_bf16", h, 0, A.data_ptr(), B.data_ptr(), 128, 192, 64,
                  ctypes.byref(_gemm_out(_lib.OUT_BF16_SWIGLU, out, out2=out)))
    with pytest.raises(F_error()):   # no forward values
        _lib.call("fcu_gemm_bf16", h, 1, A.data_ptr(), B.data_ptr(), 128, 192, 64,
                  ctypes.byref(_gemm_out(_lib.OUT_BF16_SWIGLU_BWD, out)))
    device_ok()


def F_error():
    from forgellm import ForgeCUError
    return ForgeCUError


# ------------------------------------------------------------------ attention (bf16 mode)
ATTN_BF16_BOUND = 2e-2   # bf16 Q/K/V/P/dS operands, fp32 softmax and accumulation


@pytest.mark.parametrize("B,T,nH,nKV,dH", [(1, 64, 4, 4, 16), (2, 130, 4, 1, 64), (3, 100, 6, 2, 32),
                                          (1, 257, 2, 2, 128), (2, 1024, 12, 4, 64), (2, 300, 8, 2, 128)])
def test_tc_attention_bf16_bound(B, T, nH, nKV, dH):
    import forgellm as F
    rng = O.RNG(31 + B * T + dH)
    Q = rng.normals(B * T * nH * dH)
    K = rng.normals(B * T * nKV * dH)
    V = rng.normals(B * T * nKV * dH)
    g = rng.normals(B * T * nH * dH)
    F.resetTape()
    Qn, Kn, Vn = F.param(Q), F.param(K), F.param(V)
    Out = F.causalAttnBatch(Qn, Kn, Vn, B, T, nH, nKV, dH)
    Out.grad = g
    Out._b(Out.grad)
    torch.cuda.synchronize()
    if B * T > 512:   # oracle on the first sequence only
        sl = lambda a, h: a.reshape(B, T, h, dH)[0].ravel()  # noqa: E731
        Qs, Ks, Vs, gs = sl(Q, nH), sl(K, nKV), sl(V, nKV), sl(g, nH)
        Bo = 1
    else:
        Qs, Ks, Vs, gs, Bo = Q, K, V, g, B
        sl = lambda a, h: a  # noqa: E731
    Oo, P = O.attn_fwd(Qs, Ks, Vs, Bo, T, nH, nKV, dH)
    gQ, gK, gV = O.attn_bwd(gs, Qs, Ks, Vs, P, Bo, T, nH, nKV, dH)
    errs = {
        "O": O.rel_l2(Oo, sl(host(Out.data), nH)),
        "dQ": O.rel_l2(gQ, sl(host(Qn.grad), nH)),
        "dK": O.rel_l2(gK, sl(host(Kn.grad), nKV)),
        "dV": O.rel_l2(gV, sl(host(Vn.grad), nKV)),
    }
    assert max(errs.values()) <= ATTN_BF16_BOUND, errs
    assert errs["O"] <= 1e-2, errs


# ------------------------------------------------------------------ fcu_attn_fwd_bf16 (fused-path entry)
def _attn_ref64(qkv, B, T, nH, nKV, dH):
    """float64 causal GQA attention of the same bf16 q/k/v: (O [B*T, nH*dH], lse [B, nH, T])."""
    x = qkv.double().view(B, T, -1)
    q = x[..., :nH * dH].view(B, T, nH, dH).permute(0, 2, 1, 3)
    k = x[..., nH * dH:(nH + nKV) * dH].view(B, T, nKV, dH).permute(0, 2, 1, 3)
    v = x[..., (nH + nKV) * dH:(nH + 2 * nKV) * dH].view(B, T, nKV, dH).permute(0, 2, 1, 3)
    g = nH // nKV
    k, v = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
    s = q @ k.transpose(-1, -2) / dH ** 0.5
    s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool, device=s.device), 1), float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1) @ v
    return o.permute(0, 2, 1, 3).reshape(B * T, nH * dH), lse


@pytest.mark.parametrize("B,T,nH,nKV,extra,dH", [(1, 64, 2, 2, 0, 64), (2, 130, 4, 1, 0, 64), (3, 300, 6, 2, 64, 64),
                                                 (2, 1024, 12, 4, 0, 64), (1, 2048, 32, 8, 0, 64),
                                                 (1, 64, 4, 4, 0, 16), (2, 130, 4, 1, 8, 16),
                                                 (3, 300, 6, 2, 64, 32), (2, 1024, 12, 4, 0, 32),
                                                 (2, 130, 4, 1, 0, 128), (3, 300, 6, 2, 128, 128),
                                                 (1, 2048, 16, 4, 0, 128)])
def test_attn_fwd_bf16_entry(B, T, nH, nKV, extra, dH):
    """The fused path's attention forward (bf16 qkv in, bf16 O + fp32 lse out)
    against float64 attention of the same bf16 inputs: only P's and O's bf16
    rounding differ (relL2 <= 1e-2), the log-sum-exp to 1e-5.  Head dims 16
    and 32 run the same tcgen05 kernels on zero-padded 64-column heads, head
    dim 128 the forward kernel's 128-column instantiation."""
    from forgellm import _lib
    from forgellm.autograd import ctx
    width = (nH + 2 * nKV) * dH
    ld = width + extra
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + T)
    qkv = (torch.randn(B * T, ld, device="cuda", generator=g) * 1.5).to(torch.bfloat16)
    O = torch.full((B * T, nH * dH), float("nan"), device="cuda").to(torch.bfloat16)
    lse = torch.full((B * nH * T,), float("nan"), device="cuda")
    outs = []
    for _ in range(2):
        _lib.call("fcu_attn_fwd_bf16", ctx().handle, qkv.data_ptr(), ld, B, T, nH, nKV, dH,
                  O.data_ptr(), lse.data_ptr())
        torch.cuda.synchronize()
        outs.append((O.clone(), lse.clone()))
    device_ok()
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    o_ref, lse_ref = _attn_ref64(qkv[:, :width], B, T, nH, nKV, dH)
    assert torch.isfinite(O.float()).all() and torch.isfinite(lse).all()
    assert relf(o_ref.cpu().numpy(), O.double().cpu().numpy()) <= 1e-2
    assert float((lse.double().view(B, nH, T) - lse_ref).abs().max()) <= 1e-4


def _rope_back64(d, B, T, heads, dH, theta):
    """Rotate per-head interleaved pairs of d [B*T, heads*dH] back by R^T (float64)."""
    pos = torch.arange(T, dtype=torch.float64, device=d.device).repeat(B)
    i = torch.arange(dH // 2, dtype=torch.float64, device=d.device)
    ang = pos[:, None] / theta ** (2 * i / dH)[None, :]
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    x = d.view(B * T, heads, dH // 2, 2)
    a, b = x[..., 0], x[..., 1]
    return torch.stack((a * c + b * s, -a * s + b * c), -1).reshape(B * T, heads * dH)


@pytest.mark.parametrize("B,T,nH,nKV,theta,dH", [(1, 64, 2, 2, 0.0, 64), (2, 130, 4, 1, 10000.0, 64),
                                                 (3, 300, 6, 2, 10000.0, 64), (2, 1024, 12, 4, 10000.0, 64),
                                                 (16, 1024, 12, 4, 10000.0, 64), (40, 512, 12, 4, 10000.0, 64),
                                                 (1, 2048, 32, 8, 10000.0, 64),
                                                 (1, 64, 4, 4, 10000.0, 16), (2, 130, 4, 1, 0.0, 16),
                                                 (3, 300, 6, 2, 10000.0, 32), (16, 256, 12, 4, 10000.0, 32),
                                                 (2, 130, 4, 2, 10000.0, 128), (3, 300, 4, 4, 0.0, 128),
                                                 (8, 1024, 8, 2, 10000.0, 128), (1, 2048, 16, 4, 10000.0, 128),
                                                 (64, 512, 8, 4, 10000.0, 128)])
def test_attn_bwd_bf16_entry(B, T, nH, nKV, theta, dH):
    """The fused path's attention backward (dq | dk | dv into the bf16 dqkv
    buffer, RoPE rotated back) against float64 autograd of the same bf16
    inputs: relL2 <= 2e-2 (P and dS are bf16 operands), every gradient finite.
    Head dims 16 and 32 run on zero-padded 64-column heads; head dim 128 on
    the 128-wide tcgen05 kernels (dV / dK in two 64-column halves), with one
    CTA per kv head and, for few sequences, one per q head (head split)."""
    from forgellm import _lib
    from forgellm.autograd import ctx
    width = (nH + 2 * nKV) * dH
    g = torch.Generator(device="cuda").manual_seed(B * 77 + T)
    qkv = torch.randn(B * T, width, device="cuda", generator=g).to(torch.bfloat16)
    dO = torch.randn(B * T, nH * dH, device="cuda", generator=g).to(torch.bfloat16)
    O = torch.empty(B * T, nH * dH, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * nH * T, device="cuda")
    h = ctx().handle
    _lib.call("fcu_attn_fwd_bf16", h, qkv.data_ptr(), width, B, T, nH, nKV, dH, O.data_ptr(), lse.data_ptr())
    dqkv = torch.full((B * T, width), float("nan"), device="cuda").to(torch.bfloat16)
    outs = []
    for _ in range(2):
        _lib.call("fcu_attn_bwd_bf16", h, dO.data_ptr(), qkv.data_ptr(), width, O.data_ptr(),
                  lse.data_ptr(), B, T, nH, nKV, dH, theta, dqkv.data_ptr())
        torch.cuda.synchronize()
        outs.append(dqkv.clone())
    device_ok()
    assert torch.equal(outs[0], outs[1])                     # deterministic
    x = qkv.double().requires_grad_(True)
    o_ref, _ = _attn_ref64(x, B, T, nH, nKV, dH)
    o_ref.backward(dO.double())
    ref = x.grad
    qD, kD = nH * dH, nKV * dH
    if theta > 0:
        ref = torch.cat((_rope_back64(ref[:, :qD], B, T, nH, dH, theta),
                         _rope_back64(ref[:, qD:qD + kD], B, T, nKV, dH, theta), ref[:, qD + kD:]), 1)
    got = dqkv.double()
    assert torch.isfinite(got).all()
    for name, sl in (("dq", slice(0, qD)), ("dk", slice(qD, qD + kD)), ("dv", slice(qD + kD, width))):
        err = relf(ref[:, sl].cpu().numpy(), got[:, sl].cpu().numpy())
        assert err <= 2e-2, (name, err)


@pytest.mark.parametrize("dH", [64, 32, 16, 128])
def test_tc_attention_operator_accumulates_on_tcgen05(dH):
    """causalAttnBatch in bf16 mode runs the tcgen05 kernels on packed bf16
    copies of its fp32 operands (heads below 64 columns zero-padded); its
    backward follows the JS `grad +=`: a second backward without zeroing
    doubles every gradient exactly (the packed gradient is deterministic)."""
    from forgellm import _lib
    from forgellm.autograd import ctx
    B, T, nH, nKV = 2, 200, 6, 2
    rng = O.RNG(77)
    q, k, v, g = (torch.from_numpy(rng.normals(B * T * h * dH)).cuda() for h in (nH, nKV, nKV, nH))
    o = torch.empty(B * T * nH * dH, device="cuda")
    lse = torch.empty(B * nH * T, device="cuda")
    grads = [torch.zeros(B * T * h * dH, device="cuda") for h in (nH, nKV, nKV)]
    h = ctx().handle
    _lib.call("fcu_attn_fwd", h, q.data_ptr(), k.data_ptr(), v.data_ptr(), B, T, nH, nKV, dH, o.data_ptr(),
              lse.data_ptr())
    snaps = []
    for acc in (0, 1):
        _lib.call("fcu_attn_bwd", h, g.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                  lse.data_ptr(), B, T, nH, nKV, dH, *(t.data_ptr() for t in grads), acc)
        torch.cuda.synchronize()
        snaps.append([t.clone() for t in grads])
    device_ok()
    for one, two in zip(*snaps):
        assert torch.isfinite(one).all()
        assert torch.equal(two, 2 * one)


# ------------------------------------------------------------------ CTA-pair (cta_group::2) tiles
def _gemm_case(op, M, N, K, mode, accumulate, seed):
    """Operands and a float64 reference for one fcu_gemm_bf16 call."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    na = M * K if op != 2 else K * M
    nb = N * K if op == 0 else K * N
    A = torch.randn(na, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(nb, device="cuda", generator=g).to(torch.bfloat16)
    R = torch.randn(M * N, device="cuda", generator=g)
    out0 = torch.randn(M * N, device="cuda", generator=g)
    Ad, Bd = A.double().cpu(), B.double().cpu()
    if op == 0:
        ref = Ad.view(M, K) @ Bd.view(N, K).T
    elif op == 1:
        ref = Ad.view(M, K) @ Bd.view(K, N)
    else:
        ref = Ad.view(K, M).T @ Bd.view(K, N)
    if accumulate:
        ref += out0.double().cpu().view(M, N)
    if mode == 1:
        ref += R.double().cpu().view(M, N)
    return A, B, R, out0, ref


@pytest.mark.parametrize("op,M,N,K", [(0, 300, 520, 768),      # ragged rows and columns
                                      (0, 1000, 1280, 768),
                                      (1, 513, 768, 1024),     # dX layout: B MN-major
                                      (2, 768, 512, 1024),     # dW layout: A and B MN-major
                                      (0, 200, 256, 64)])      # second CTA of the pair past M
@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4])
def test_gemm_pair_tile_matches_single_cta(op, M, N, K, mode, monkeypatch):
    """The 256 x 256 CTA-pair tile (FORGECU_GEMM_PAIR=1) writes the same bits
    as the single-CTA tiles (=0) in every output mode, and both match float64
    of the same bf16 operands."""
    import ctypes
    from forgellm import _lib
    from forgellm.autograd import ctx
    accumulate = 1 if mode == 4 else 0
    mode = 0 if mode == 4 else mode
    A, B, R, out0, ref = _gemm_case(op, M, N, K, mode, accumulate, 31 * op + 7 * mode + M)
    T_rope, hd, rc = 64, 64, 128
    outs = {}
    for setting in ("0", "1"):
        monkeypatch.setenv("FORGECU_GEMM_PAIR", setting)
        out = out0.clone() if mode < 2 else torch.zeros(M * N, device="cuda", dtype=torch.bfloat16)
        o = _lib.GemmOut(mode, out.data_ptr(), accumulate, R.data_ptr() if mode == 1 else None,
                         T_rope if mode == 3 else 0, rc if mode == 3 else 0, hd if mode == 3 else 0,
                         10000.0 if mode == 3 else 0.0)
        _lib.call("fcu_gemm_bf16", ctx().handle, op, A.data_ptr(), B.data_ptr(), M, N, K, ctypes.byref(o))
        torch.cuda.synchronize()
        device_ok()
        outs[setting] = out
    assert torch.equal(outs["0"], outs["1"])
    if mode < 2:
        assert relf(ref.numpy(), outs["1"].double().cpu().view(M, N).numpy()) <= EXACT


@pytest.mark.parametrize("M,H,K", [(333, 384, 96), (1000, 2048, 768)])
def test_gemm_pair_tile_swiglu_epilogues(M, H, K, monkeypatch):
    """Both SwiGLU epilogues on the CTA-pair tile (rank 0 stages the gate
    rows, rank 1 the up rows) write what the single-CTA tiles write."""
    import ctypes
    from forgellm import _lib
    from forgellm.autograd import ctx
    h = ctx().handle
    g = torch.Generator(device="cuda").manual_seed(3 * M + H + K)
    A = torch.randn(M * K, device="cuda", generator=g).to(torch.bfloat16)
    B = (0.3 * torch.randn(2 * H * K, device="cuda", generator=g)).to(torch.bfloat16)
    W = (0.3 * torch.randn(K * H, device="cuda", generator=g)).to(torch.bfloat16)
    res = {}
    for setting in ("0", "1"):
        monkeypatch.setenv("FORGECU_GEMM_PAIR", setting)
        gu = torch.full((M * 2 * H,), 7.0, device="cuda", dtype=torch.bfloat16)
        act = torch.full((M * H,), 7.0, device="cuda", dtype=torch.bfloat16)
        dgu = torch.full((M * 2 * H,), 7.0, device="cuda", dtype=torch.bfloat16)
        _lib.call("fcu_gemm_bf16", h, 0, A.data_ptr(), B.data_ptr(), M, 2 * H, K,
                  ctypes.byref(_gemm_out(_lib.OUT_BF16_SWIGLU, gu, out2=act)))
        _lib.call("fcu_gemm_bf16", h, 1, A.data_ptr(), W.data_ptr(), M, H, K,
                  ctypes.byref(_gemm_out(_lib.OUT_BF16_SWIGLU_BWD, dgu, aux=gu)))
        torch.cuda.synchronize()
        device_ok()
        res[setting] = (gu, act, dgu)
    for a, b in zip(res["0"], res["1"]):
        assert torch.equal(a, b)
    ref = A.double().view(M, K) @ B.double().view(2 * H, K).T
    assert relf(ref.cpu().numpy(), res["1"][0].double().cpu().view(M, 2 * H).numpy()) <= 5e-3
