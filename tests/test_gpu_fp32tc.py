"""FCU_PREC_FP32_TC: matmulT on the tensor cores at the fp32 parity bound.

Each fp32 operand is split into three bf16 parts and the six part products
a_i b_j (i + j <= 2) run as one tcgen05 contraction six times as long, so the
tensor cores deliver fp32-level results: relL2 <= 1e-5 against the oracle's
matmulT (src/L2/tensor.js:34-52, double accumulation) for the forward, dX and
dW with their `+=` flags, on shapes the bf16 TMA path could not take (K = 5,
odd M / N: the split pads with zeros) and at BASELINE config 2.  The same
shapes run 2 split kernels + the GEMM per contraction, where the CUDA-core
mode runs one SIMT kernel.
"""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(autouse=True)
def tc_mode():
    import forgellm as F
    F.set_precision("fp32tc")
    yield
    F.set_precision("fp32")


def _call(name, *args):
    from forgellm import _lib
    from forgellm.autograd import ctx
    _lib.call(name, ctx().handle, *args)


@pytest.mark.parametrize("M,K,N", [(3, 5, 4), (37, 13, 29), (130, 256, 72), (256, 768, 1280), (1, 2048, 96)])
def test_matmulT_fp32tc_matches_oracle(M, K, N):
    rng = O.RNG(500 + M + K + N)
    X, W, g = rng.normals(M * K), rng.normals(N * K), rng.normals(M * N)
    gX0, gW0 = rng.normals(M * K), rng.normals(N * K)
    Y = O.matmulT_fwd(X, W, M, K, N)
    gX, gW = O.matmulT_bwd(g, X, W, M, K, N, gX0.copy(), gW0.copy())   # += into the given gradients
    d = {k: torch.from_numpy(v).cuda() for k, v in dict(X=X, W=W, g=g, gX=gX0, gW=gW0).items()}
    y = torch.empty(M * N, device="cuda")
    _call("fcu_matmulT_fwd", d["X"].data_ptr(), d["W"].data_ptr(), y.data_ptr(), M, K, N)
    _call("fcu_matmulT_bwd", d["g"].data_ptr(), d["X"].data_ptr(), d["W"].data_ptr(), d["gX"].data_ptr(), 1,
          d["gW"].data_ptr(), 1, M, K, N)
    torch.cuda.synchronize()
    assert O.rel_l2(Y, y.cpu().numpy()) <= TOL
    assert O.rel_l2(gX, d["gX"].cpu().numpy()) <= TOL
    assert O.rel_l2(gW, d["gW"].cpu().numpy()) <= TOL


def test_matmulT_fp32tc_config2_rows():
    """BASELINE config 2 (X 4096 x 2048, W 8192 x 2048, seed 2): the whole
    product on the GPU, 24 rows of Y / dX and 24 rows of dW against the
    oracle."""
    M, K, N = 4096, 2048, 8192
    rng = O.RNG(2)
    X, W = rng.normals(M * K), rng.normals(N * K)
    g = rng.normals(M * N)
    d = {k: torch.from_numpy(v).cuda() for k, v in dict(X=X, W=W, g=g).items()}
    y = torch.empty(M * N, device="cuda")
    gX = torch.empty(M * K, device="cuda")
    gW = torch.empty(N * K, device="cuda")
    _call("fcu_matmulT_fwd", d["X"].data_ptr(), d["W"].data_ptr(), y.data_ptr(), M, K, N)
    _call("fcu_matmulT_bwd", d["g"].data_ptr(), d["X"].data_ptr(), d["W"].data_ptr(), gX.data_ptr(), 0,
          gW.data_ptr(), 0, M, K, N)
    torch.cuda.synchronize()
    rows = np.linspace(0, M - 1, 24).astype(int)
    yh, gxh = y.cpu().numpy().reshape(M, N), gX.cpu().numpy().reshape(M, K)
    O.set_threads(16)
    try:
        for r in rows:
            x = X.reshape(M, K)[r]
            assert O.rel_l2(O.matmulT_fwd(x, W, 1, K, N), yh[r]) <= TOL
            assert O.rel_l2(O.matmulT_bwd_dx(g.reshape(M, N)[r], W, 1, K, N), gxh[r]) <= TOL
        nrows = np.linspace(0, N - 1, 24).astype(int)
        gwh = gW.cpu().numpy().reshape(N, K)
        for n in nrows:
            want = O.matmulT_bwd_dw_rows(g, X, M, K, N, int(n), int(n) + 1)
            assert O.rel_l2(want, gwh[n]) <= TOL
    finally:
        O.set_threads(1)


def test_fp32tc_runs_the_split_and_the_tensor_core_gemm():
    """One contraction launches the two split kernels and the tcgen05 GEMM
    (the CUDA-core mode launches one SIMT kernel)."""
    import forgellm as F
    from forgellm import _lib
    M, K, N = 64, 64, 64
    a = torch.randn(M * K, device="cuda")
    b = torch.randn(N * K, device="cuda")
    y = torch.empty(M * N, device="cuda")
    counts = {}
    for mode in ("fp32", "fp32tc"):
        F.set_precision(mode)
        n0 = _lib.lib().fcu_launch_count()
        _call("fcu_matmulT_fwd", a.data_ptr(), b.data_ptr(), y.data_ptr(), M, K, N)
        torch.cuda.synchronize()
        counts[mode] = _lib.lib().fcu_launch_count() - n0
    assert counts["fp32"] == 1
    assert counts["fp32tc"] >= 3
