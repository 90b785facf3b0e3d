"""fcu_ce_fwd_static: the cross-entropy forward for callers that cannot
allocate device memory.

Some hosts of this library plan every device byte before training starts (a
runtime with a fixed memory pool, or a host whose buffers are owned by a
different allocator) and may not let a library call cudaMalloc in the middle
of a step, where it can fail under memory pressure and stalls the whole
device.  fcu_ce_fwd_static does the same work as fcu_ce_fwd with its per-row
scratch in a fixed array built into the library.

The tests call both entry points straight through the C-ABI, twice in a row
with different inputs, and require the same loss and gradient (relL2 <= 1e-5,
the parity tolerance of the other GPU tests); one case is also checked
against the CPU oracle's crossEntropyMean.  A context that only ever runs the
static entry point must hold no scratch afterwards, and the device's free
memory must not move across a call.  Every visible GPU is exercised (the
array's address is looked up once per device).  The file name makes pytest
collect it last.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


def _rel(ref, got):
    ref = np.asarray(ref, np.float64).ravel()
    got = np.asarray(got, np.float64).ravel()
    return float(np.linalg.norm(ref - got) / max(np.linalg.norm(ref), 1e-30))


def _devices():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return list(range(min(n, 2))) or [0]


@pytest.fixture(scope="module")
def L():
    from forgellm import _lib
    return _lib.lib()


def _ctx(L, dev):
    h = ctypes.c_void_p()
    assert L.fcu_ctx_create(dev, ctypes.byref(h)) == 0, L.fcu_last_error()
    return h


def _scratch(L, h):
    n = ctypes.c_size_t(123)
    assert L.fcu_ctx_scratch_bytes(h, ctypes.byref(n)) == 0
    return n.value


@pytest.mark.parametrize("dev", _devices())
@pytest.mark.parametrize("T,V", [(37, 1003), (4096, 32000)])
def test_static_scratch_ce_matches_fcu_ce_fwd(L, dev, T, V):
    torch.cuda.set_device(dev)
    stat = _ctx(L, dev)    # runs only the static entry point
    ref = _ctx(L, dev)     # runs fcu_ce_fwd (allocates its scratch)
    try:
        stream = torch.cuda.current_stream()
        for h in (stat, ref):
            assert L.fcu_ctx_set_stream(h, ctypes.c_void_p(stream.cuda_stream)) == 0
        gen = torch.Generator(device=f"cuda:{dev}").manual_seed(T + V)
        for call in range(2):   # two calls in a row: the shared array keeps no state that matters
            logits = torch.randn(T * V, device=f"cuda:{dev}", generator=gen) * (2.0 + call)
            targets = torch.randint(0, V, (T,), device=f"cuda:{dev}", dtype=torch.int32, generator=gen)
            loss_a = torch.empty(1, device=f"cuda:{dev}")
            loss_b = torch.empty(1, device=f"cuda:{dev}")
            d_a = torch.empty(T * V, device=f"cuda:{dev}")
            d_b = torch.empty(T * V, device=f"cuda:{dev}")
            assert L.fcu_ce_fwd(ref, logits.data_ptr(), targets.data_ptr(), T, V, loss_a.data_ptr(),
                                d_a.data_ptr()) == 0, L.fcu_last_error()
            torch.cuda.synchronize()
            free0 = torch.cuda.mem_get_info(dev)[0]
            assert L.fcu_ce_fwd_static(stat, logits.data_ptr(), targets.data_ptr(), T, V,
                                       loss_b.data_ptr(), d_b.data_ptr()) == 0, L.fcu_last_error()
            torch.cuda.synchronize()
            if call:   # the first call may still load the library's code on this device
                assert torch.cuda.mem_get_info(dev)[0] == free0
            assert _scratch(L, stat) == 0
            la, lb = float(loss_a.item()), float(loss_b.item())
            assert abs(la - lb) <= TOL * abs(la), (call, la, lb)
            assert _rel(d_a.cpu().numpy(), d_b.cpu().numpy()) <= TOL, call
        assert _scratch(L, ref) > 0
    finally:
        torch.cuda.synchronize()
        L.fcu_ctx_destroy(stat)
        L.fcu_ctx_destroy(ref)


def test_static_scratch_ce_matches_oracle(L):
    """The static entry point against the CPU restatement of crossEntropyMean
    (src/L2/tensor.js:393-417): loss and (P - onehot)/T."""
    import oracle as O
    T, V = 19, 517
    rng = O.RNG(3)
    logits = (2.0 * rng.normals(T * V)).astype(np.float32)
    targets = rng.ints(T, V).astype(np.int32)
    want_loss, probs = O.ce_fwd(logits, targets, T, V)
    want_grad = O.ce_bwd(1.0, probs, targets, T, V)
    torch.cuda.set_device(0)
    h = _ctx(L, 0)
    try:
        stream = torch.cuda.current_stream()
        assert L.fcu_ctx_set_stream(h, ctypes.c_void_p(stream.cuda_stream)) == 0
        lg = torch.from_numpy(logits).cuda()
        tg = torch.from_numpy(targets).cuda()
        loss = torch.empty(1, device="cuda")
        du = torch.empty(T * V, device="cuda")
        for _ in range(2):
            du.fill_(7.0)
            assert L.fcu_ce_fwd_static(h, lg.data_ptr(), tg.data_ptr(), T, V, loss.data_ptr(),
                                       du.data_ptr()) == 0, L.fcu_last_error()
            torch.cuda.synchronize()
            assert abs(float(loss.item()) - float(want_loss)) <= TOL * abs(float(want_loss))
            assert _rel(want_grad, du.cpu().numpy()) <= TOL
        assert _scratch(L, h) == 0
    finally:
        torch.cuda.synchronize()
        L.fcu_ctx_destroy(h)


def test_static_scratch_ce_rejects_too_many_rows(L):
    torch.cuda.set_device(0)
    h = _ctx(L, 0)
    try:
        T, V = 65537, 4
        buf = torch.zeros(T * V, device="cuda")
        tg = torch.zeros(T, device="cuda", dtype=torch.int32)
        loss = torch.empty(1, device="cuda")
        rc = L.fcu_ce_fwd_static(h, buf.data_ptr(), tg.data_ptr(), T, V, loss.data_ptr(),
                                 buf.data_ptr())
        assert rc != 0
        assert b"65536" in L.fcu_last_error()
    finally:
        L.fcu_ctx_destroy(h)
