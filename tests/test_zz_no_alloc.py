"""fcu_ce_fwd_static: the cross-entropy forward for callers that cannot
allocate device memory.

Some hosts of this library plan every device byte before training starts (a
runtime with a fixed memory pool, or a host whose buffers are owned by a
different allocator) and may not let a library call cudaMalloc in the middle
of a step, where it can fail under memory pressure and stalls the whole
device.  fcu_ce_fwd_static does the same work as fcu_ce_fwd with its per-row
scratch in a fixed array built into the library.  This test calls both entry
points straight through the C-ABI, twice in a row with different inputs, and
requires the same loss and gradient (relL2 <= 1e-5, the parity tolerance of
the other GPU tests).  The file name makes pytest collect it last.
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


@pytest.fixture(scope="module")
def cabi():
    from forgellm import _lib
    L = _lib.lib()
    torch.cuda.set_device(0)
    h = ctypes.c_void_p()
    assert L.fcu_ctx_create(0, ctypes.byref(h)) == 0, L.fcu_last_error()
    yield L, h
    torch.cuda.synchronize()
    L.fcu_ctx_destroy(h)


@pytest.mark.parametrize("T,V", [(37, 1003), (4096, 32000)])
def test_static_scratch_ce_matches_fcu_ce_fwd(cabi, T, V):
    L, h = cabi
    stream = torch.cuda.current_stream()
    assert L.fcu_ctx_set_stream(h, ctypes.c_void_p(stream.cuda_stream)) == 0
    gen = torch.Generator(device="cuda").manual_seed(T + V)
    for call in range(2):   # two calls in a row: the shared array keeps no state that matters
        logits = torch.randn(T * V, device="cuda", generator=gen) * (2.0 + call)
        targets = torch.randint(0, V, (T,), device="cuda", dtype=torch.int32, generator=gen)
        loss_a = torch.empty(1, device="cuda")
        loss_b = torch.empty(1, device="cuda")
        d_a = torch.empty(T * V, device="cuda")
        d_b = torch.empty(T * V, device="cuda")
        assert L.fcu_ce_fwd(h, logits.data_ptr(), targets.data_ptr(), T, V, loss_a.data_ptr(),
                            d_a.data_ptr()) == 0, L.fcu_last_error()
        assert L.fcu_ce_fwd_static(h, logits.data_ptr(), targets.data_ptr(), T, V,
                                   loss_b.data_ptr(), d_b.data_ptr()) == 0, L.fcu_last_error()
        torch.cuda.synchronize()
        la, lb = float(loss_a.item()), float(loss_b.item())
        assert abs(la - lb) <= TOL * abs(la), (call, la, lb)
        assert _rel(d_a.cpu().numpy(), d_b.cpu().numpy()) <= TOL, call


def test_static_scratch_ce_rejects_too_many_rows(cabi):
    L, h = cabi
    T, V = 65537, 4
    buf = torch.zeros(T * V, device="cuda")
    tg = torch.zeros(T, device="cuda", dtype=torch.int32)
    loss = torch.empty(1, device="cuda")
    rc = L.fcu_ce_fwd_static(h, buf.data_ptr(), tg.data_ptr(), T, V, loss.data_ptr(),
                             buf.data_ptr())
    assert rc != 0
    assert b"65536" in L.fcu_last_error()
