"""Failure detection without a GPU fault: a bounded wait that can never
complete runs out after ~1 ms, the device error word records it,
fcu_check_device_error reports FCU_ERR_TIMEOUT once, and the context keeps
working (a GEMM on the same stream afterwards is exact)."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives():
    import forgellm as F
    from forgellm import _lib
    from forgellm.autograd import ctx
    lib, h = _lib.lib(), ctx().handle
    assert lib.fcu_check_device_error(h) == 0
    assert lib.fcu_selftest_bounded_wait(h, 2_000_000) == 0      # ~1 ms of SM clocks
    rc = lib.fcu_check_device_error(h)
    assert rc == -4, lib.fcu_last_error()                          # FCU_ERR_TIMEOUT
    assert b"99" in lib.fcu_last_error()
    assert lib.fcu_check_device_error(h) == 0                      # reported once
    F.set_precision("bf16")
    try:
        M, N, K = 256, 256, 512
        g = torch.Generator(device="cuda").manual_seed(1)
        A = torch.randn(M * K, device="cuda", generator=g).to(torch.bfloat16)
        B = torch.randn(N * K, device="cuda", generator=g).to(torch.bfloat16)
        out = torch.empty(M * N, device="cuda")
        o = _lib.GemmOut(0, out.data_ptr(), 0, None, 0, 0, 0, 0.0)
        _lib.call("fcu_gemm_bf16", h, 0, A.data_ptr(), B.data_ptr(), M, N, K, ctypes.byref(o))
        torch.cuda.synchronize()
        assert lib.fcu_check_device_error(h) == 0
        ref = A.double().view(M, K) @ B.double().view(N, K).T
        err = float((out.double().view(M, N) - ref).norm() / ref.norm())
        assert err <= 1e-5
    finally:
        F.set_precision("fp32")
