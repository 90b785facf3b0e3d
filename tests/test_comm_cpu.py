"""The data-parallel communicator's failure handling (fcu_comm_* in
libforgecu), on CPU, against a stand-in NCCL (tests/fake_nccl/fake_nccl.c)
that can play a healthy communicator, a rank that never joins, an init that
fails, and a peer that fails after init.

Checked: the library asks NCCL for a non-blocking communicator and hands it
the id fcu_comm_unique_id produced; a rank that never joins ends the init
with FCU_ERR_TIMEOUT after the stated timeout, not later, and aborts the
communicator; an asynchronous peer error seen by fcu_comm_poll aborts it and
returns FCU_ERR_NCCL; an aborted communicator refuses every collective and is
freed by fcu_comm_destroy without a second finalize; bad arguments are
rejected before NCCL is called.  No GPU is touched: the stand-in needs none
and the failing calls return before any CUDA work.
"""
import os
import shutil
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "forge-llm_b200", "libforgecu.so")
FAKE_SRC = os.path.join(ROOT, "tests", "fake_nccl", "fake_nccl.c")

SCRIPT = textwrap.dedent(r"""
    import ctypes as C, os, sys, time
    L = C.CDLL(sys.argv[1])
    fake = C.CDLL(os.environ["FORGECU_NCCL_LIB"])
    L.fcu_last_error.restype = C.c_char_p
    P = C.c_void_p
    L.fcu_comm_init.argtypes = [C.c_int, P, C.c_int, C.c_int, C.c_double, C.POINTER(P)]
    L.fcu_comm_poll.argtypes = [P, C.c_double]
    L.fcu_comm_destroy.argtypes = [P]
    L.fcu_comm_abort.argtypes = [P]
    L.fcu_comm_info.argtypes = [P, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.fcu_allreduce_grads.argtypes = [P, P, P, C.c_int64]
    L.fcu_comm_unique_id.argtypes = [P]
    ARG, NCCL, TIMEOUT = -1, -3, -4

    uid = C.create_string_buffer(128)
    assert L.fcu_comm_unique_id(uid) == 0, L.fcu_last_error()
    assert uid.raw[:3] == bytes([1, 8, 15])
    assert L.fcu_comm_unique_id(None) == ARG

    # bad arguments never reach NCCL
    h = P()
    assert L.fcu_comm_init(-1, uid, 2, 2, 5.0, C.byref(h)) == ARG
    assert L.fcu_comm_init(-1, uid, 2, 0, 0.0, C.byref(h)) == ARG
    assert L.fcu_comm_init(-1, None, 2, 0, 5.0, C.byref(h)) == ARG
    assert fake.fake_nccl_inits() == 0

    # healthy: init, info, destroy (finalize polled, then destroy)
    fake.fake_nccl_set_mode(0)
    assert L.fcu_comm_init(-1, uid, 2, 1, 5.0, C.byref(h)) == 0, L.fcu_last_error()
    n, r, d = C.c_int(), C.c_int(), C.c_int()
    assert L.fcu_comm_info(h, C.byref(n), C.byref(r), C.byref(d)) == 0
    assert (n.value, r.value, d.value) == (2, 1, -1)
    assert L.fcu_comm_poll(h, 1.0) == 0           # nothing launched, no error
    assert L.fcu_allreduce_grads(None, h, None, 0) == ARG   # no context
    assert L.fcu_comm_destroy(h) == 0, L.fcu_last_error()
    assert (fake.fake_nccl_finalizes(), fake.fake_nccl_destroys(), fake.fake_nccl_aborts()) == (1, 1, 0)

    # a rank never joins: the init gives up after its timeout and aborts
    fake.fake_nccl_set_mode(1)
    t0 = time.monotonic()
    rc = L.fcu_comm_init(-1, uid, 2, 0, 0.3, C.byref(h))
    dt = time.monotonic() - t0
    assert rc == TIMEOUT, rc
    assert 0.3 <= dt < 5.0, dt
    assert b"not complete within" in L.fcu_last_error()
    assert fake.fake_nccl_aborts() == 1
    assert not h.value

    # init fails at once
    fake.fake_nccl_set_mode(2)
    assert L.fcu_comm_init(-1, uid, 2, 0, 5.0, C.byref(h)) == NCCL
    assert b"system error" in L.fcu_last_error()

    # a peer fails after init: the poll sees it, aborts, and the comm is dead
    fake.fake_nccl_set_mode(0)
    assert L.fcu_comm_init(-1, uid, 2, 0, 5.0, C.byref(h)) == 0, L.fcu_last_error()
    fake.fake_nccl_set_mode(3)
    assert L.fcu_comm_poll(h, 1.0) == NCCL
    assert b"remote error" in L.fcu_last_error()
    assert fake.fake_nccl_aborts() == 2
    assert L.fcu_allreduce_grads(None, h, None, 0) == NCCL     # refused: aborted
    assert b"aborted" in L.fcu_last_error()
    assert L.fcu_comm_poll(h, 1.0) == NCCL
    assert b"aborted" in L.fcu_last_error()
    assert L.fcu_comm_info(h, None, None, None) == NCCL
    assert L.fcu_comm_abort(h) == 0                            # idempotent
    assert fake.fake_nccl_aborts() == 2
    fin = fake.fake_nccl_finalizes()
    assert L.fcu_comm_destroy(h) == 0
    assert fake.fake_nccl_finalizes() == fin                   # no finalize after an abort
    print("COMM_CPU_OK")
""")


@pytest.fixture(scope="module")
def fake_nccl(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None or not os.path.exists("/usr/include/nccl.h"):
        pytest.skip("needs a C compiler and nccl.h to build the stand-in NCCL")
    out = str(tmp_path_factory.mktemp("fake_nccl") / "libfake_nccl.so")
    cuda_inc = "/usr/local/cuda/include"
    subprocess.run([cc, "-shared", "-fPIC", "-O1", "-I", cuda_inc, "-o", out, FAKE_SRC], check=True)
    return out


def test_comm_failure_paths_against_stand_in_nccl(fake_nccl, tmp_path):
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is not built (run __graft_entry__.build())")
    script = tmp_path / "drive_comm.py"
    script.write_text(SCRIPT)
    env = dict(os.environ, FORGECU_NCCL_LIB=fake_nccl, CUDA_VISIBLE_DEVICES="")
    p = subprocess.run([sys.executable, str(script), LIB], env=env, capture_output=True, text=True,
                       timeout=120)
    assert p.returncode == 0 and "COMM_CPU_OK" in p.stdout, p.stdout + p.stderr


def test_comm_reports_missing_nccl(tmp_path):
    script = tmp_path / "no_nccl.py"
    script.write_text(textwrap.dedent("""
        import ctypes as C, sys
        L = C.CDLL(sys.argv[1])
        L.fcu_last_error.restype = C.c_char_p
        uid = C.create_string_buffer(128)
        rc = L.fcu_comm_unique_id(uid)
        assert rc == -5, rc
        assert b"cannot load NCCL" in L.fcu_last_error()
        print("NO_NCCL_OK")
    """))
    env = dict(os.environ, FORGECU_NCCL_LIB=str(tmp_path / "does_not_exist.so"), CUDA_VISIBLE_DEVICES="")
    p = subprocess.run([sys.executable, str(script), LIB], env=env, capture_output=True, text=True,
                       timeout=120)
    assert p.returncode == 0 and "NO_NCCL_OK" in p.stdout, p.stdout + p.stderr
