"""The C-ABI library loads and exports every entry point include/forgecu.h
declares (CPU only: no compute calls)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "forgecu.h")
LIB = os.path.join(ROOT, "forge-llm_b200", "libforgecu.so")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"\b(fcu_[A-Za-z0-9_]+)\s*\(", src)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is not built (run __graft_entry__.build())")
    return ctypes.CDLL(LIB)


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("fcu_matmulT_fwd", "fcu_matmulT_bwd", "fcu_attn_fwd", "fcu_attn_bwd",
                 "fcu_ce_fwd", "fcu_rmsnorm_bwd", "fcu_embed_bwd", "fcu_adam_step"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_covers_header():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "forge-llm_b200"))
    from forgellm import _lib
    bound = set(_lib.exported_symbols())
    missing = [n for n in declared_functions() if n not in bound]
    assert not missing, f"header functions without a ctypes signature: {missing}"


def test_error_reporting_without_gpu(lib):
    lib.fcu_last_error.restype = ctypes.c_char_p
    lib.fcu_ctx_create.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
    h = ctypes.c_void_p()
    # device -1 is rejected before any CUDA call can matter
    rc = lib.fcu_ctx_create(-1, ctypes.byref(h))
    assert rc != 0
    assert lib.fcu_last_error()


def test_host_rng_matches_oracle():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "forge-llm_b200"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    from forgellm.train import RNG, Config, init_weights_flat
    a, b = RNG(12345), O.RNG(12345)
    assert [a.next() for _ in range(50)] == [b.next() for _ in range(50)]
    assert np.array_equal(a.normals(1000, 0.5), b.normals(1000, 0.5))
    assert np.array_equal(a.ints(1000, 32000), b.ints(1000, 32000))
    kw = dict(dim=64, hidden=176, nLayers=2, nHeads=4, nKvHeads=4, vocabSize=64)
    assert np.array_equal(init_weights_flat(Config(**kw), 1), O.init_weights(O.Config(**kw), 1))


def test_config_gqa_check():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "forge-llm_b200"))
    from forgellm.train import Config
    with pytest.raises(ValueError):
        Config(dim=64, nHeads=6, nKvHeads=4)
    c = Config(dim=768, nHeads=12, nKvHeads=4, hidden=2048, nLayers=12, vocabSize=32000)
    assert c.dHead == 64 and c.qkvOut == 1280 and c.groupSize == 3
