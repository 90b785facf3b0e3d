"""The tcgen05 GEMM's launch plan (tile, split-K slices, raster) through
fcu_gemm_plan, the host-only function fcu_gemm_bf16 itself follows (CPU:
no device is touched).  The expected plans are the choices measured for the
config-5 step on a B200 (148 SMs, 74 concurrent CTA pairs); the split counts
are cross-checked against a Python restatement of the cost model."""
import ctypes
import math
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "forge-llm_b200", "libforgecu.so")

F32, F32_RES, BF16, BF16_ROPE, SWIGLU, SWIGLU_BWD = range(6)
SMS, PAIRS = 148, 74
D, H, V, QKV = 768, 2048, 32000, 1280


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is not built (run __graft_entry__.build())")
    lib = ctypes.CDLL(LIB)
    lib.fcu_gemm_plan.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    lib.fcu_gemm_plan.restype = ctypes.c_int
    return lib


def plan(lib, M, N, K, mode=F32, sms=SMS, pairs=PAIRS, setting=-1):
    out = (ctypes.c_int * 6)()
    assert lib.fcu_gemm_plan(M, N, K, mode, sms, pairs, setting, out) == 0
    return dict(zip(("pair", "bn", "splits", "row_major", "tiles_m", "tiles_n"), list(out)))


def model_splits(tiles, nk, slots, outputs):
    """The slice cost model: waves x (k-blocks per slice + 4) + slices x the
    partial tiles' traffic, in k-block times of 0.45 us."""
    hi = min(16, nk // 16)
    red = outputs * 8 / 6e12 / 0.45e-6
    best, best_t = 1, math.ceil(tiles / slots) * (nk + 4)
    for s in range(2, hi + 1):
        t = math.ceil(tiles * s / slots) * (math.ceil(nk / s) + 4) + s * red
        if t < best_t:
            best, best_t = s, t
    return best


@pytest.mark.parametrize("tokens", [65536, 8192])
def test_forward_products_take_the_pair_tile_when_they_fill_two_waves(lib, tokens):
    p = plan(lib, tokens, 4096, D, SWIGLU)                  # gate | up with the SwiGLU epilogue
    assert p["pair"] == 1 and p["splits"] == 1 and p["tiles_n"] == 4096 // 256
    p = plan(lib, tokens, QKV, D, BF16_ROPE)
    assert p["pair"] == 1 and p["splits"] == 1 and p["row_major"] == 1
    assert p["tiles_m"] == tokens // 256 and p["tiles_n"] == 5


def test_narrow_short_products_at_batch_8_keep_128_wide_single_tiles(lib):
    p = plan(lib, 8192, D, D)                               # wo projection: 96 pair tiles, 12 k-blocks
    assert p == dict(pair=0, bn=128, splits=1, row_major=1, tiles_m=64, tiles_n=6)


def test_logits_sweep_rows_in_groups(lib):
    p = plan(lib, 65536, V, D)                              # 125 column tiles: more than half a wave
    assert p["pair"] == 1 and p["row_major"] == 0 and p["splits"] == 1


@pytest.mark.parametrize("M,N,K,want", [(QKV, D, 65536, 9), (D, D, 65536, 8), (D, H, 65536, 3),
                                        (2 * H, D, 65536, 3), (2 * H, D, 8192, 3), (D, D, 8192, 8)])
def test_weight_gradients_split_as_measured(lib, M, N, K, want):
    p = plan(lib, M, N, K)
    assert p["pair"] == 1
    tiles = math.ceil(M / 256) * math.ceil(N / 256)
    assert p["splits"] == want == model_splits(tiles, math.ceil(K / 64), PAIRS, M * N)


def test_lm_head_input_gradient_at_batch_8_splits(lib):
    p = plan(lib, 8192, D, V)
    assert p["pair"] == 1 and p["splits"] == model_splits(32 * 3, 500, PAIRS, 8192 * D) == 3


def test_swiglu_epilogues_never_split(lib):
    assert plan(lib, 8192, H, 4096, SWIGLU_BWD)["splits"] == 1
    assert plan(lib, 2048, 4096, 8192, SWIGLU)["splits"] == 1


def test_pair_switch_and_devices_without_pairs(lib):
    assert plan(lib, 200, 256, 64)["pair"] == 0             # one 256-row tile: single CTA
    assert plan(lib, 200, 256, 64, setting=1)["pair"] == 1
    assert plan(lib, 65536, QKV, D, setting=0)["pair"] == 0
    assert plan(lib, 65536, QKV, D, pairs=0)["pair"] == 0   # no CTA pair fits
    assert plan(lib, 128, 4096, 768, setting=1)["pair"] == 0  # a single row tile never pairs


def test_bad_arguments_are_rejected(lib):
    out = (ctypes.c_int * 6)()
    assert lib.fcu_gemm_plan(0, 1, 1, F32, SMS, PAIRS, -1, out) != 0
    assert lib.fcu_gemm_plan(64, 64, 64, 9, SMS, PAIRS, -1, out) != 0
    assert lib.fcu_gemm_plan(64, 64, 64, F32, 0, PAIRS, -1, out) != 0
