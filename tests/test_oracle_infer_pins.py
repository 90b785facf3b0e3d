"""The inference-side oracle (oracle/forge_oracle_infer.c) pinned to the
reference's own results (CPU only).

forge-llm ships no golden files for its quantizers or attention; its
invariant harness (src/L10/verify.js) draws every input from one RNG(12345)
and prints the results, recorded in docs/ALGORITHMS.md:447-465.  The L3 / L4 /
L5 blocks (verify.js:329-415) come after the training invariants, whose 702
normal() draws tests/test_oracle_pins.py replays value for value (I-70 and
I-71 use their own generators).  Replaying the same stream here reproduces:
  I-20  dequantize(quantizeRow(x)) RMSE  Q8_0 3.7e-3, Q4_K 5.2e-2, Q6_K 1.2e-2
  I-22  dotQ == dot(dequantize)          printed 0.00e+0 (or 1.78e-15)
  I-40  QuantLinear(Q8_0) vs f32 cosine  0.999985
  I-41  SwiGLU block == manual           0.00e+0
  I-50  flashAttention vs naive          8.94e-8
  I-54  KV-cache view vs full            8.94e-8
and the known answers of the reference's unit tests (test/l3-l5.test.js).

The printed table comes from a run whose L3 loop covered the three formats
its I-20 row names (Q8_0, Q4_K, Q6_K: one 1024-draw y vector each); today's
verify.js:335 also loops over Q5_K, which draws one more y vector and so
shifts every later input.  Replaying the three-format order reproduces I-40
and I-50 digit for digit (with Q5_K in the loop they come out 0.999988 and
1.34e-7), so the replay follows the printed run; Q5_K is checked on the same
x against verify.js's bound.
"""
import math

import numpy as np
import pytest

import oracle as O

# normal() draws of verify.js:36-283 (L0, L1, L2, L2b blocks), in order:
# L0 96+192+12, L1 7+8+16, I-33a 15+20+12, I-33b 12+12, I-33c 24+24,
# I-33d 64+32+32+64, I-34 15, I-35 10+10+10, I-36 15
DRAWS_BEFORE_L3 = 702


def _cos(a, b):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return O.dot(a.astype(np.float32), b.astype(np.float32)) / (math.hypot(*a) * math.hypot(*b))


@pytest.fixture(scope="module")
def verify_l3_l5():
    rng = O.RNG(12345)
    for _ in range(DRAWS_BEFORE_L3):
        rng.normal()
    out = {}
    # ---- L3 (verify.js:329-349)
    N = 1024
    x = np.array([rng.normal() * 0.7 for _ in range(N)], np.float32)
    for name, t in (("Q8_0", O.Q8_0), ("Q4_K", O.Q4_K), ("Q6_K", O.Q6_K)):
        q = O.quantize_row(t, x)
        dq = O.dequantize(t, q, N)
        out[f"I-20+{name}"] = math.sqrt(sum((float(b) - float(a)) ** 2 for a, b in zip(x, dq)) / N)
        y = rng.normals(N)
        out[f"I-22+{name}"] = abs(O.dotq(t, q, y, N) - O.dot(dq, y))
    q = O.quantize_row(O.Q5_K, x)          # Q5_K on the same x, no draw (see above)
    dq = O.dequantize(O.Q5_K, q, N)
    out["I-20+Q5_K"] = math.sqrt(sum((float(b) - float(a)) ** 2 for a, b in zip(x, dq)) / N)
    out["I-22+Q5_K"] = abs(O.dotq(O.Q5_K, q, y, N) - O.dot(dq, y))
    # ---- L4 (verify.js:352-374)
    Nn, K = 32, 64
    W = rng.normals(Nn * K)
    xv = rng.normals(K)
    o1 = O.quantlinear_fwd(O.F32, O.quantize_row(O.F32, W), xv, Nn, K)
    o2 = O.quantlinear_fwd(O.Q8_0, O.quantize_row(O.Q8_0, W), xv, Nn, K)
    out["I-40"] = _cos(o1, o2)
    dim, hidden = 16, 32
    gW, uW, dW = rng.normals(hidden * dim), rng.normals(hidden * dim), rng.normals(dim * hidden)
    x16 = xv[:dim]
    gv, uv = O.matvec(gW, x16, hidden, dim), O.matvec(uW, x16, hidden, dim)
    tmp = np.array([(float(g) / (1 + math.exp(-float(g)))) * float(u) for g, u in zip(gv, uv)], np.float32)
    ref = O.matvec(dW, tmp, dim, hidden)
    # SwiGLU.forward (nn.js:56-66) through QuantLinear type 0 is the same matvecs
    g2 = O.quantlinear_fwd(O.F32, gW, x16, hidden, dim)
    u2 = O.quantlinear_fwd(O.F32, uW, x16, hidden, dim)
    act = np.array([(float(g) / (1 + math.exp(-float(g)))) * float(u) for g, u in zip(g2, u2)], np.float32)
    out["I-41"] = float(np.max(np.abs(O.quantlinear_fwd(O.F32, dW, act, dim, hidden) - ref)))
    # ---- L5 (verify.js:377-415)
    n, d = 32, 8
    q = rng.normals(d)
    K_ = np.empty(n * d, np.float32)
    V_ = np.empty(n * d, np.float32)
    for i in range(n * d):
        K_[i] = rng.normal()
        V_[i] = rng.normal()
    sc = 1 / math.sqrt(d)
    o_flash = O.flash_attention(q, K_, V_, n, d, sc, True, n - 1, 0)
    o_naive = O.attention_naive(q, K_, V_, n, d, sc, True, n - 1, 0)
    out["I-50"] = float(np.max(np.abs(o_flash - o_naive)))
    q2 = rng.normals(d)
    o2 = O.flash_attention(q2, K_, V_, n, d, sc, True, 4, 0)
    out["I-52"] = float(np.max(np.abs(o2 - O.attention_naive(q2, K_, V_, 5, d, sc, True, 4, 0))))
    # I-54: the KVCache(1, n, d) view is the same contiguous rows
    out["I-54"] = float(np.max(np.abs(O.flash_attention(q, K_.copy(), V_.copy(), n, d, sc, True, n - 1, 0)
                                      - o_naive)))
    return out


def test_I20_rmse_values(verify_l3_l5):
    assert f"{verify_l3_l5['I-20+Q8_0']:.1e}" == "3.7e-03"
    assert f"{verify_l3_l5['I-20+Q4_K']:.1e}" == "5.2e-02"
    assert f"{verify_l3_l5['I-20+Q6_K']:.1e}" == "1.2e-02"
    assert verify_l3_l5["I-20+Q5_K"] < 0.04            # verify.js:336 bound for Q5_K


def test_I22_dotq_equals_dequantized_dot(verify_l3_l5):
    for name in ("Q8_0", "Q4_K", "Q5_K", "Q6_K"):
        assert verify_l3_l5[f"I-22+{name}"] <= 1.78e-15 * 4, name


def test_I40_quantlinear_q8_cosine(verify_l3_l5):
    assert f"{verify_l3_l5['I-40']:.6f}" == "0.999985"


def test_I41_swiglu_block(verify_l3_l5):
    assert verify_l3_l5["I-41"] == 0.0


def test_I50_I54_flash_vs_naive(verify_l3_l5):
    assert f"{verify_l3_l5['I-50']:.2e}" == "8.94e-08"
    assert f"{verify_l3_l5['I-54']:.2e}" == "8.94e-08"
    assert verify_l3_l5["I-52"] < 1e-5


# ------------------------------------------------------------ test/l3-l5.test.js known answers
def test_bpw_and_row_bytes():
    bpw = {t: O.block_bytes(t) * 8 / O.block_size(t) for t in (0, 1, 8, 12, 13, 14)}
    assert bpw == {0: 32, 1: 16, 8: 8.5, 12: 4.5, 13: 5.5, 14: 6.5625}
    assert O.row_bytes(O.Q4_K, 256) == 144 and O.row_bytes(O.Q4_K, 512) == 288
    assert O.row_bytes(O.Q6_K, 256) == 210 and O.row_bytes(O.Q8_0, 32) == 34
    assert O.row_bytes(O.Q8_0, 64) == 68 and O.row_bytes(O.F32, 100) == 400


def test_f16_round_trip():
    rng = O.RNG(1)
    x = rng.normals(64)
    dq = O.dequantize(O.F16, O.quantize_row(O.F16, x), 64)
    assert np.max(np.abs(dq - x) / (np.abs(x) + 1e-3)) < 1e-3


def test_fp16_conversion_edges():
    assert O.fp32_to_fp16(1.0) == 0x3C00 and O.fp32_to_fp16(-2.0) == 0xC000
    assert O.fp32_to_fp16(65520.0) == 0x7C00                 # rounds up into Inf
    assert O.fp32_to_fp16(float("inf")) == 0x7C00 and O.fp32_to_fp16(float("nan")) == 0x7E00
    assert O.fp32_to_fp16(2 ** -24) == 1                     # smallest subnormal
    assert O.fp16_to_fp32(0x3555) == np.float32(0.333251953125)
    assert O.fp16_to_fp32(0x0001) == np.float32(2 ** -24)


def test_q8_0_error_bound():
    rng = O.RNG(2)
    x = rng.normals(256)
    dq = O.dequantize(O.Q8_0, O.quantize_row(O.Q8_0, x), 256)
    assert np.max(np.abs(dq - x)) <= np.max(np.abs(x)) / 254 + 1e-6


def test_dotq_matches_dequantized_dot():
    n = 512
    rng = O.RNG(3)
    x = np.empty(n, np.float32)
    y = np.empty(n, np.float32)
    for i in range(n):
        x[i] = rng.normal() * 0.8
        y[i] = rng.normal()
    for t in (O.F16, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K):
        q = O.quantize_row(t, x)
        a = O.dot(O.dequantize(t, q, n), y)
        b = O.dotq(t, q, y, n)
        assert abs(a - b) <= 1e-3 * (abs(a) + 1), t


def test_q5_k_writer():
    rng = O.RNG(7)
    x = np.array([rng.normal() * 0.5 for _ in range(256)], np.float32)
    q = O.quantize_row(O.Q5_K, x)
    assert q.size == 176
    dq = O.dequantize(O.Q5_K, q, 256)
    assert math.sqrt(float(np.sum((dq.astype(np.float64) - x) ** 2) / np.sum(x.astype(np.float64) ** 2))) < 0.05
    assert np.count_nonzero(q[16:48]) > 0                     # the 5th bit is written


def test_q6_k_super_block_scale_at_the_end():
    rng = O.RNG(8)
    x = rng.normals(256)
    qx, qy = O.quantize_row(O.Q6_K, x), O.quantize_row(O.Q6_K, x * np.float32(4))
    assert qx.size == 210
    assert np.array_equal(qx[:208], qy[:208])
    assert not np.array_equal(qx[208:], qy[208:])
    dx = O.fp16_to_fp32(int(qx[208]) | int(qx[209]) << 8)
    dy = O.fp16_to_fp32(int(qy[208]) | int(qy[209]) << 8)
    assert abs(dy / dx - 4) < 0.02


def test_quality_report_ratio_and_cosine():
    rng = O.RNG(4)
    x = np.array([rng.normal() * 0.6 for _ in range(1024)], np.float32)
    for t, lo, hi, cmin in ((O.Q8_0, 3.5, 4.0, 0.999), (O.Q4_K, 6.5, 7.5, 0.995)):
        q = O.quantize_row(t, x)
        dq = O.dequantize(t, q, 1024)
        assert lo < 4096 / q.size < hi
        assert _cos(x, dq) > cmin


def test_quantlinear_q8_close_to_f32():
    rng = O.RNG(5)
    N, K = 64, 128
    W = rng.normals(N * K)
    x = rng.normals(K)
    o1 = O.quantlinear_fwd(O.F32, O.quantize_row(O.F32, W), x, N, K)
    o2 = O.quantlinear_fwd(O.Q8_0, O.quantize_row(O.Q8_0, W), x, N, K)
    assert _cos(o1, o2) > 0.999
    # QuantLinear.toF32 == dequantize (l3-l5.test.js:141-148)
    rng = O.RNG(6)
    W = rng.normals(32 * 64)
    q = O.quantize_row(O.Q8_0, W)
    assert np.array_equal(O.dequantize(O.Q8_0, q, 32 * 64),
                          np.concatenate([O.dequantize(O.Q8_0, q, 64, r * 68) for r in range(32)]))


def test_attention_known_answers():
    n, d = 64, 16
    rng = O.RNG(8)
    q = rng.normals(d)
    K = np.empty(n * d, np.float32)
    V = np.empty(n * d, np.float32)
    for i in range(n * d):
        K[i] = rng.normal()
        V[i] = rng.normal()
    sc = 1 / math.sqrt(d)
    f = O.flash_attention(q, K, V, n, d, sc, True, n - 1, 0)
    assert np.max(np.abs(f - O.attention_naive(q, K, V, n, d, sc, True, n - 1, 0))) < 1e-4
    assert np.max(np.abs(f - O.attention_decode(q, K, V, n, d, sc, True, n - 1, 0))) < 1e-5
    # causal mask: positions after pos do not take part (l3-l5.test.js:186-200)
    rng = O.RNG(9)
    n, d, pos = 16, 8, 5
    q = rng.normals(d)
    K = np.empty(n * d, np.float32)
    V = np.empty(n * d, np.float32)
    for i in range(n * d):
        K[i] = rng.normal()
        V[i] = rng.normal()
    sc = 1 / math.sqrt(d)
    o = O.flash_attention(q, K, V, n, d, sc, True, pos, 0)
    assert np.max(np.abs(o - O.attention_naive(q, K, V, pos + 1, d, sc, True, pos, 0))) < 1e-5
    assert np.max(np.abs(O.attention_decode(q, K, V, n, d, sc, True, pos, 0) - o)) < 1e-5


def test_inference_forward_matches_training_forward():
    """I-70 (verify.js:288-308): the oracle's inference forward, token by token
    through the KV cache, against its training forward (model_step logits),
    max |diff| < 2e-3; f32 weights."""
    cfg = O.Config(dim=32, hidden=64, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=40)
    P = O.init_weights(cfg, 4242)
    ids = np.array([1, 5, 9, 13, 2, 7], np.int32)
    G = np.zeros_like(P)
    _, logits = O.model_step(cfg, P, ids, np.zeros_like(ids), 1, len(ids), G, want_logits=True)
    m = O.InferModel(cfg, O.unflatten_weights(cfg, P), max_seq=16)
    worst = 0.0
    for t, tok in enumerate(ids):
        li = m.forward(int(tok), t)
        worst = max(worst, float(np.max(np.abs(li - logits[t * 40:(t + 1) * 40]))))
    assert worst < 2e-3, worst
