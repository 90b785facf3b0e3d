"""ctypes/numpy view of the CPU oracle (``liboracle.so``) -- TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and the cpu_baseline / reference
legs of ``bench.py`` import this module, and only as the checker or as the
timed CPU baseline.  The product (``forge-llm_b200``) never imports it.

Every function mirrors one JS function of forge-llm (cited in
``forge_oracle.c``); arrays are float32 / int32 numpy arrays.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")


def build() -> str:
    """Compile liboracle.so from forge_oracle.c and forge_oracle_infer.c (make,
    in this directory)."""
    srcs = [os.path.join(_HERE, f) for f in ("forge_oracle.c", "forge_oracle_infer.c")]
    if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < max(map(os.path.getmtime, srcs)):
        subprocess.run(["make", "-s", "-C", _HERE, "CC=gcc"], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_f = C.POINTER(C.c_float)
_i = C.POINTER(C.c_int32)
_d = C.POINTER(C.c_double)
_i64 = C.c_int64


class _Rng(C.Structure):
    _fields_ = [("s0", C.c_uint32), ("s1", C.c_uint32)]


class OrCfg(C.Structure):
    _fields_ = [("vocab", C.c_int), ("dim", C.c_int), ("n_layers", C.c_int),
                ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("hidden", C.c_int),
                ("norm_eps", C.c_double), ("rope_theta", C.c_double)]


def _declare(L):
    sig = {
        "or_set_threads": (None, [C.c_int]),
        "or_get_threads": (C.c_int, []),
        "or_rng_init": (None, [C.POINTER(_Rng), C.c_uint32]),
        "or_rng_next": (C.c_double, [C.POINTER(_Rng)]),
        "or_rng_normal": (C.c_double, [C.POINTER(_Rng)]),
        "or_rng_int": (C.c_int, [C.POINTER(_Rng), C.c_int]),
        "or_rng_fill_normal": (None, [C.POINTER(_Rng), _f, _i64, C.c_double]),
        "or_rng_fill_int": (None, [C.POINTER(_Rng), _i, _i64, C.c_int]),
        "or_rel_l2": (C.c_double, [_f, _f, _i64]),
        "or_gemm": (None, [_f, _f, _f, _i64, _i64, _i64]),
        "or_matmulT_bwd_dx": (None, [_f, _f, _f, _i64, _i64, _i64]),
        "or_matmulT_bwd_dw": (None, [_f, _f, _f, _i64, _i64, _i64, _i64, _i64]),
        "or_matmulT_bwd": (None, [_f, _f, _f, _f, _f, _i64, _i64, _i64]),
        "or_embed_fwd": (None, [_f, _i, _i64, _i64, _f]),
        "or_embed_bwd": (None, [_f, _i, _i64, _i64, _i64, _f]),
        "or_rmsnorm_fwd": (None, [_f, _f, _i64, _i64, C.c_double, _f, _f]),
        "or_rmsnorm_bwd": (None, [_f, _f, _f, _f, _i64, _i64, _f, _f]),
        "or_rope_fwd": (None, [_f, _i64, C.c_int, C.c_int, C.c_int, C.c_double, C.c_int, _f]),
        "or_rope_bwd": (None, [_f, _i64, C.c_int, C.c_int, C.c_int, C.c_double, C.c_int, _f]),
        "or_slicecols_fwd": (None, [_f, _i64, _i64, _i64, _i64, _f]),
        "or_slicecols_bwd": (None, [_f, _i64, _i64, _i64, _i64, _f]),
        "or_attn_fwd": (None, [_f, _f, _f, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _f, _f]),
        "or_attn_bwd": (None, [_f, _f, _f, _f, _f, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                               _f, _f, _f]),
        "or_swiglu_fwd": (None, [_f, _f, _i64, _f, _f]),
        "or_swiglu_bwd": (None, [_f, _f, _f, _f, _i64, _f, _f]),
        "or_ce_fwd": (C.c_float, [_f, _i, _i64, _i64, _f]),
        "or_ce_bwd": (None, [C.c_float, _f, _i, _i64, _i64, _f]),
        "or_wsum_fwd": (C.c_float, [_f, _f, _i64]),
        "or_wsum_bwd": (None, [C.c_float, _f, _i64, _f]),
        "or_linear_fwd": (None, [_f, _f, _i64, _i64, _f]),
        "or_linear_bwd": (None, [_f, _f, _f, _i64, _i64, _f, _f]),
        "or_softmaxce_fwd": (C.c_float, [_f, _i64, C.c_int, _f]),
        "or_softmaxce_bwd": (None, [C.c_float, _f, _i64, C.c_int, _f]),
        "or_adam_step": (None, [_f, _f, _f, _f, _i64, C.c_int, C.c_double, C.c_double,
                                C.c_double, C.c_double, C.c_double, C.c_double, C.c_double, _d]),
        "or_model_num_params": (C.c_int64, [C.POINTER(OrCfg)]),
        "or_init_weights": (None, [C.POINTER(OrCfg), C.c_uint32, _f]),
        "or_model_step": (C.c_float, [C.POINTER(OrCfg), _f, _f, _i, _i, C.c_int, C.c_int, _f]),
    }
    _u8 = C.POINTER(C.c_uint8)
    sig.update({
        "or_fp16_to_fp32": (C.c_float, [C.c_int]),
        "or_fp32_to_fp16": (C.c_int, [C.c_double]),
        "or_block_size": (C.c_int, [C.c_int]),
        "or_block_bytes": (C.c_int, [C.c_int]),
        "or_row_bytes": (C.c_int64, [C.c_int, _i64]),
        "or_dot": (C.c_double, [_f, _f, _i64]),
        "or_matvec": (None, [_f, _f, _f, _i64, _i64]),
        "or_dequantize": (C.c_int, [C.c_int, _u8, _i64, _f, _i64]),
        "or_dotq": (C.c_double, [C.c_int, _u8, _f, _i64, _i64, _i64]),
        "or_quantlinear_fwd": (None, [C.c_int, _u8, _f, _i64, _i64, _f, _i64]),
        "or_quantize_row": (C.c_int64, [C.c_int, _f, _i64, _u8]),
        "or_attention_decode": (None, [_f, _f, _f, _f, _i64, _i64, C.c_double, C.c_int, _i64, _i64]),
        "or_attention_naive": (None, [_f, _f, _f, _f, _i64, _i64, C.c_double, C.c_int, _i64, _i64]),
        "or_flash_attention": (None, [_f, _f, _f, _f, _i64, _i64, C.c_double, C.c_int, _i64, _i64,
                                      C.c_int]),
        "or_rmsnorm_vec": (None, [_f, _f, _f, _i64, C.c_double]),
        "or_rope_table": (None, [_i64, C.c_int, C.c_double, _f, _f]),
        "or_transformer_forward": (None, [C.c_void_p, C.c_int, _i64, _f, _f, _f]),
    })
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _fp(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(_f)


def _ip(a):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_i)


def f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


# ---------------------------------------------------------------- RNG
class RNG:
    """xorshift128+ of src/L0/numeric.js:27-49."""

    def __init__(self, seed: int = 0x9E3779B9):
        self._s = _Rng()
        lib().or_rng_init(C.byref(self._s), C.c_uint32(seed & 0xFFFFFFFF))

    def next(self) -> float:
        return lib().or_rng_next(C.byref(self._s))

    def normal(self) -> float:
        return lib().or_rng_normal(C.byref(self._s))

    def int(self, n: int) -> int:
        return lib().or_rng_int(C.byref(self._s), n)

    def normals(self, n: int, scale: float = 1.0) -> np.ndarray:
        """Float32Array of n draws of normal()*scale (verify.js randArr)."""
        out = np.empty(int(n), np.float32)
        lib().or_rng_fill_normal(C.byref(self._s), _fp(out), int(n), float(scale))
        return out

    def ints(self, n: int, rng_max: int) -> np.ndarray:
        out = np.empty(int(n), np.int32)
        lib().or_rng_fill_int(C.byref(self._s), _ip(out), int(n), int(rng_max))
        return out


def rel_l2(a, b) -> float:
    a, b = f32(a).ravel(), f32(b).ravel()
    return lib().or_rel_l2(_fp(a), _fp(b), a.size)


# ---------------------------------------------------------------- ops
def matmulT_fwd(X, W, M, K, N):
    Y = np.empty(M * N, np.float32)
    lib().or_gemm(_fp(Y), _fp(f32(X)), _fp(f32(W)), M, N, K)
    return Y


def matmulT_bwd(g, X, W, M, K, N, gX=None, gW=None):
    gX = np.zeros(M * K, np.float32) if gX is None else gX
    gW = np.zeros(N * K, np.float32) if gW is None else gW
    lib().or_matmulT_bwd(_fp(f32(g)), _fp(f32(X)), _fp(f32(W)), _fp(gX), _fp(gW), M, K, N)
    return gX, gW


def matmulT_bwd_dx(g, W, M, K, N, gX=None):
    gX = np.zeros(M * K, np.float32) if gX is None else gX
    lib().or_matmulT_bwd_dx(_fp(f32(g)), _fp(f32(W)), _fp(gX), M, K, N)
    return gX


def matmulT_bwd_dw_rows(g, X, M, K, N, n0, n1, gW_rows=None):
    """Rows [n0, n1) of dW, returned as a [(n1-n0)*K] array."""
    full = np.zeros(N * K, np.float32)
    if gW_rows is not None:
        full[n0 * K:n1 * K] = gW_rows
    lib().or_matmulT_bwd_dw(_fp(f32(g)), _fp(f32(X)), _fp(full), M, K, N, n0, n1)
    return full[n0 * K:n1 * K].copy()


def embed_fwd(W, ids, V, D):
    ids = np.ascontiguousarray(ids, np.int32)
    out = np.empty(ids.size * D, np.float32)
    lib().or_embed_fwd(_fp(f32(W)), _ip(ids), ids.size, D, _fp(out))
    return out


def embed_bwd(g, ids, V, D, gW=None):
    ids = np.ascontiguousarray(ids, np.int32)
    gW = np.zeros(V * D, np.float32) if gW is None else gW
    lib().or_embed_bwd(_fp(f32(g)), _ip(ids), ids.size, V, D, _fp(gW))
    return gW


def rmsnorm_fwd(X, w, T, D, eps):
    out = np.empty(T * D, np.float32)
    inv = np.empty(T, np.float32)
    lib().or_rmsnorm_fwd(_fp(f32(X)), _fp(f32(w)), T, D, eps, _fp(out), _fp(inv))
    return out, inv


def rmsnorm_bwd(g, X, w, inv, T, D, gX=None, gw=None):
    gX = np.zeros(T * D, np.float32) if gX is None else gX
    gw = np.zeros(D, np.float32) if gw is None else gw
    lib().or_rmsnorm_bwd(_fp(f32(g)), _fp(f32(X)), _fp(f32(w)), _fp(f32(inv)), T, D, _fp(gX),
                         _fp(gw))
    return gX, gw


def rope_fwd(X, T, nHead, dHead, pos0=0, theta=10000.0, posStride=0):
    out = np.empty(T * nHead * dHead, np.float32)
    lib().or_rope_fwd(_fp(f32(X)), T, nHead, dHead, pos0, theta, posStride, _fp(out))
    return out


def rope_bwd(g, T, nHead, dHead, pos0=0, theta=10000.0, posStride=0, gX=None):
    gX = np.zeros(T * nHead * dHead, np.float32) if gX is None else gX
    lib().or_rope_bwd(_fp(f32(g)), T, nHead, dHead, pos0, theta, posStride, _fp(gX))
    return gX


def slicecols_fwd(X, M, K, off, ln):
    out = np.empty(M * ln, np.float32)
    lib().or_slicecols_fwd(_fp(f32(X)), M, K, off, ln, _fp(out))
    return out


def slicecols_bwd(g, M, K, off, ln, gX=None):
    gX = np.zeros(M * K, np.float32) if gX is None else gX
    lib().or_slicecols_bwd(_fp(f32(g)), M, K, off, ln, _fp(gX))
    return gX


def attn_fwd(Q, K, V, B, T, nH, nKV, dH):
    out = np.empty(B * T * nH * dH, np.float32)
    P = np.zeros(B * nH * T * T, np.float32)
    lib().or_attn_fwd(_fp(f32(Q)), _fp(f32(K)), _fp(f32(V)), B, T, nH, nKV, dH, _fp(out), _fp(P))
    return out, P


def attn_bwd(g, Q, K, V, P, B, T, nH, nKV, dH, gQ=None, gK=None, gV=None):
    gQ = np.zeros(B * T * nH * dH, np.float32) if gQ is None else gQ
    gK = np.zeros(B * T * nKV * dH, np.float32) if gK is None else gK
    gV = np.zeros(B * T * nKV * dH, np.float32) if gV is None else gV
    lib().or_attn_bwd(_fp(f32(g)), _fp(f32(Q)), _fp(f32(K)), _fp(f32(V)), _fp(f32(P)), B, T, nH,
                      nKV, dH, _fp(gQ), _fp(gK), _fp(gV))
    return gQ, gK, gV


def swiglu_fwd(G, U):
    G, U = f32(G).ravel(), f32(U).ravel()
    out = np.empty(G.size, np.float32)
    sig = np.empty(G.size, np.float32)
    lib().or_swiglu_fwd(_fp(G), _fp(U), G.size, _fp(out), _fp(sig))
    return out, sig


def swiglu_bwd(g, G, U, sig, gG=None, gU=None):
    G = f32(G).ravel()
    gG = np.zeros(G.size, np.float32) if gG is None else gG
    gU = np.zeros(G.size, np.float32) if gU is None else gU
    lib().or_swiglu_bwd(_fp(f32(g)), _fp(G), _fp(f32(U)), _fp(f32(sig)), G.size, _fp(gG), _fp(gU))
    return gG, gU


def ce_fwd(logits, targets, T, V):
    probs = np.empty(T * V, np.float32)
    t = np.ascontiguousarray(targets, np.int32)
    loss = lib().or_ce_fwd(_fp(f32(logits)), _ip(t), T, V, _fp(probs))
    return np.float32(loss), probs


def ce_bwd(gout, probs, targets, T, V, gL=None):
    gL = np.zeros(T * V, np.float32) if gL is None else gL
    t = np.ascontiguousarray(targets, np.int32)
    lib().or_ce_bwd(float(gout), _fp(f32(probs)), _ip(t), T, V, _fp(gL))
    return gL


def wsum_fwd(Y, t):
    Y, t = f32(Y).ravel(), f32(t).ravel()
    return np.float32(lib().or_wsum_fwd(_fp(Y), _fp(t), Y.size))


def wsum_bwd(gout, t, gY=None):
    t = f32(t).ravel()
    gY = np.zeros(t.size, np.float32) if gY is None else gY
    lib().or_wsum_bwd(float(gout), _fp(t), t.size, _fp(gY))
    return gY


def linear_fwd(W, x, N, K):
    out = np.empty(N, np.float32)
    lib().or_linear_fwd(_fp(f32(W)), _fp(f32(x)), N, K, _fp(out))
    return out


def linear_bwd(g, W, x, N, K, gW=None, gx=None):
    gW = np.zeros(N * K, np.float32) if gW is None else gW
    gx = np.zeros(K, np.float32) if gx is None else gx
    lib().or_linear_bwd(_fp(f32(g)), _fp(f32(W)), _fp(f32(x)), N, K, _fp(gW), _fp(gx))
    return gW, gx


def softmaxce_fwd(logits, target):
    logits = f32(logits)
    p = np.empty(logits.size, np.float32)
    loss = lib().or_softmaxce_fwd(_fp(logits), logits.size, int(target), _fp(p))
    return np.float32(loss), p


def softmaxce_bwd(gout, p, target, gl=None):
    p = f32(p)
    gl = np.zeros(p.size, np.float32) if gl is None else gl
    lib().or_softmaxce_bwd(float(gout), _fp(p), p.size, int(target), _fp(gl))
    return gl


def adam_step(p, grad, m, v, t, lr=3e-4, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, clip=1.0,
              total=1000):
    """In place on p, m, v (flat float32).  Returns {lr, gnorm, scale}."""
    info = (C.c_double * 3)()
    lib().or_adam_step(_fp(p), _fp(f32(grad)), _fp(m), _fp(v), p.size, int(t), lr, b1, b2, eps,
                       wd, clip, float(total), info)
    return {"lr": info[0], "gnorm": info[1], "scale": info[2]}


# ---------------------------------------------------------------- model
@dataclass
class Config:
    """src/L6/transformer.js:29-53 (the fields training uses)."""
    dim: int = 288
    hidden: int = 768
    nLayers: int = 6
    nHeads: int = 6
    nKvHeads: int = 6
    vocabSize: int = 32000
    normEps: float = 1e-5
    ropeTheta: float = 10000.0

    def c(self) -> OrCfg:
        return OrCfg(self.vocabSize, self.dim, self.nLayers, self.nHeads, self.nKvHeads,
                     self.hidden, self.normEps, self.ropeTheta)


def num_params(cfg: Config) -> int:
    c = cfg.c()
    return int(lib().or_model_num_params(C.byref(c)))


def init_weights(cfg: Config, seed: int) -> np.ndarray:
    c = cfg.c()
    P = np.empty(num_params(cfg), np.float32)
    lib().or_init_weights(C.byref(c), C.c_uint32(seed & 0xFFFFFFFF), _fp(P))
    return P


def model_step(cfg: Config, P, ids, targets, B, T, G=None, want_logits=False):
    """Forward + CE loss (+ backward accumulating into G when given).
    ids/targets are flat [B*T].  Returns loss (and logits if asked)."""
    c = cfg.c()
    ids = np.ascontiguousarray(ids, np.int32)
    tg = np.ascontiguousarray(targets, np.int32)
    logits = np.empty(B * T * cfg.vocabSize, np.float32) if want_logits else None
    loss = lib().or_model_step(C.byref(c), _fp(P), _fp(G), _ip(ids), _ip(tg), B, T, _fp(logits))
    return (np.float32(loss), logits) if want_logits else np.float32(loss)


# ---------------------------------------------------------------- inference side
# GGML type numbers (quant.js:34-38) of the formats the decode kernels read.
F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 6, 8, 12, 13, 14


def _u8p(a):
    assert a.dtype == np.uint8 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_uint8))


def _bytes(data) -> np.ndarray:
    """A weight byte stream: uint8 as is, float32 / float16 arrays by their bytes."""
    a = np.ascontiguousarray(data)
    return a if a.dtype == np.uint8 else a.view(np.uint8)


def fp32_to_fp16(x: float) -> int:
    return int(lib().or_fp32_to_fp16(float(x)))


def fp16_to_fp32(h: int) -> float:
    return float(lib().or_fp16_to_fp32(int(h)))


def block_size(t: int) -> int:
    return int(lib().or_block_size(t))


def block_bytes(t: int) -> int:
    return int(lib().or_block_bytes(t))


def row_bytes(t: int, n: int) -> int:
    return int(lib().or_row_bytes(t, n))


def dot(a, b) -> float:
    a, b = f32(a).ravel(), f32(b).ravel()
    return float(lib().or_dot(_fp(a), _fp(b), a.size))


def matvec(W, x, N, K):
    out = np.empty(N, np.float32)
    lib().or_matvec(_fp(out), _fp(f32(W)), _fp(f32(x)), N, K)
    return out


def quantize_row(t: int, x) -> np.ndarray:
    """quantizeRow (quant.js:594-604) of a flat float32 array (types 0, 1, 8,
    12, 13, 14)."""
    x = f32(x).ravel()
    out = np.zeros(max(1, row_bytes(t, x.size)), np.uint8)
    n = lib().or_quantize_row(t, _fp(x), x.size, _u8p(out))
    if n < 0:
        raise ValueError(f"quantizeRow: type {t} not supported")
    return out[:n]


def dequantize(t: int, data, n: int, byte_off: int = 0) -> np.ndarray:
    data = _bytes(data)
    out = np.zeros(n, np.float32)
    if lib().or_dequantize(t, _u8p(data), n, _fp(out), byte_off):
        raise ValueError(f"dequantize: type {t} not supported")
    return out


def dotq(t: int, data, x, n: int, x_off: int = 0, byte_off: int = 0) -> float:
    data = _bytes(data)
    return float(lib().or_dotq(t, _u8p(data), _fp(f32(x)), n, x_off, byte_off))


def quantlinear_fwd(t: int, data, x, N: int, K: int) -> np.ndarray:
    """QuantLinear.forward (nn.js:27-32): out[N] = W . x."""
    data = _bytes(data)
    out = np.empty(N, np.float32)
    lib().or_quantlinear_fwd(t, _u8p(data), _fp(f32(x)), N, K, _fp(out), 0)
    return out


def _attn(fn, q, K, V, n, d, scale, causal, q_off, k_off, *extra):
    out = np.empty(d, np.float32)
    getattr(lib(), fn)(_fp(out), _fp(f32(q)), _fp(f32(K)), _fp(f32(V)), n, d, float(scale),
                       1 if causal else 0, q_off, k_off, *extra)
    return out


def attention_decode(q, K, V, n, d, scale, causal=True, q_off=0, k_off=0):
    return _attn("or_attention_decode", q, K, V, n, d, scale, causal, q_off, k_off)


def attention_naive(q, K, V, n, d, scale, causal=True, q_off=0, k_off=0):
    return _attn("or_attention_naive", q, K, V, n, d, scale, causal, q_off, k_off)


def flash_attention(q, K, V, n, d, scale, causal=True, q_off=0, k_off=0, block=64):
    return _attn("or_flash_attention", q, K, V, n, d, scale, causal, q_off, k_off, block)


def rmsnorm_vec(x, w, eps):
    x = f32(x).ravel()
    out = np.empty_like(x)
    lib().or_rmsnorm_vec(_fp(out), _fp(x), _fp(f32(w)), x.size, float(eps))
    return out


def rope_table(max_pos, dim, theta=10000.0):
    cos = np.empty(max_pos * dim // 2, np.float32)
    sin = np.empty_like(cos)
    lib().or_rope_table(max_pos, dim, float(theta), _fp(cos), _fp(sin))
    return cos, sin


class _InferModel(C.Structure):
    _fields_ = [("vocab", C.c_int), ("dim", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("hidden", C.c_int), ("max_seq", C.c_int),
                ("norm_eps", C.c_double), ("rope_theta", C.c_double), ("tok_type", C.c_int),
                ("w_type", C.c_int), ("tok_emb", C.c_void_p), ("ln_f", C.c_void_p),
                ("ln1", C.c_void_p), ("ln2", C.c_void_p), ("wqkv", C.c_void_p), ("wo", C.c_void_p),
                ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p)]


class InferModel:
    """Transformer (transformer.js:67-185) for the oracle's inference forward:
    weights as QuantLinear byte streams.  `w` maps the export names
    (tok_emb, ln_f, layer.{l}.{ln1, ln2, wqkv, wo, ffn_gate, ffn_up,
    ffn_down}) to float32 arrays; matrices are quantized to `w_type`, the
    embedding / LM head to `tok_type`."""

    def __init__(self, cfg: "Config", w: dict, max_seq: int, w_type: int = 0, tok_type: int = 0):
        self.cfg, self.max_seq = cfg, max_seq
        D, H = cfg.dim, cfg.hidden
        dH = D // cfg.nHeads
        qkv = (cfg.nHeads + 2 * cfg.nKvHeads) * dH
        self._keep = []

        def q(arr, t):
            b = quantize_row(t, arr)
            self._keep.append(b)
            return b

        self.tok = q(w["tok_emb"], tok_type)
        self.ln_f = f32(w["ln_f"])
        L = cfg.nLayers
        names = ("wqkv", "wo", "ffn_gate", "ffn_up", "ffn_down")
        self.mats = {k: [q(w[f"layer.{l}"][k], w_type) for l in range(L)] for k in names}
        self.norms = {k: [f32(w[f"layer.{l}"][k]) for l in range(L)] for k in ("ln1", "ln2")}
        self._keep += [self.ln_f] + self.norms["ln1"] + self.norms["ln2"]

        def ptrs(arrs):
            a = (C.c_void_p * len(arrs))(*[x.ctypes.data for x in arrs])
            self._keep.append(a)
            return C.cast(a, C.c_void_p)

        self.s = _InferModel(cfg.vocabSize, D, L, cfg.nHeads, cfg.nKvHeads, H, max_seq,
                             float(cfg.normEps), float(cfg.ropeTheta), tok_type, w_type,
                             self.tok.ctypes.data, self.ln_f.ctypes.data,
                             ptrs(self.norms["ln1"]), ptrs(self.norms["ln2"]),
                             ptrs(self.mats["wqkv"]), ptrs(self.mats["wo"]), ptrs(self.mats["ffn_gate"]),
                             ptrs(self.mats["ffn_up"]), ptrs(self.mats["ffn_down"]))
        kv = cfg.nKvHeads * dH
        self.cache_k = np.zeros(L * max_seq * kv, np.float32)
        self.cache_v = np.zeros_like(self.cache_k)
        del qkv

    def forward(self, token: int, pos: int) -> np.ndarray:
        logits = np.empty(self.cfg.vocabSize, np.float32)
        lib().or_transformer_forward(C.byref(self.s), int(token), int(pos), _fp(self.cache_k),
                                     _fp(self.cache_v), _fp(logits))
        return logits


def unflatten_weights(cfg: "Config", P) -> dict:
    """The flat paramList-order buffer of init_weights as the export dict
    (toParams / exportWeights order, train.js:60-78)."""
    P = f32(P).ravel()
    V, D, H, L = cfg.vocabSize, cfg.dim, cfg.hidden, cfg.nLayers
    dH = D // cfg.nHeads
    qkv = (cfg.nHeads + 2 * cfg.nKvHeads) * dH
    w, off = {}, 0

    def take(n):
        nonlocal off
        a = P[off:off + n]
        off += n
        return a

    w["tok_emb"] = take(V * D)
    w["ln_f"] = take(D)
    for l in range(L):
        w[f"layer.{l}"] = {"ln1": take(D), "ln2": take(D), "wqkv": take(qkv * D), "wo": take(D * D),
                           "ffn_gate": take(H * D), "ffn_up": take(H * D), "ffn_down": take(D * H)}
    assert off == P.size
    return w
