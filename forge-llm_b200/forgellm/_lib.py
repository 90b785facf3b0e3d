"""ctypes binding of libforgecu.so (the C-ABI declared in include/forgecu.h).

The library is the only compute path: there is no CPU fallback.  If the
shared object is missing or cannot be loaded, or no CUDA device is present,
every operator raises ``ForgeCUError``.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("FORGECU_LIB", os.path.join(_PKG_ROOT, "libforgecu.so"))

FCU_PREC_FP32, FCU_PREC_FP32_TC, FCU_PREC_BF16 = 0, 1, 2
FCU_ERR_ARG, FCU_ERR_CUDA, FCU_ERR_NCCL, FCU_ERR_TIMEOUT, FCU_ERR_UNSUPPORTED = -1, -2, -3, -4, -5
FCU_COMM_ID_BYTES = 128
PRECISIONS = {"fp32": FCU_PREC_FP32, "fp32tc": FCU_PREC_FP32_TC, "bf16": FCU_PREC_BF16}


class ForgeCUError(RuntimeError):
    """A libforgecu entry point returned a non-zero fcu_status (`.status`)."""

    def __init__(self, msg, status=None):
        super().__init__(msg)
        self.status = status


class RngState(C.Structure):
    _fields_ = [("s0", C.c_uint32), ("s1", C.c_uint32)]


class ModelCfg(C.Structure):
    _fields_ = [("vocab", C.c_int), ("dim", C.c_int), ("n_layers", C.c_int),
                ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("hidden", C.c_int),
                ("norm_eps", C.c_double), ("rope_theta", C.c_double)]


class GemmOut(C.Structure):
    """fcu_gemm_out."""
    _fields_ = [("mode", C.c_int), ("out", C.c_void_p), ("accumulate", C.c_int),
                ("residual", C.c_void_p), ("rope_T", C.c_int), ("rope_cols", C.c_int),
                ("head_dim", C.c_int), ("rope_theta", C.c_double), ("out2", C.c_void_p),
                ("aux", C.c_void_p)]


GEMM_FWD, GEMM_DX, GEMM_DW = 0, 1, 2
OUT_F32, OUT_F32_RESIDUAL, OUT_BF16, OUT_BF16_ROPE = 0, 1, 2, 3
OUT_BF16_SWIGLU, OUT_BF16_SWIGLU_BWD = 4, 5


class AdamHyper(C.Structure):
    _fields_ = [("lr", C.c_double), ("b1", C.c_double), ("b2", C.c_double),
                ("eps", C.c_double), ("wd", C.c_double), ("clip", C.c_double),
                ("bc1", C.c_double), ("bc2", C.c_double)]


class AdamSched(C.Structure):
    _fields_ = [("lr", C.c_double), ("b1", C.c_double), ("b2", C.c_double),
                ("eps", C.c_double), ("wd", C.c_double), ("clip", C.c_double),
                ("total_steps", C.c_double)]


_P = C.c_void_p
_I64 = C.c_int64
_INT = C.c_int
_D = C.c_double

# name -> (restype, argtypes); every compute entry returns int (fcu_status).
_SIGS = {
    "fcu_last_error": (C.c_char_p, []),
    "fcu_version": (C.c_char_p, []),
    "fcu_ctx_create": (_INT, [_INT, C.POINTER(_P)]),
    "fcu_ctx_destroy": (_INT, [_P]),
    "fcu_ctx_set_stream": (_INT, [_P, _P]),
    "fcu_ctx_set_precision": (_INT, [_P, _INT]),
    "fcu_ctx_get_precision": (_INT, [_P]),
    "fcu_sync": (_INT, [_P]),
    "fcu_launch_count": (C.c_ulonglong, []),
    "fcu_ctx_scratch_bytes": (_INT, [_P, C.POINTER(C.c_size_t)]),
    "fcu_check_device_error": (_INT, [_P]),
    "fcu_malloc": (_INT, [_P, C.c_size_t, C.POINTER(_P)]),
    "fcu_free": (_INT, [_P, _P]),
    "fcu_memcpy_h2d": (_INT, [_P, _P, _P, C.c_size_t]),
    "fcu_memcpy_d2h": (_INT, [_P, _P, _P, C.c_size_t]),
    "fcu_memset_zero": (_INT, [_P, _P, C.c_size_t]),
    "fcu_matmulT_fwd": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64]),
    "fcu_matmulT_bwd": (_INT, [_P, _P, _P, _P, _P, _INT, _P, _INT, _I64, _I64, _I64]),
    "fcu_embed_fwd": (_INT, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "fcu_embed_bwd": (_INT, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "fcu_rmsnorm_fwd": (_INT, [_P, _P, _P, _I64, _I64, _D, _P, _P]),
    "fcu_rmsnorm_bwd": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _P, _INT, _P, _INT]),
    "fcu_rope_fwd": (_INT, [_P, _P, _I64, _INT, _INT, _INT, _D, _INT, _P]),
    "fcu_rope_bwd": (_INT, [_P, _P, _I64, _INT, _INT, _INT, _D, _INT, _P, _INT]),
    "fcu_slicecols_fwd": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _P]),
    "fcu_slicecols_bwd": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _P, _INT]),
    "fcu_attn_fwd": (_INT, [_P, _P, _P, _P, _INT, _INT, _INT, _INT, _INT, _P, _P]),
    "fcu_attn_bwd": (_INT, [_P, _P, _P, _P, _P, _P, _P, _INT, _INT, _INT, _INT, _INT,
                            _P, _P, _P, _INT]),
    "fcu_swiglu_fwd": (_INT, [_P, _P, _P, _I64, _P]),
    "fcu_swiglu_bwd": (_INT, [_P, _P, _P, _P, _I64, _P, _P, _INT]),
    "fcu_add_fwd": (_INT, [_P, _P, _P, _I64, _P]),
    "fcu_add_bwd": (_INT, [_P, _P, _I64, _P, _INT, _P, _INT]),
    "fcu_ce_fwd": (_INT, [_P, _P, _P, _I64, _I64, _P, _P]),
    "fcu_ce_fwd_static": (_INT, [_P, _P, _P, _I64, _I64, _P, _P]),
    "fcu_axpy_dev": (_INT, [_P, _P, _P, _I64, _P, _INT]),
    "fcu_wsum_fwd": (_INT, [_P, _P, _P, _I64, _P]),
    "fcu_adam_step": (_INT, [_P, _P, _P, _P, _P, _I64, C.POINTER(AdamHyper), _P]),
    "fcu_adam_step_sumsq": (_INT, [_P, _P, _P, _P, _P, _I64, C.POINTER(AdamHyper), _P, _P]),
    "fcu_sumsq": (_INT, [_P, _P, _I64, _P, _INT]),
    "fcu_scale": (_INT, [_P, _P, _I64, C.c_float]),
    "fcu_gemm_bf16": (_INT, [_P, _INT, _P, _P, _I64, _I64, _I64, _P]),
    "fcu_gemm_plan": (_INT, [_I64, _I64, _I64, _INT, _INT, _INT, _INT, _P]),
    "fcu_rmsnorm_fwd_bf16": (_INT, [_P, _P, _P, _I64, _I64, _D, _P, _P]),
    "fcu_rmsnorm_fwd_bf16_add": (_INT, [_P, _P, _P, _P, _I64, _I64, _D, _P, _P, _P]),
    "fcu_rmsnorm_bwd_fused": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _P, _INT, _P, _P, _INT]),
    "fcu_swiglu_fwd_bf16": (_INT, [_P, _P, _I64, _I64, _P]),
    "fcu_swiglu_bwd_bf16": (_INT, [_P, _P, _P, _I64, _I64, _P]),
    "fcu_ce_fwd_bf16grad": (_INT, [_P, _P, _P, _I64, _I64, _P, _P]),
    "fcu_attn_fwd_bf16": (_INT, [_P, _P, _I64, _INT, _INT, _INT, _INT, _INT, _P, _P]),
    "fcu_attn_bwd_bf16": (_INT, [_P, _P, _P, _I64, _P, _P, _INT, _INT, _INT, _INT, _INT, _D, _P]),
    "fcu_adam_step_shadow": (_INT, [_P, _P, _P, _P, _P, _I64, C.POINTER(AdamHyper), _P, _P, _P]),
    "fcu_adam_step_sched": (_INT, [_P, _P, _P, _P, _P, _I64, C.POINTER(AdamSched), _P, _P, _P]),
    "fcu_selftest_bounded_wait": (_INT, [_P, _I64]),
    "fcu_gather_windows": (_INT, [_P, _P, _I64, _P, _INT, _INT, _P]),
    "fcu_adam_sched_advance": (_INT, [_P, C.POINTER(AdamSched), _P, _P]),
    "fcu_adam_update_dev": (_INT, [_P, _P, _P, _P, _P, _I64, _P, _P, _P, _P]),
    "fcu_to_bf16": (_INT, [_P, _P, _I64, _P]),
    "fcu_scale_bf16_dev": (_INT, [_P, _P, _I64, _P]),
    "fcu_ggml_row_bytes": (_I64, [_INT, _I64]),
    "fcu_quant_matvec": (_INT, [_P, _INT, _P, _I64, _I64, _P, _I64, _P]),
    "fcu_dequantize_rows": (_INT, [_P, _INT, _P, _I64, _I64, _P, _I64, _P]),
    "fcu_decode_rope_kv": (_INT, [_P, _P, _I64, _INT, _INT, _INT, _INT, _D, _P, _P, _P, _I64, _P, _INT, _INT]),
    "fcu_attn_decode": (_INT, [_P, _P, _I64, _P, _P, _I64, _P, _INT, _INT, _P, _INT, _INT, _INT, _INT, _D, _P]),
    "fcu_comm_unique_id": (_INT, [_P]),
    "fcu_comm_init": (_INT, [_INT, _P, _INT, _INT, _D, C.POINTER(_P)]),
    "fcu_comm_destroy": (_INT, [_P]),
    "fcu_comm_abort": (_INT, [_P]),
    "fcu_comm_info": (_INT, [_P, C.POINTER(_INT), C.POINTER(_INT), C.POINTER(_INT)]),
    "fcu_allreduce_grads": (_INT, [_P, _P, _P, _I64]),
    "fcu_reduce_scatter_grads": (_INT, [_P, _P, _P, _I64]),
    "fcu_allgather_params": (_INT, [_P, _P, _P, _I64, _INT]),
    "fcu_allreduce_sum_f64": (_INT, [_P, _P, _P, _I64]),
    "fcu_comm_join": (_INT, [_P, _P]),
    "fcu_comm_poll": (_INT, [_P, _D]),
    "fcu_comm_profile": (_INT, [_P, _INT]),
    "fcu_comm_profile_read": (_INT, [_P, _P, _INT, _P]),
    "fcu_rng_init": (None, [C.POINTER(RngState), C.c_uint32]),
    "fcu_rng_next": (_D, [C.POINTER(RngState)]),
    "fcu_rng_normal": (_D, [C.POINTER(RngState)]),
    "fcu_rng_int": (_INT, [C.POINTER(RngState), _INT]),
    "fcu_rng_fill_normal": (None, [C.POINTER(RngState), _P, _I64, _D]),
    "fcu_rng_fill_int": (None, [C.POINTER(RngState), _P, _I64, _INT]),
    "fcu_model_num_params": (_I64, [C.POINTER(ModelCfg)]),
    "fcu_init_weights": (_INT, [C.POINTER(ModelCfg), C.c_uint32, _P]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded libforgecu.so (raises ForgeCUError if it cannot load)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ForgeCUError(
                    f"libforgecu.so not found at {LIB_PATH}; build it with "
                    "`make -C forge-llm_b200` (or __graft_entry__.build())")
            try:
                L = C.CDLL(LIB_PATH)
            except OSError as e:  # pragma: no cover
                raise ForgeCUError(f"cannot load {LIB_PATH}: {e}") from e
            for name, (res, args) in _SIGS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def exported_symbols():
    return sorted(_SIGS)


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().fcu_last_error().decode(errors="replace")
        raise ForgeCUError(f"{what} failed (status {rc}): {msg}", rc)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


class Context:
    """One fcu_ctx per CUDA device (created lazily)."""

    _per_device: dict = {}

    def __init__(self, device: int):
        h = _P()
        check(lib().fcu_ctx_create(device, C.byref(h)), "fcu_ctx_create")
        self.handle = h
        self.device = device
        self._stream = None
        self._precision = FCU_PREC_FP32

    @classmethod
    def get(cls, device: int | None = None) -> "Context":
        import torch
        if not torch.cuda.is_available():
            raise ForgeCUError("forgecu needs a CUDA device; none is available")
        if device is None:
            device = torch.cuda.current_device()
        ctx = cls._per_device.get(device)
        if ctx is None:
            ctx = cls._per_device[device] = Context(device)
        return ctx

    def bind_stream(self, stream_handle: int) -> None:
        if stream_handle != self._stream:
            check(lib().fcu_ctx_set_stream(self.handle, _P(stream_handle)), "fcu_ctx_set_stream")
            self._stream = stream_handle

    def set_precision(self, mode: int) -> None:
        if mode != self._precision:
            check(lib().fcu_ctx_set_precision(self.handle, mode), "fcu_ctx_set_precision")
            self._precision = mode

    @property
    def precision(self) -> int:
        return self._precision
