"""ctypes binding of the C ABI in include/wgd.h (libwgd.so, built in-tree).

There is no fallback: if the shared library is missing or a call fails, the
error is raised. The library is loaded once per process.
"""
from __future__ import annotations

import ctypes
import os
import threading

from ._build_paths import wgd_lib_path

c_int, c_int32, c_int64, c_uint32, c_uint64, c_float, c_void_p, c_char_p = (
    ctypes.c_int, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float, ctypes.c_void_p,
    ctypes.c_char_p)

WGD_OK, WGD_EINVAL, WGD_EBUDGET, WGD_ECUDA, WGD_ECANCELLED, WGD_ETIMEOUT, WGD_ESTATE, WGD_ENONFINITE, WGD_EIO = range(9)
STATUS_NAMES = {0: "OK", 1: "EINVAL", 2: "EBUDGET", 3: "ECUDA", 4: "ECANCELLED", 5: "ETIMEOUT", 6: "ESTATE",
                7: "ENONFINITE", 8: "EIO"}


class ModelConfigC(ctypes.Structure):
    """wgd_model_config (mirrors ModelConfig, gguf.ts:87-107 of the reference)."""
    _fields_ = [("family", c_int32), ("hidden", c_int32), ("intermediate", c_int32), ("layers", c_int32),
                ("heads", c_int32), ("kv_heads", c_int32), ("head_dim", c_int32), ("vocab", c_int32),
                ("epsilon", c_float), ("theta", c_float), ("local_theta", c_float), ("window", c_int32),
                ("period", c_int32), ("attention_scale", c_float), ("rope_scale", c_float), ("rotary_dim", c_int32),
                ("rope_mode", c_int32), ("sliding_window", c_int32), ("qk_norm", c_int32), ("ffn_gate", c_int32),
                ("activation", c_int32), ("bias_q", c_int32), ("bias_k", c_int32), ("bias_v", c_int32),
                ("bias_output", c_int32)]


class StatsC(ctypes.Structure):
    _fields_ = [("read_bytes", c_uint64), ("uploads", c_uint64), ("cache_hits", c_uint64), ("cache_bytes", c_uint64),
                ("gpu_bytes", c_uint64), ("peak_gpu_bytes", c_uint64), ("page_bytes", c_uint64), ("read_ms", ctypes.c_double),
                ("forwards", c_uint64), ("tokens", c_uint64), ("last_forward_ms", ctypes.c_double),
                ("streamed_bytes", c_uint64), ("kernel_launches", c_uint64)]


READ_FN = ctypes.CFUNCTYPE(c_int, c_void_p, c_uint64, c_uint64, c_void_p)

# name -> (restype, argtypes)
SIGNATURES = {
    "wgd_abi_version": (c_int, []),
    "wgd_last_error": (c_char_p, []),
    "wgd_device_count": (c_int, [ctypes.POINTER(c_int)]),
    "wgd_create": (c_void_p, [c_int, c_int, c_int, c_uint64, c_uint32, ctypes.POINTER(c_int)]),
    "wgd_destroy": (None, [c_void_p]),
    "wgd_tp_handle_size": (c_int, []),
    "wgd_tp_export": (c_int, [c_void_p, c_void_p]),
    "wgd_tp_open_peers": (c_int, [c_void_p, c_void_p]),
    "wgd_tp_set_timeout": (c_int, [c_void_p, c_uint64]),
    "wgd_model_begin": (c_int, [c_void_p, ctypes.POINTER(ModelConfigC), c_int, c_int]),
    "wgd_tensor_register": (c_int, [c_void_p, c_char_p, c_int, ctypes.POINTER(c_uint64), c_int, c_uint64, c_uint64, c_uint64]),
    "wgd_model_end": (c_int, [c_void_p]),
    "wgd_tensor_upload": (c_int, [c_void_p, c_char_p, c_uint64, c_void_p, c_uint64]),
    "wgd_tensor_host": (c_int, [c_void_p, c_char_p, c_void_p, c_int]),
    "wgd_set_page_reader": (c_int, [c_void_p, READ_FN, c_void_p]),
    "wgd_load_weights": (c_int, [c_void_p]),
    "wgd_model_ready": (c_int, [c_void_p, ctypes.POINTER(c_int)]),
    "wgd_model_placement": (c_int, [c_void_p, ctypes.POINTER(c_uint64), ctypes.POINTER(c_uint64)]),
    "wgd_plan_residency": (c_int, [ctypes.POINTER(c_uint64), c_int, c_uint64, c_uint64, c_uint64, c_uint64,
                                   ctypes.POINTER(c_int32), ctypes.POINTER(c_uint64)]),
    "wgd_forward": (c_int, [c_void_p, ctypes.POINTER(c_int32), c_int, c_int, c_int, ctypes.POINTER(c_int32), ctypes.POINTER(c_float)]),
    "wgd_decode": (c_int, [c_void_p, c_int32, c_int, c_int, ctypes.POINTER(c_int32)]),
    "wgd_forward_sample": (c_int, [c_void_p, ctypes.POINTER(c_int32), c_int, c_int, ctypes.c_double, c_int, ctypes.c_double,
                                   ctypes.c_double, ctypes.POINTER(c_int32)]),
    "wgd_decode_sample": (c_int, [c_void_p, c_int32, c_int, c_int, ctypes.c_double, c_int, ctypes.c_double,
                                  ctypes.POINTER(ctypes.c_double), ctypes.POINTER(c_int32)]),
    "wgd_op_sample": (c_int, [c_void_p, c_int, ctypes.c_double, c_int, ctypes.c_double, ctypes.c_double, ctypes.POINTER(c_int32),
                              c_void_p]),
    "wgd_kernels_per_token": (c_int, [c_void_p, ctypes.POINTER(c_int)]),
    "wgd_truncate_kv": (c_int, [c_void_p, c_int]),
    "wgd_cancel": (None, [c_void_p]),
    "wgd_stats_get": (c_int, [c_void_p, ctypes.POINTER(StatsC)]),
    "wgd_set_graphs": (c_int, [c_void_p, c_int]),
    "wgd_set_persistent": (c_int, [c_void_p, c_int]),
    "wgd_set_prefill_gemm": (c_int, [c_void_p, c_int]),
    "wgd_persistent_status": (c_int, [c_void_p, c_char_p, c_int]),
    "wgd_dev_row_bytes": (c_int64, [c_int, c_int64]),
    "wgd_op_repack": (c_int, [c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "wgd_op_dequant": (c_int, [c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "wgd_op_gemv": (c_int, [c_int, c_int64, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "wgd_tiled_bytes": (c_int64, [c_int, c_int64, c_int64]),
    "wgd_op_repack_tiled": (c_int, [c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "wgd_op_dequant_tiled": (c_int, [c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "wgd_op_gemv_tiled": (c_int, [c_int, c_int64, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "wgd_op_gemv_tiled_noalloc": (c_int, [c_int, c_int64, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "wgd_op_gemm_tiled": (c_int, [c_int, c_int64, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "wgd_op_gemm_tiled_status": (c_int, [ctypes.POINTER(c_int)]),
    "wgd_op_rmsnorm": (c_int, [c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_void_p]),
    "wgd_op_rope": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_float, c_float, c_int, c_int, c_void_p]),
    "wgd_op_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_int,
                                 c_int, c_void_p]),
    "wgd_op_argmax": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
}

_lib = None
_lock = threading.Lock()


class WgdError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status
        self.code = STATUS_NAMES.get(status, str(status))


def lib():
    """Loads libwgd.so (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            path = wgd_lib_path()
            if not os.path.exists(path):
                raise RuntimeError(f"wgd CUDA library missing: {path}. Build it with python -m webgpu_b200.build")
            L = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            if L.wgd_abi_version() != 1:
                raise RuntimeError("wgd ABI version mismatch")
            _lib = L
    return _lib


def last_error() -> str:
    msg = lib().wgd_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str = "") -> None:
    if status != WGD_OK:
        msg = last_error()
        raise WgdError(status, msg or f"{what} failed with {STATUS_NAMES.get(status, status)}")
