"""ctypes binding of librie_cuda.so (the C ABI declared in include/rie_cuda.h).

The shared library is the product; this module only declares its signatures. There is
no fallback: if the library is missing or cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librie_cuda.so")

RCU_OK, RCU_ERR_INVALID, RCU_ERR_CUDA, RCU_ERR_UNSUPPORTED, RCU_ERR_OOM, RCU_ERR_TIMEOUT, RCU_ERR_RUNTIME = range(7)
STATUS_NAMES = {0: "ok", 1: "invalid", 2: "cuda", 3: "unsupported", 4: "oom", 5: "timeout", 6: "runtime"}

# Every symbol of include/rie_cuda.h with (restype, argtypes).
P, U64, I32, U32, F = C.c_void_p, C.c_uint64, C.c_int32, C.c_uint32, C.c_float
SIGNATURES = {
    "rcu_version": (I32, []),
    "rcu_ctx_create": (I32, [I32, P, C.POINTER(P), C.c_char_p, C.c_size_t]),
    "rcu_ctx_destroy": (None, [P]),
    "rcu_set_stream": (I32, [P, P]),
    "rcu_set_rounding": (I32, [P, I32]),
    "rcu_set_prefill_gemm": (I32, [P, I32]),
    "rcu_set_static_weights": (I32, [P, I32]),
    "rcu_last_error": (C.c_char_p, [P]),
    "rcu_sync": (I32, [P]),
    "rcu_check_device": (I32, [P, C.POINTER(U32)]),
    "rcu_set_wait_limit_ms": (I32, [P, U64]),
    "rcu_diag_expire_peer_wait": (I32, [P]),
    "rcu_row_bytes": (U64, [U32, U64]),
    "rcu_weight_upload": (I32, [P, U32, U64, U64, P, C.POINTER(P)]),
    "rcu_weight_view": (I32, [P, U32, U64, U64, P, C.POINTER(P)]),
    "rcu_weight_slice_rows": (I32, [P, U64, U64, C.POINTER(P)]),
    "rcu_weight_free": (None, [P]),
    "rcu_weight_device_ptr": (P, [P]),
    "rcu_acts_create": (I32, [P, U64, U64, C.POINTER(P)]),
    "rcu_acts_free": (None, [P]),
    "rcu_acts_prepare": (I32, [P, P, P, U64, U64, U32]),
    "rcu_acts_export": (I32, [P, P, U32, P]),
    "rcu_matmul_multi": (I32, [P, P, P, U64]),
    "rcu_matmul": (I32, [P, P, P, P]),
    "rcu_block_sums": (I32, [P, P, P, U64, U64, P]),
    "rcu_matmul_block_sums": (I32, [P, P, P, P, P, I32]),
    "rcu_turbo4_row_bytes": (U64, [U64]),
    "rcu_turbo4_quantize": (I32, [P, P, U64, U64, P]),
    "rcu_turbo4_rotate": (I32, [P, P, U64, U64, I32]),
    "rcu_kv_create": (I32, [P, I32, U64, U64, U64, C.POINTER(P)]),
    "rcu_kv_free": (None, [P]),
    "rcu_kv_store": (I32, [P, P, P, P, U64, U64]),
    "rcu_kv_export": (I32, [P, P, P, P]),
    "rcu_kv_import": (I32, [P, P, P, P]),
    "rcu_attention": (I32, [P, P, P, U64, U64, U64, U64, F, P]),
    "rcu_model_create": (I32, [P, P, C.POINTER(P)]),
    "rcu_model_free": (None, [P]),
    "rcu_model_set_tensor": (I32, [P, C.c_char_p, U32, U64, U64, P]),
    "rcu_model_set_tensor_device": (I32, [P, C.c_char_p, U32, U64, U64, P]),
    "rcu_quantize_weight": (I32, [P, U32, U64, U64, P, U64, P]),
    "rcu_backend_create": (I32, [P, U64, U64, I32, C.POINTER(P)]),
    "rcu_backend_free": (None, [P]),
    "rcu_backend_max_batch": (U64, [P]),
    "rcu_backend_n_ctx": (U64, [P]),
    "rcu_backend_forward": (I32, [P, P, U64, U64, I32, P, U64]),
    "rcu_backend_forward_device": (I32, [P, P, U64, U64, I32, P]),
    "rcu_backend_forward_layers": (I32, [P, P, U64, U64, U64, U64, P, P]),
    "rcu_backend_hidden": (I32, [P, P, U64, C.POINTER(U64)]),
    "rcu_matmul_f32_static": (I32, [P, P, P, U64, P, U64]),
    "rcu_backend_kv": (I32, [P, U64, C.POINTER(P)]),
    "rcu_model_create_tp": (I32, [P, P, I32, I32, C.POINTER(P)]),
    "rcu_tp_shard": (I32, [P, C.c_char_p, U32, U64, U64, P, I32, I32, P, U64, C.POINTER(U64), C.POINTER(U64)]),
    "rcu_tp_unique_id": (I32, [P, U64]),
    "rcu_backend_create_tp": (I32, [P, U64, U64, I32, P, C.POINTER(P)]),
}


class RcuJob(C.Structure):
    _fields_ = [("w", C.c_void_p), ("out", C.c_void_p), ("ld", C.c_uint64)]


class RcuError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


_lib = None


def load() -> C.CDLL:
    """Load librie_cuda.so (built in-tree by rust_interference_engine_b200.build)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m rust_interference_engine_b200.build`")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib
