"""ctypes binding of libfunasr_cuda.so (declared in include/funasr_cuda.h).

The library must exist in-tree (built by ``python -m funasrnet_b200.build`` or
``__graft_entry__.build()``); there is no CPU fallback, so a missing library
raises at import of the first call.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libfunasr_cuda.so"

FA_OK = 0
FA_DECLINED = 1
ERRORS = {
    -1: "argument",
    -2: "capacity",
    -3: "disposed",
    -4: "cuda",
    -5: "io",
    -6: "timeout",
}

_lock = threading.Lock()
_lib = None

i32, i64, u64, f32 = C.c_int32, C.c_int64, C.c_uint64, C.c_float
vp, cp = C.c_void_p, C.c_char_p
P = C.POINTER

SIGNATURES = {
    "fa_last_error": (cp, []),
    "fa_version": (cp, []),
    "fa_backend_create": (i32, [i32, P(vp)]),
    "fa_backend_destroy": (i32, [vp]),
    "fa_backend_name": (cp, [vp]),
    "fa_weight_upload_q8": (i32, [vp, vp, vp, i32, i32, P(vp)]),
    "fa_weight_upload_f32": (i32, [vp, vp, i32, i32, P(vp)]),
    "fa_weight_release": (i32, [vp, vp]),
    "fa_try_quantized_linear": (i32, [vp, vp, i32, vp, vp, vp]),
    "fa_try_linear": (i32, [vp, vp, i32, vp, vp, vp]),
    "fa_try_linear_many": (i32, [vp, vp, i32, P(vp), i32, P(vp)]),
    "fa_op_quantize": (i32, [vp, vp, i64, vp, vp]),
    "fa_op_rmsnorm": (i32, [vp, vp, i64, i32, vp, f32, vp]),
    "fa_op_round_half": (i32, [vp, vp, i64, vp]),
    "fa_op_silu_mul": (i32, [vp, vp, vp, i64]),
    "fa_op_greedy": (i32, [vp, vp, i64, P(i32)]),
    "fa_op_attention_pair": (i32, [vp, vp, vp, vp, i32, i32, i32, vp]),
    "fa_model_load_gguf": (i32, [vp, cp, i32, P(vp)]),
    "fa_model_free": (i32, [vp]),
    "fa_model_dims": (i32, [vp, vp]),
    "fa_model_weight_bytes": (i64, [vp]),
    "fa_synth_write_gguf": (i32, [cp, u64, i32, i32, i32, i32, i32]),
    "fa_synth_normals": (i32, [u64, u64, u64, i64, vp]),
    "fa_session_create": (i32, [vp, P(vp)]),
    "fa_session_free": (i32, [vp]),
    "fa_session_reset": (i32, [vp]),
    "fa_session_position": (i32, [vp]),
    "fa_session_embed": (i32, [vp, vp, i32, vp]),
    "fa_session_decode": (i32, [vp, vp, i32, i32, vp, P(i32)]),
    "fa_session_step": (i32, [vp, i32, vp, P(i32)]),
    "fa_session_generate": (i32, [vp, i32, vp, i32, vp, P(i32)]),
    "fa_session_last_generate_ms": (i32, [vp, P(f32)]),
    "fa_session_cache_prefix": (i32, [vp, vp, i32]),
    "fa_session_restore_prefix": (i32, [vp]),
    "fa_session_share_prefix": (i32, [vp, vp]),
    "fa_session_kv": (i32, [vp, i32, vp, vp]),
    "fa_session_kernels_per_step": (i32, [vp]),
    "fa_session_uses_persistent_kernel": (i32, [vp]),
    "fa_session_set_persistent_kernel": (i32, [vp, i32]),
    "fa_session_set_resident": (i32, [vp, i32, i32]),
    "fa_session_set_trace": (i32, [vp, i32]),
    "fa_session_set_fault_test": (i32, [vp, C.c_uint32, i32]),
    "fa_session_get_trace": (i32, [vp, vp, i32]),
    "fa_session_set_debug": (i32, [vp, i32]),
    "fa_session_set_exact_attention": (i32, [vp, i32]),
    "fa_session_debug_layer0": (i32, [vp, cp, vp]),
    "fa_session_time_lm_head": (i32, [vp, i32, P(f32)]),
    "fa_lm_head_argmax_noalloc": (i32, [vp, vp, vp, vp, f32, vp, vp, vp]),
    "fa_batch_create": (i32, [vp, i32, P(vp)]),
    "fa_batch_free": (i32, [vp]),
    "fa_batch_size": (i32, [vp]),
    "fa_batch_step": (i32, [vp, vp, vp, vp]),
    "fa_batch_generate": (i32, [vp, i32, vp]),
    "fa_batch_generate_until": (i32, [vp, i32, vp, i32, vp, vp]),
    "fa_batch_last_ms": (i32, [vp, P(f32)]),
}


class FaError(RuntimeError):
    """A negative status from the library (message from fa_last_error)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{ERRORS.get(code, code)}] {message}")
        self.code = code


def lib() -> C.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m funasrnet_b200.build` "
                                   "(there is no CPU fallback)")
            handle = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
        return _lib


def check(status: int) -> int:
    """Raises FaError on a negative status; returns FA_OK or FA_DECLINED."""
    if status < 0:
        raise FaError(status, lib().fa_last_error().decode(errors="replace"))
    return status


def ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("arrays passed to the library must be C-contiguous")
    return a.ctypes.data
