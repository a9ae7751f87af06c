"""Host-side mirror of FunAsrNet's compute-backend slot for the CUDA library.

``CudaFloatBackend`` implements the reference's three projection interfaces
with the same argument meaning and error behaviour:

* ``IFloatComputeBackend.TryLinear`` (src/FunAsrNet/IFloatComputeBackend.cs:19)
* ``IQuantizedComputeBackend.TryQuantizedLinear`` (src/FunAsrNet/IQuantizedComputeBackend.cs:13)
* ``IGroupedComputeBackend.TryLinearMany`` (src/FunAsrNet/IGroupedComputeBackend.cs:12)

"return False" means unsupported: the output is untouched and the caller's
CPU path continues.  Shape mismatches raise ``ValueError`` (ArgumentException),
use after ``dispose`` raises ``RuntimeError`` (ObjectDisposedException).
Weights become resident on first use and are keyed by object identity, like
the Vulkan backend's residency cache (src/FunAsrNet.Vulkan/VulkanFloatBackend.cs:14,242-283).
"""
from __future__ import annotations

import ctypes as C
import threading
import weakref
from dataclasses import dataclass, field

import numpy as np

from ._lib import FA_DECLINED, FA_OK, FaError, check, lib, ptr


@dataclass(eq=False)
class Weight:
    """The reference's Weight (src/FunAsrNet/Gguf.cs:264-346).

    shape is innermost first: Columns = shape[0] (K), Rows = shape[1] (N).
    Q8 weights carry ``quantized`` (int8, rows x cols) and ``scales``
    (float32, rows x cols/32); FP32 weights carry ``values``.
    """

    name: str
    shape: tuple
    values: np.ndarray | None = None
    quantized: np.ndarray | None = None
    scales: np.ndarray | None = None
    extra: dict = field(default_factory=dict)

    @property
    def columns(self) -> int:
        return int(self.shape[0])

    @property
    def rows(self) -> int:
        return int(self.shape[1]) if len(self.shape) > 1 else 1


class CudaFloatBackend:
    """Drop-in for VulkanFloatBackend in ``FunAsr.FloatBackend`` (FunAsr.cs:67-71)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib().fa_backend_create(device, C.byref(h)))
        self._h = h
        self._lock = threading.Lock()
        self._resident: "weakref.WeakKeyDictionary[Weight, C.c_void_p]" = weakref.WeakKeyDictionary()
        self._disposed = False

    # IFloatComputeBackend.Name
    @property
    def name(self) -> str:
        return lib().fa_backend_name(self._h).decode()

    @property
    def handle(self) -> C.c_void_p:
        self._check()
        return self._h

    def _check(self) -> None:
        if self._disposed:
            raise RuntimeError("CudaFloatBackend is disposed")

    def _resident_handle(self, w: Weight) -> C.c_void_p:
        h = self._resident.get(w)
        if h is not None:
            return h
        h = C.c_void_p()
        if w.quantized is not None:
            q = np.ascontiguousarray(w.quantized, dtype=np.int8).reshape(-1)
            s = np.ascontiguousarray(w.scales, dtype=np.float32).reshape(-1)
            if q.size < w.rows * w.columns or s.size < w.rows * (w.columns // 32):
                raise ValueError(f"{w.name}: truncated Q8 weight")
            check(lib().fa_weight_upload_q8(self._h, ptr(q), ptr(s), w.rows, w.columns, C.byref(h)))
        else:
            v = np.ascontiguousarray(w.values, dtype=np.float32).reshape(-1)
            if v.size < w.rows * w.columns:
                raise ValueError(f"{w.name}: truncated weight")
            check(lib().fa_weight_upload_f32(self._h, ptr(v), w.rows, w.columns, C.byref(h)))
        self._resident[w] = h
        return h

    def _linear(self, fn, inp: np.ndarray, frames: int, w: Weight, bias: Weight | None, out: np.ndarray) -> bool:
        self._check()
        if frames <= 0 or w.columns <= 0 or w.rows <= 0:
            return False
        x = np.ascontiguousarray(inp, dtype=np.float32).reshape(-1)
        if x.size != frames * w.columns or out.size != frames * w.rows:
            raise ValueError(f"{w.name}: projection shape mismatch")
        if out.dtype != np.float32 or not out.flags["C_CONTIGUOUS"]:
            raise ValueError("output must be a contiguous float32 array")
        b = None
        if bias is not None and bias.values is not None:
            b = np.ascontiguousarray(bias.values, dtype=np.float32).reshape(-1)
            if b.size != w.rows:
                raise ValueError("bias length differs from the output rows")
        with self._lock:
            h = self._resident_handle(w)
            rc = check(fn(self._h, ptr(x), frames, h, ptr(b), ptr(out)))
        return rc == FA_OK

    # IQuantizedComputeBackend.TryQuantizedLinear
    def try_quantized_linear(self, inp, frames, w: Weight, bias, out) -> bool:
        if w.quantized is None or w.scales is None or w.columns % 32 != 0:
            return False
        return self._linear(lib().fa_try_quantized_linear, inp, frames, w, bias, out)

    # IFloatComputeBackend.TryLinear
    def try_linear(self, inp, frames, w: Weight, bias, out) -> bool:
        if w.values is None:
            return False
        return self._linear(lib().fa_try_linear, inp, frames, w, bias, out)

    # IFloatComputeBackend.TryConvolution: encoder-only, never handled here.
    def try_convolution(self, *args, **kwargs):
        return False, None

    # IGroupedComputeBackend.TryLinearMany
    def try_linear_many(self, inp, frames, weights) -> tuple[bool, list[np.ndarray] | None]:
        self._check()
        if len(weights) < 2 or frames <= 0:
            return False, None
        if any(w.quantized is None or w.columns != weights[0].columns or w.columns % 32 for w in weights):
            return False, None
        x = np.ascontiguousarray(inp, dtype=np.float32).reshape(-1)
        if x.size != frames * weights[0].columns:
            raise ValueError("Grouped projection dimensions differ")
        outs = [np.empty(frames * w.rows, dtype=np.float32) for w in weights]
        with self._lock:
            hs = (C.c_void_p * len(weights))(*[self._resident_handle(w).value for w in weights])
            os_ = (C.c_void_p * len(weights))(*[o.ctypes.data for o in outs])
            rc = check(lib().fa_try_linear_many(self._h, ptr(x), frames, hs, len(weights), os_))
        if rc == FA_DECLINED:
            return False, None
        return True, outs

    def make_resident(self, w: Weight) -> None:
        """Uploads ``w`` to the device now rather than on its first use."""
        self._check()
        with self._lock:
            self._resident_handle(w)

    # Allocation-free lm_head step (no counterpart in the reference).
    def lm_head_argmax_noalloc(self, w: Weight, x: int, gamma: int | None, eps: float, logits: int | None,
                               token: int, stream: int | None = None) -> bool:
        """Enqueues RMSNorm (skipped when ``gamma`` is None) + the Q8 projection
        by ``w`` + the greedy argmax of one frame on ``stream`` and returns
        without waiting.  ``x``, ``gamma``, ``logits`` and ``token`` are device
        addresses; ``w`` must be resident already (``make_resident``), so that
        the call allocates nothing.  False when declined."""
        self._check()
        with self._lock:
            h = self._resident.get(w)
            if h is None:
                raise ValueError(f"{w.name}: not resident; call make_resident first")
            rc = check(lib().fa_lm_head_argmax_noalloc(self._h, h, x, gamma, eps, logits, token, stream))
        return rc == FA_OK

    def dispose(self) -> None:
        if self._disposed:
            return
        self._resident.clear()
        check(lib().fa_backend_destroy(self._h))
        self._disposed = True

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class Ops:
    """Single decoder ops through the C ABI (the kernels of the decode step)."""

    def __init__(self, backend: CudaFloatBackend):
        self.b = backend

    def quantize(self, x):
        x = _f32(x).reshape(-1)
        q = np.empty(x.size, np.int8)
        s = np.empty(x.size // 32, np.float32)
        check(lib().fa_op_quantize(self.b.handle, ptr(x), x.size, ptr(q), ptr(s)))
        return q, s

    def rmsnorm(self, x, width, gamma, eps=1e-6):
        x = _f32(x).reshape(-1)
        g = _f32(gamma).reshape(-1)
        y = np.empty_like(x)
        check(lib().fa_op_rmsnorm(self.b.handle, ptr(x), x.size, width, ptr(g), eps, ptr(y)))
        return y

    def round_half(self, x):
        x = _f32(x).reshape(-1)
        y = np.empty_like(x)
        check(lib().fa_op_round_half(self.b.handle, ptr(x), x.size, ptr(y)))
        return y

    def silu_mul(self, gate, up):
        g = _f32(gate).reshape(-1).copy()
        u = _f32(up).reshape(-1)
        check(lib().fa_op_silu_mul(self.b.handle, ptr(g), ptr(u), g.size))
        return g

    def greedy(self, logits) -> int:
        x = _f32(logits).reshape(-1)
        t = C.c_int32()
        check(lib().fa_op_greedy(self.b.handle, ptr(x), x.size, C.byref(t)))
        return t.value

    def attention_pair(self, q, k, v, frames, kv_heads, size, out=None):
        q, k, v = _f32(q).reshape(-1), _f32(k).reshape(-1), _f32(v).reshape(-1)
        if out is None:
            out = np.zeros(q.size, np.float32)
        rc = check(lib().fa_op_attention_pair(self.b.handle, ptr(q), ptr(k), ptr(v), frames, kv_heads, size, ptr(out)))
        return (rc == FA_OK), out


__all__ = ["CudaFloatBackend", "Weight", "Ops", "FaError"]
