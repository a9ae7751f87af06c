"""TEST INFRASTRUCTURE ONLY: ctypes wrapper of the CPU oracle (liboracle.so).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may use
this module, and only as the checker or the timed CPU baseline.  It restates
FunAsrNet's C# decoder (see qwen_oracle.h for the per-function citations).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

_lib = None


def build() -> Path:
    r = subprocess.run(["make", "-C", str(HERE)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed\n{r.stdout}\n{r.stderr}")
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        h = C.CDLL(str(LIB))
        vp, i32, i64, f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_float
        sigs = {
            "or_set_threads": (None, [i32]),
            "or_get_threads": (i32, []),
            "or_quantize": (i32, [vp, i64, vp, vp]),
            "or_q8_linear": (i32, [vp, i32, vp, vp, i32, i32, vp, vp]),
            "or_f32_linear": (i32, [vp, i32, vp, i32, i32, vp, vp]),
            "or_rmsnorm": (i32, [vp, i64, i32, vp, f32, vp]),
            "or_rope_table": (None, [i32, i32, f32, vp, vp]),
            "or_rotate_half": (None, [vp, i32, vp, vp]),
            "or_round_half": (None, [vp, i64, vp]),
            "or_dot": (f32, [vp, vp, i32]),
            "or_softmax": (None, [vp, i32]),
            "or_attention_pair": (i32, [vp, vp, vp, i32, i32, i32, vp]),
            "or_silu_mul": (None, [vp, vp, i64]),
            "or_greedy": (i64, [vp, i64]),
            "or_exp": (f32, [f32]),
            "or_set_exp_mode": (i32, [i32]),
            "or_get_exp_mode": (i32, []),
            "or_half_to_float": (f32, [C.c_uint16]),
            "or_float_to_half": (C.c_uint16, [f32]),
            "or_model_load": (vp, [C.c_char_p, i32]),
            "or_model_free": (None, [vp]),
            "or_last_error": (C.c_char_p, []),
            "or_model_dims": (i32, [vp, vp]),
            "or_embed": (i32, [vp, vp, i32, vp]),
            "or_tensor_info": (i32, [vp, C.c_char_p, vp, vp]),
            "or_tensor_q8": (i32, [vp, C.c_char_p, vp, vp]),
            "or_tensor_f32": (i32, [vp, C.c_char_p, vp]),
            "or_session_create": (vp, [vp]),
            "or_session_free": (None, [vp]),
            "or_session_reset": (None, [vp]),
            "or_session_position": (i32, [vp]),
            "or_session_decode": (i32, [vp, vp, i32, vp]),
            "or_session_cache_prefix": (i32, [vp, vp, i32]),
            "or_session_restore_prefix": (i32, [vp]),
            "or_session_kv": (i32, [vp, i32, vp, vp]),
            "or_session_trace_layer0": (i32, [vp, vp]),
            "or_session_debug": (i32, [vp, C.c_char_p, vp]),
            "or_synth_normals": (i32, [C.c_uint64, C.c_uint64, C.c_uint64, i64, vp]),
            "or_synth_write_gguf": (i32, [C.c_char_p, C.c_uint64, i32, i32, i32, i32, i32]),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


EXP_LOCAL, EXP_RUNTIME = 0, 1


def set_exp_mode(mode: int) -> None:
    """0: the reference's ExpAvx everywhere (its .NET 11 selection, the default);
    1: the correctly rounded exp standing in for the .NET 10 runtime exp."""
    if lib().or_set_exp_mode(int(mode)) != 0:
        raise ValueError(f"bad exp mode {mode}")


def get_exp_mode() -> int:
    return int(lib().or_get_exp_mode())


def quantize(x):
    x = f32(x).reshape(-1)
    q = np.empty(x.size, np.int8)
    s = np.empty(x.size // 32, np.float32)
    if lib().or_quantize(_p(x), x.size, _p(q), _p(s)) != 0:
        raise ValueError("Quantization needs matching complete blocks")
    return q, s


def q8_linear(x, frames, q, scales, rows, cols, bias=None):
    x = f32(x).reshape(-1)
    q = np.ascontiguousarray(q, dtype=np.int8).reshape(-1)
    s = f32(scales).reshape(-1)
    b = None if bias is None else f32(bias).reshape(-1)
    out = np.empty(frames * rows, np.float32)
    if lib().or_q8_linear(_p(x), frames, _p(q), _p(s), rows, cols, _p(b), _p(out)) != 0:
        raise ValueError("bad q8 linear arguments")
    return out


def f32_linear(x, frames, w, rows, cols, bias=None):
    x = f32(x).reshape(-1)
    w = f32(w).reshape(-1)
    b = None if bias is None else f32(bias).reshape(-1)
    out = np.empty(frames * rows, np.float32)
    lib().or_f32_linear(_p(x), frames, _p(w), rows, cols, _p(b), _p(out))
    return out


def rmsnorm(x, width, gamma, eps=1e-6):
    x = f32(x).reshape(-1)
    g = f32(gamma).reshape(-1)
    y = np.empty_like(x)
    if lib().or_rmsnorm(_p(x), x.size, width, _p(g), eps, _p(y)) != 0:
        raise ValueError("Invalid normalization dimensions")
    return y


def rope_table(capacity, head_size, base):
    c = np.empty(capacity * head_size // 2, np.float32)
    s = np.empty_like(c)
    lib().or_rope_table(capacity, head_size, base, _p(c), _p(s))
    return c, s


def rotate_half(x, cos, sin):
    x = f32(x).copy()
    lib().or_rotate_half(_p(x), x.size // 2, _p(f32(cos)), _p(f32(sin)))
    return x


def round_half(x):
    x = f32(x).reshape(-1)
    y = np.empty_like(x)
    lib().or_round_half(_p(x), x.size, _p(y))
    return y


def softmax(x):
    x = f32(x).copy()
    lib().or_softmax(_p(x), x.size)
    return x


def attention_pair(q, k, v, frames, kv_heads, size):
    q, k, v = f32(q).reshape(-1), f32(k).reshape(-1), f32(v).reshape(-1)
    out = np.empty(q.size, np.float32)
    lib().or_attention_pair(_p(q), _p(k), _p(v), frames, kv_heads, size, _p(out))
    return out


def silu_mul(g, u):
    g = f32(g).reshape(-1).copy()
    u = f32(u).reshape(-1)
    lib().or_silu_mul(_p(g), _p(u), g.size)
    return g


def greedy(logits) -> int:
    x = f32(logits).reshape(-1)
    return int(lib().or_greedy(_p(x), x.size))


def synth_normals(seed: int, stream: int, start: int, n: int):
    out = np.empty(n, np.float32)
    if lib().or_synth_normals(seed, stream, start, n, _p(out)) != 0:
        raise ValueError("bad synth_normals arguments")
    return out


def synth_write_gguf(path, seed: int, layers=0, vocab=0, width=0, ffn=0, quantized=True) -> None:
    if lib().or_synth_write_gguf(str(path).encode(), seed, layers, vocab, width, ffn, 1 if quantized else 0) != 0:
        raise OSError(f"cannot write {path}")


def half_to_float(bits: int) -> float:
    return float(lib().or_half_to_float(bits))


class Model:
    def __init__(self, path, capacity=2048):
        self.h = lib().or_model_load(str(path).encode(), capacity)
        if not self.h:
            raise RuntimeError(lib().or_last_error().decode())
        d = np.zeros(8, np.int32)
        lib().or_model_dims(self.h, _p(d))
        (self.width, self.heads, self.kv_heads, self.head_size, self.layers, self.vocab, self.ffn,
         self.quantized) = (int(v) for v in d)

    def embed(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        out = np.empty(t.size * self.width, np.float32)
        if lib().or_embed(self.h, _p(t), t.size, _p(out)) != 0:
            raise ValueError(lib().or_last_error().decode())
        return out

    def tensor_q8(self, name):
        shape = np.zeros(4, np.int64)
        typ = np.zeros(1, np.int32)
        if lib().or_tensor_info(self.h, name.encode(), _p(shape), _p(typ)) != 0:
            raise KeyError(name)
        cols, rows = int(shape[0]), int(shape[1])
        q = np.empty(rows * cols, np.int8)
        s = np.empty(rows * cols // 32, np.float32)
        if lib().or_tensor_q8(self.h, name.encode(), _p(q), _p(s)) != 0:
            raise KeyError(name)
        return q.reshape(rows, cols), s.reshape(rows, cols // 32)

    def tensor_f32(self, name):
        shape = np.zeros(4, np.int64)
        typ = np.zeros(1, np.int32)
        if lib().or_tensor_info(self.h, name.encode(), _p(shape), _p(typ)) != 0:
            raise KeyError(name)
        n = int(np.prod(shape))
        v = np.empty(n, np.float32)
        if lib().or_tensor_f32(self.h, name.encode(), _p(v)) != 0:
            raise KeyError(name)
        return v

    def close(self):
        if self.h:
            lib().or_model_free(self.h)
            self.h = None


class Session:
    def __init__(self, model: Model):
        self.model = model
        self.h = lib().or_session_create(model.h)

    @property
    def position(self):
        return int(lib().or_session_position(self.h))

    def reset(self):
        lib().or_session_reset(self.h)

    def decode(self, emb, frames, want_logits=True):
        e = f32(emb).reshape(-1)
        logits = np.empty(self.model.vocab, np.float32) if want_logits else None
        if lib().or_session_decode(self.h, _p(e), frames, _p(logits)) != 0:
            raise ValueError(lib().or_last_error().decode())
        return logits

    def cache_prefix(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        if lib().or_session_cache_prefix(self.h, _p(t), t.size) != 0:
            raise ValueError(lib().or_last_error().decode())

    def restore_prefix(self):
        lib().or_session_restore_prefix(self.h)

    def debug_layer0(self, name):
        n = lib().or_session_debug(self.h, name.encode(), None)
        if n < 0:
            raise KeyError(name)
        out = np.empty(n, np.float32)
        lib().or_session_debug(self.h, name.encode(), _p(out))
        return out

    def kv(self, layer):
        n = self.position * self.model.kv_heads * self.model.head_size
        k = np.empty(n, np.float32)
        v = np.empty(n, np.float32)
        lib().or_session_kv(self.h, layer, _p(k), _p(v))
        return k, v

    def close(self):
        if self.h:
            lib().or_session_free(self.h)
            self.h = None
