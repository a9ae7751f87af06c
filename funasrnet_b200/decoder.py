"""QwenDecoder and the FunAsr.Transcribe token loop on the CUDA library.

Mirrors the reference's decoder surface (src/FunAsrNet/QwenDecoder.cs):
``reset`` (:117), ``embed`` (:143-152), ``decode`` (:161-271), ``greedy``
(:278-326), ``cache_prefix``/``restore_prefix`` (:122-137), and the greedy
loop of ``FunAsr.Transcribe`` (src/FunAsrNet/FunAsr.cs:164-189) as
``transcribe_tokens``.  Every op runs in libfunasr_cuda.so; errors surface as
``FaError`` (ArgumentException for exhausted context or bad embeddings).
"""
from __future__ import annotations

import ctypes as C
import time
from dataclasses import dataclass

import numpy as np

from ._lib import FA_OK, check, lib, ptr
from .backend import CudaFloatBackend, Ops

# ByteBpe.IsEnd (src/FunAsrNet/ByteBpe.cs:57-71) ends on <|endoftext|>, <|im_end|>,
# <|fim_suffix|> when the vocabulary has them, plus tokenizer.ggml.eos_token_id.
# The ids below are <|endoftext|> and <|im_end|> of the Qwen3 vocabulary (and of
# the synthetic GGUF); callers with a real tokenizer pass its own set.
QWEN_END_TOKENS = (151643, 151645)


class CudaModel:
    """A GGUF decoder model resident on one GPU (Gguf + QwenDecoder weights)."""

    def __init__(self, backend: CudaFloatBackend, path: str, capacity: int = 2048):
        self.backend = backend
        h = C.c_void_p()
        check(lib().fa_model_load_gguf(backend.handle, str(path).encode(), capacity, C.byref(h)))
        self._h = h
        dims = np.zeros(8, np.int32)
        check(lib().fa_model_dims(h, ptr(dims)))
        (self.width, self.heads, self.kv_heads, self.head_size, self.layers, self.vocab, self.ffn,
         self.capacity) = (int(v) for v in dims)
        self.weight_bytes = int(lib().fa_model_weight_bytes(h))

    @property
    def handle(self):
        return self._h

    def close(self) -> None:
        if self._h is not None:
            check(lib().fa_model_free(self._h))
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class QwenDecoder:
    """One decoding context: its own F16 KV cache, position and CUDA stream."""

    def __init__(self, model: CudaModel):
        self.model = model
        h = C.c_void_p()
        check(lib().fa_session_create(model.handle, C.byref(h)))
        self._h = h

    @property
    def width(self) -> int:
        return self.model.width

    @property
    def position(self) -> int:
        return int(lib().fa_session_position(self._h))

    def reset(self) -> None:
        check(lib().fa_session_reset(self._h))

    def embed(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        out = np.empty(t.size * self.width, np.float32)
        check(lib().fa_session_embed(self._h, ptr(t), t.size, ptr(out)))
        return out

    def decode(self, embeddings, frames: int, output_logits: bool = True, want_logits: bool = True):
        """Decode(embeddings, frames, outputLogits): returns (logits or None, argmax or None)."""
        e = np.ascontiguousarray(embeddings, dtype=np.float32).reshape(-1)
        if frames < 1 or e.size != frames * self.width:
            raise ValueError("Decoder context exhausted or invalid embeddings")
        logits = np.empty(self.model.vocab, np.float32) if (output_logits and want_logits) else None
        arg = C.c_int32(-1)
        check(lib().fa_session_decode(self._h, ptr(e), frames, 1 if output_logits else 0, ptr(logits),
                                      C.byref(arg)))
        return logits, (arg.value if output_logits else None)

    def step(self, token: int, want_logits: bool = False):
        """Decode(Embed([token]), 1) + Greedy: returns (next_token, logits or None)."""
        logits = np.empty(self.model.vocab, np.float32) if want_logits else None
        nxt = C.c_int32()
        check(lib().fa_session_step(self._h, int(token), ptr(logits), C.byref(nxt)))
        return nxt.value, logits

    def generate(self, max_tokens: int, end_ids=QWEN_END_TOKENS) -> list[int]:
        """The FunAsr.Transcribe greedy loop on the device, from the last argmax."""
        ends = np.ascontiguousarray(end_ids, dtype=np.int32)
        toks = np.empty(max(1, max_tokens), np.int32)
        n = C.c_int32()
        check(lib().fa_session_generate(self._h, int(max_tokens), ptr(ends) if ends.size else None, ends.size,
                                        ptr(toks), C.byref(n)))
        return toks[: n.value].tolist()

    def last_generate_ms(self) -> float:
        ms = C.c_float()
        check(lib().fa_session_last_generate_ms(self._h, C.byref(ms)))
        return float(ms.value)

    def set_exact_attention(self, on: bool = True) -> None:
        """True (default): the reference's attention order, bit-identical logits."""
        check(lib().fa_session_set_exact_attention(self._h, 1 if on else 0))

    def set_debug(self, on: bool = True) -> None:
        check(lib().fa_session_set_debug(self._h, 1 if on else 0))

    def debug_layer0(self, name: str) -> np.ndarray:
        n = check(lib().fa_session_debug_layer0(self._h, name.encode(), None))
        out = np.empty(n, np.float32)
        check(lib().fa_session_debug_layer0(self._h, name.encode(), ptr(out)))
        return out

    def persistent_grid(self) -> int:
        """CTAs of the persistent decode kernel (0: CUDA-graph step path)."""
        return int(lib().fa_session_uses_persistent_kernel(self._h))

    def set_persistent(self, on: bool = True) -> bool:
        return check(lib().fa_session_set_persistent_kernel(self._h, 1 if on else 0)) == FA_OK

    def set_resident(self, on: bool = True, idle_us: int = 0) -> bool:
        """Resident serving: step() without logits posts its token to one
        persistent launch that stays running between calls (ends after idle_us
        without a token, 0 = 20 ms, or at any other call).  False when the
        persistent kernel is unavailable."""
        return check(lib().fa_session_set_resident(self._h, 1 if on else 0, int(idle_us))) == FA_OK

    def set_fault_test(self, wait_limit: int = 0, withhold_cta: int = -1) -> None:
        """Failure-path test hook for the next persistent-kernel launch only: a
        shorter bounded-wait limit (polls) and a GEMV CTA whose first q/k/v rows
        stay unpublished, so that the waits give up (FA_ERR_TIMEOUT)."""
        check(lib().fa_session_set_fault_test(self._h, int(wait_limit), int(withhold_cta)))

    def trace_phases(self, on: bool = True) -> None:
        check(lib().fa_session_set_trace(self._h, 1 if on else 0))

    def phase_trace(self) -> np.ndarray:
        """[grid x events] %globaltimer stamps (ns) of the last launch's first step."""
        n = check(lib().fa_session_get_trace(self._h, None, 0))
        out = np.zeros(n, np.uint64)
        check(lib().fa_session_get_trace(self._h, ptr(out), n))
        return out.reshape(self.persistent_grid(), -1)

    def kernels_per_step(self) -> int:
        return int(lib().fa_session_kernels_per_step(self._h))

    def time_lm_head(self, iters: int = 20) -> float:
        ms = C.c_float()
        check(lib().fa_session_time_lm_head(self._h, iters, C.byref(ms)))
        return float(ms.value)

    def cache_prefix(self, tokens) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        check(lib().fa_session_cache_prefix(self._h, ptr(t), t.size))

    def restore_prefix(self) -> None:
        check(lib().fa_session_restore_prefix(self._h))

    def share_prefix(self, source: "QwenDecoder") -> None:
        """CachePrefix from `source`'s cached prefix without decoding it again (device-to-device KV copy)."""
        check(lib().fa_session_share_prefix(self._h, source._h))

    def kv(self, layer: int):
        n = self.position * self.model.kv_heads * self.model.head_size
        k = np.empty(n, np.float32)
        v = np.empty(n, np.float32)
        check(lib().fa_session_kv(self._h, layer, ptr(k), ptr(v)))
        return k, v

    @staticmethod
    def greedy(backend: CudaFloatBackend, logits) -> int:
        return Ops(backend).greedy(logits)

    def close(self) -> None:
        if self._h is not None:
            check(lib().fa_session_free(self._h))
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class BatchDecoder:
    """n QwenDecoder sessions of one model decoded together, one token each per step.

    The reference decodes independent utterances in separate contexts that share
    read-only weights (src/FunAsrNet/SpeechRuntime.cs:18-22); this group reads every
    weight once per step for all of them.  Tokens and logits equal those of each
    session stepping alone.  Close the group before its sessions.
    """

    def __init__(self, sessions):
        self.sessions = list(sessions)
        arr = (C.c_void_p * len(self.sessions))(*[s._h.value for s in self.sessions])
        h = C.c_void_p()
        rc = check(lib().fa_batch_create(arr, len(self.sessions), C.byref(h)))
        if rc != FA_OK:
            raise NotImplementedError("model shape not supported by the batched decode path")
        self._h = h
        self.vocab = self.sessions[0].model.vocab

    def __len__(self) -> int:
        return len(self.sessions)

    def step(self, tokens=None, want_logits: bool = False):
        """One greedy step of every session: returns (next tokens [n], logits [n x vocab] or None)."""
        n = len(self.sessions)
        t = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32).reshape(n)
        nxt = np.empty(n, np.int32)
        logits = np.empty((n, self.vocab), np.float32) if want_logits else None
        check(lib().fa_batch_step(self._h, ptr(t), ptr(nxt), ptr(logits)))
        return nxt, logits

    def generate(self, steps: int) -> np.ndarray:
        """`steps` Transcribe-loop iterations per session (no end stop): [steps x n] emitted
        tokens, the first row being each session's last argmax, as QwenDecoder.generate."""
        out = np.empty((max(1, steps), len(self.sessions)), np.int32)
        check(lib().fa_batch_generate(self._h, int(steps), ptr(out)))
        return out[:steps]

    def generate_until(self, max_steps: int, end_ids=QWEN_END_TOKENS) -> list[list[int]]:
        """The Transcribe loop with its end-token stop, per session (as QwenDecoder.generate)."""
        ends = np.ascontiguousarray(end_ids, dtype=np.int32)
        n = len(self.sessions)
        out = np.empty((max(1, max_steps), n), np.int32)
        counts = np.zeros(n, np.int32)
        check(lib().fa_batch_generate_until(self._h, int(max_steps), ptr(ends) if ends.size else None, ends.size,
                                            ptr(out), ptr(counts)))
        return [out[: counts[i], i].tolist() for i in range(n)]

    def last_ms(self) -> float:
        ms = C.c_float()
        check(lib().fa_batch_last_ms(self._h, C.byref(ms)))
        return float(ms.value)

    def close(self) -> None:
        if getattr(self, "_h", None) is not None:
            check(lib().fa_batch_free(self._h))
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


@dataclass
class DecodeResult:
    tokens: list
    prefill_seconds: float
    generation_seconds: float


def transcribe_tokens(decoder: QwenDecoder, embeddings: np.ndarray, frames: int, max_tokens: int = 128,
                      end_ids=QWEN_END_TOKENS, on_device: bool = True) -> DecodeResult:
    """The decoder half of FunAsr.Transcribe (FunAsr.cs:156-189) with prompt cache off.

    on_device=True runs the whole greedy loop as replayed CUDA graphs with one
    synchronisation at the end; on_device=False drives it token by token from
    the host, as the reference's loop does.
    """
    t0 = time.perf_counter()
    decoder.reset()
    _, token = decoder.decode(embeddings, frames, output_logits=True, want_logits=False)
    t1 = time.perf_counter()
    if on_device:
        tokens = decoder.generate(max_tokens, end_ids)
    else:
        ends = set(int(e) for e in end_ids)
        tokens = []
        for _ in range(max_tokens):
            if token in ends:
                break
            tokens.append(token)
            token, _ = decoder.step(token)
    t2 = time.perf_counter()
    return DecodeResult(tokens, t1 - t0, t2 - t1)
