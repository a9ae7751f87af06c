"""Host-side checks that need no GPU: the C ABI library loads and exports every
entry point include/funasr_cuda.h declares; the Python binding declares each
one; GGUF files written by the library parse with an independent reader and
load in the oracle; device entry points fail cleanly without a device."""
import ctypes as C
import re
import struct
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "funasr_cuda.h"


def header_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(fa_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(built_lib):
    lib = C.CDLL(str(built_lib))
    names = header_functions()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_declares_every_symbol():
    from funasrnet_b200._lib import SIGNATURES

    assert set(header_functions()) == set(SIGNATURES)


def test_binding_matches_header_prototypes():
    """Each ctypes declaration has the header prototype's parameters: the
    same count, and per parameter the same kind (pointer, integer, float) and
    width, so no call passes a 32-bit value where the C side reads 64 bits."""
    import ctypes

    from funasrnet_b200._lib import SIGNATURES

    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    protos = re.findall(r"\b(fa_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S)
    scalars = {"int": ("int", 4), "int32_t": ("int", 4), "uint32_t": ("int", 4), "unsigned": ("int", 4),
               "int64_t": ("int", 8), "uint64_t": ("int", 8), "size_t": ("int", 8), "float": ("float", 4),
               "double": ("float", 8)}

    def header_kind(param):
        if "*" in param:
            return ("pointer", 8)
        words = param.replace("const ", "").split()
        return scalars.get(" ".join(words[:-1]), ("unknown", param))

    def binding_kind(t):
        if t in (ctypes.c_void_p, ctypes.c_char_p) or issubclass(t, ctypes._Pointer):
            return ("pointer", 8)
        return ("float" if t in (ctypes.c_float, ctypes.c_double) else "int", ctypes.sizeof(t))

    assert {name for name, _ in protos} == set(SIGNATURES)
    for name, params in protos:
        params = params.strip()
        want = [] if params in ("", "void") else [header_kind(x.strip()) for x in params.split(",")]
        got = [binding_kind(t) for t in SIGNATURES[name][1]]
        assert want == got, name


def test_binding_loads(built_lib):
    from funasrnet_b200._lib import lib

    assert b"sm_100a" in lib().fa_version()


def test_backend_create_without_gpu_is_an_error(built_lib):
    import os

    from funasrnet_b200._lib import lib

    if os.path.exists("/dev/nvidia0"):
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    rc = lib().fa_backend_create(0, C.byref(h))
    assert rc < 0 and not h.value
    assert lib().fa_last_error()


def test_null_handles_are_argument_errors(built_lib):
    from funasrnet_b200._lib import lib

    assert lib().fa_backend_destroy(None) == -1
    assert lib().fa_session_free(None) == -1
    assert lib().fa_model_free(None) == -1
    assert lib().fa_session_reset(None) == -1
    assert lib().fa_try_quantized_linear(None, None, 1, None, None, None) == -1
    assert lib().fa_model_weight_bytes(None) == -1


def read_gguf(path):
    """Minimal independent GGUF v3 reader (header, metadata, tensor table)."""
    b = Path(path).read_bytes()
    off = 0

    def take(fmt):
        nonlocal off
        v = struct.unpack_from("<" + fmt, b, off)
        off += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def string():
        n = take("Q")
        nonlocal off
        s = b[off:off + n].decode()
        off += n
        return s

    def value(t):
        fmts = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "B", 10: "Q", 11: "q", 12: "d"}
        if t == 8:
            return string()
        if t == 9:
            et, n = take("I"), take("Q")
            return [value(et) for _ in range(n)]
        return take(fmts[t])

    assert take("I") == 0x46554747 and take("I") == 3
    nt, nm = take("Q"), take("Q")
    meta = {}
    for _ in range(nm):
        k = string()
        meta[k] = value(take("I"))
    tensors = {}
    for _ in range(nt):
        name = string()
        dims = [take("Q") for _ in range(take("I"))]
        typ, o = take("I"), take("Q")
        tensors[name] = (dims, typ, o)
    align = meta.get("general.alignment", 32)
    start = (off + align - 1) // align * align
    return meta, tensors, b, start


def test_synthetic_gguf_roundtrip(tmp_path, built_lib, oracle):
    from funasrnet_b200._lib import check, lib

    p = tmp_path / "m.gguf"
    check(lib().fa_synth_write_gguf(str(p).encode(), 99, 2, 640, 256, 512, 1))
    meta, tensors, raw, start = read_gguf(p)
    assert meta["qwen3.block_count"] == 2 and meta["qwen3.embedding_length"] == 256
    assert meta["qwen3.feed_forward_length"] == 512 and meta["tokenizer.ggml.eos_token_id"] == 151645
    assert len(meta["tokenizer.ggml.tokens"]) == 640 and meta["tokenizer.ggml.merges"] == []
    assert "output.weight" not in tensors  # tied embedding
    dims, typ, o = tensors["blk.1.ffn_down.weight"]
    assert dims == [512, 256] and typ == 8
    blocks = np.frombuffer(raw, np.uint8, 256 * 512 // 32 * 34, start + o).reshape(-1, 34)
    scales = blocks[:, :2].copy().view(np.float16).astype(np.float32).reshape(256, 16)
    q = blocks[:, 2:].view(np.int8).reshape(256, 512)
    m = oracle.Model(p, 64)
    oq, os_ = m.tensor_q8("blk.1.ffn_down.weight")
    assert np.array_equal(oq, q) and np.array_equal(os_, scales)
    # N(0, 0.02) weights: dequantised std within 5%
    assert abs((q * np.repeat(scales, 32, axis=1)).std() - 0.02) < 1e-3
    norm = m.tensor_f32("blk.0.attn_norm.weight")
    assert np.all(norm == 1.0)
    m.close()


def test_synth_normals_deterministic(built_lib):
    from funasrnet_b200._lib import check, lib

    a = np.empty(100000, np.float32)
    b = np.empty(50000, np.float32)
    check(lib().fa_synth_normals(5, 9001, 0, a.size, a.ctypes.data))
    check(lib().fa_synth_normals(5, 9001, 50000, b.size, b.ctypes.data))
    assert np.array_equal(a[50000:], b)
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1) < 0.02


def test_gguf_truncated_file_rejected(tmp_path, built_lib, oracle):
    from funasrnet_b200._lib import check, lib

    p = tmp_path / "m.gguf"
    check(lib().fa_synth_write_gguf(str(p).encode(), 1, 1, 256, 256, 256, 1))
    data = p.read_bytes()
    t = tmp_path / "t.gguf"
    t.write_bytes(data[: len(data) - 1000])
    with pytest.raises(RuntimeError):
        oracle.Model(t, 16)
