"""Deterministic inputs shaped like the reference's own checks.

The reference's checks draw values from .NET's System.Random, which cannot be
reproduced outside .NET; the deterministic parts (patterns, half-way cases,
special values) are restated exactly and the random parts use numpy seeds.
"""
from __future__ import annotations

import numpy as np


def quantize_rounding_input(seed: int = 12104) -> np.ndarray:
    """tests/FunAsrNet.Checks/QuantizeRoundingChecks.cs:14-30."""
    rng = np.random.default_rng(seed)
    values: list[np.ndarray] = []
    for value in range(-126, 127):
        halfway = np.float32(value) + np.float32(0.5)
        block = np.zeros(32, np.float32)
        block[0] = 127.0
        block[1] = halfway
        block[2] = np.nextafter(halfway, np.float32(-np.inf))
        block[3] = np.nextafter(halfway, np.float32(np.inf))
        values.append(block)
    for b in range(2048):
        scale = np.float32(np.ldexp(1.0, b % 250 - 149))
        r = (rng.random(32) - 0.5).astype(np.float32)
        values.append((r * scale).astype(np.float32))
    specials = [0.0, -0.0, np.float32(1.4e-45), np.finfo(np.float32).max, np.nan, np.inf, -np.inf]
    for sp in specials:
        block = np.zeros(32, np.float32)
        block[17] = sp
        values.append(block)
    return np.concatenate(values).astype(np.float32)


def q8_avx_case(frames: int, width: int, rows: int):
    """tests/FunAsrNet.Checks/QuantizedAvxChecks.cs:17-32 (fully deterministic)."""
    pat_x = np.array([-1.0, 1.0, 0.0, -0.5, 0.1], np.float32)
    pat_w = np.array([-128, 127, 0, -127], np.int8)
    x = pat_x[np.arange(frames * width) % 5]
    q = pat_w[np.arange(width * rows) % 4].reshape(rows, width)
    s = np.where(np.arange(width * rows // 32) % 2 == 0, np.float32(0.013), np.float32(-0.007)).astype(np.float32)
    bias = (np.arange(rows) * 0.125).astype(np.float32)
    return x, q, s.reshape(rows, width // 32), bias


Q8_AVX_GRID = [(f, w, r) for f in (1, 3, 17) for w in (32, 96, 1024) for r in (1, 3, 19, 32)]


def half_rounding_input() -> np.ndarray:
    """tests/FunAsrNet.Checks/Program.cs:366-388: every binary16 value and both
    neighbours of every rounding midpoint, plus 10000 random bit patterns."""
    halves = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    out = [halves]
    fin = np.arange(0x7bff, dtype=np.uint32).astype(np.uint16)
    v = fin.view(np.float16).astype(np.float32)
    nxt = (fin + 1).astype(np.uint16).view(np.float16).astype(np.float32)
    mid = ((v + nxt) * np.float32(0.5)).astype(np.float32)
    up = np.nextafter(mid, np.float32(np.inf))
    dn = np.nextafter(mid, np.float32(-np.inf))
    out += [mid, up, dn, -mid, -up, -dn]
    rng = np.random.default_rng(385)
    out.append(rng.integers(0, 2**32, 10000, dtype=np.uint64).astype(np.uint32).view(np.float32))
    return np.concatenate(out).astype(np.float32)


def q8_weight(rng, rows: int, cols: int, std: float = 0.02):
    """A Q8_0 weight as the GGUF loader unpacks it: f16 scales, int8 in [-127, 127]."""
    w = (rng.standard_normal((rows, cols)) * std).astype(np.float32)
    blocks = w.reshape(rows, cols // 32, 32)
    amax = np.abs(blocks).max(axis=2)
    d = (amax / np.float32(127)).astype(np.float16).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(d[..., None] == 0, 0, np.round(blocks / d[..., None]))
    q = np.clip(q, -127, 127).astype(np.int8).reshape(rows, cols)
    return q, d.astype(np.float32)
