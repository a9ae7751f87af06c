"""Generates the golden fixtures in this folder (committed; rerun to refresh).

    python tests/golden/make_golden.py

Expected values are computed here with numpy, independently of the C++ oracle,
from the deterministic inputs of the reference's own checks:

* q8_linear_extremes.npz -- tests/FunAsrNet.Checks/QuantizedAvxChecks.cs:17-52:
  patterned activations / weights (incl. -128) / alternating scales / bias;
  expected = bias + sum_b ((float)dot_b * ws) * xs in block order.
* quantize_rounding.npz -- QuantizeRoundingChecks.cs:14-48: half-way
  neighbours, 2^-149..2^100 scaled blocks, specials; expected by the scalar
  rule d = amax/127, q = clamp(round-half-away(x * (1/d)), -127, 127).
* half_rounding.npz -- Program.cs:366-399: every binary16 value, both
  neighbours of every rounding midpoint, random bit patterns; expected =
  numpy's float32 -> float16 -> float32 (IEEE round-to-nearest-even).
* f16_scales.npz -- Q8ModelLoadingChecks.cs:13-35: all 65,536 binary16 scale
  patterns widened to float32 (NaNs: payload kept, quiet bit set).
* rmsnorm.npz -- TensorMath.Elementwise.cs:59-96 evaluated in float64 / float32.
* greedy.npz -- QwenDecoder.cs:278-326 edge cases.
* exp_ref.npz -- TensorMath.ExpAvx.cs:24-57 evaluated with Python floats
  (IEEE double; each FMA rounded once via exact rationals).
"""
from __future__ import annotations

import math
import sys
from fractions import Fraction
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from cases import Q8_AVX_GRID, half_rounding_input, q8_avx_case, quantize_rounding_input  # noqa: E402

f32 = np.float32


def quantize_expected(x: np.ndarray):
    x = x.astype(np.float32).reshape(-1, 32)
    q = np.zeros(x.shape, np.int8)
    d = np.zeros(x.shape[0], np.float32)
    with np.errstate(all="ignore"):
        for i, blk in enumerate(x):
            amax = f32(0)
            nan = False
            for v in blk:
                if np.isnan(v):
                    nan = True
                amax = max(amax, abs(v)) if not nan else amax
            if nan:
                amax = f32(np.nan)
            di = f32(amax / f32(127))
            inv = f32(0) if di == 0 else f32(f32(1) / di)
            d[i] = di
            for j, v in enumerate(blk):
                t = f32(v * inv)
                if np.isnan(t):
                    r = 0
                elif np.isinf(t):
                    r = 127 if t > 0 else -127
                else:
                    tr = np.trunc(t)
                    if abs(t - tr) >= 0.5:
                        tr = tr + np.sign(t)
                    r = int(np.clip(tr, -(2**31), 2**31 - 1))
                q[i, j] = np.clip(r, -127, 127)
    return q.reshape(-1), d


def q8_linear_expected(x, frames, q, s, rows, width, bias):
    qx, xs = quantize_expected(x)
    qx = qx.reshape(frames, width).astype(np.int32)
    xs = xs.reshape(frames, width // 32)
    w = q.astype(np.int32)
    out = np.zeros(frames * rows, np.float32)
    for t in range(frames):
        for r in range(rows):
            acc = f32(0)
            for b in range(width // 32):
                dot = int(np.dot(w[r, b * 32:(b + 1) * 32], qx[t, b * 32:(b + 1) * 32]))
                acc = f32(acc + f32(f32(f32(dot) * s[r, b]) * xs[t, b]))
            out[t * rows + r] = f32(bias[r] + acc)
    return out


def half_to_float_expected(bits: np.ndarray) -> np.ndarray:
    h = bits.astype(np.uint16)
    out = h.view(np.float16).astype(np.float32)
    nan = (h & 0x7C00) == 0x7C00
    nan &= (h & 0x03FF) != 0
    sign = (h.astype(np.uint32) & 0x8000) << 16
    payload = (h.astype(np.uint32) & 0x03FF) << 13
    nbits = sign | np.uint32(0x7FC00000) | payload
    out = out.view(np.uint32)
    out[nan] = nbits[nan]
    return out.view(np.float32)


def rmsnorm_expected(x, width, g, eps):
    x = x.astype(np.float32).reshape(-1, width)
    y = np.empty_like(x)
    for i, row in enumerate(x):
        acc = [0.0, 0.0, 0.0, 0.0]
        for k in range(0, width - width % 4, 4):
            for j in range(4):
                z = float(row[k + j])
                acc[j] = acc[j] + z * z
        var = (acc[0] + acc[2]) + (acc[1] + acc[3])
        for k in range(width - width % 4, width):
            var += float(row[k]) ** 2
        inv = f32(f32(1) / np.sqrt(f32(f32(var / width) + f32(eps))))
        y[i] = ((row * inv).astype(np.float32) * g).astype(np.float32)
    return y.reshape(-1)


def fma(a: float, b: float, c: float) -> float:
    """Correctly rounded a*b+c (exact rational arithmetic, one rounding)."""
    return float(Fraction(a) * Fraction(b) + Fraction(c))


def exp_ref(v: float) -> float:
    """TensorMath.ExpAvx, one lane, in IEEE double (Python floats)."""
    v = float(np.float32(v))
    if math.isnan(v):
        return v
    c = min(104.0, max(-104.0, v))
    n = float(round(c * 1.4426950408889634074))  # Python round(): half to even
    r = fma(n, -0.6931471805599453094, c)
    sq = r * r
    fo = sq * sq
    p23 = fma(r, 1.0 / 6, 0.5)
    p45 = fma(r, 1.0 / 120, 1.0 / 24)
    p67 = fma(r, 1.0 / 5040, 1.0 / 720)
    low = fma(sq, p23, 1.0 + r)
    high = fma(sq, fma(sq, 1.0 / 40320, p67), p45)
    e = fma(fo, high, low)
    return float(np.float32(e * math.ldexp(1.0, int(n))))


def main():
    out = {}
    # Q8 linear known answers
    arrays = {}
    for i, (frames, width, rows) in enumerate(Q8_AVX_GRID):
        x, q, s, bias = q8_avx_case(frames, width, rows)
        arrays[f"case{i}"] = q8_linear_expected(x, frames, q, s, rows, width, bias)
    arrays["grid"] = np.array(Q8_AVX_GRID, np.int32)
    np.savez_compressed(HERE / "q8_linear_extremes.npz", **arrays)
    out["q8_linear_extremes"] = len(Q8_AVX_GRID)

    x = quantize_rounding_input()
    q, d = quantize_expected(x)
    np.savez_compressed(HERE / "quantize_rounding.npz", x=x, q=q, d=d)
    out["quantize_rounding"] = x.size

    x = half_rounding_input()
    y = x.astype(np.float16).astype(np.float32)
    np.savez_compressed(HERE / "half_rounding.npz", x=x, y=y)
    out["half_rounding"] = x.size

    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    np.savez_compressed(HERE / "f16_scales.npz", bits=bits, y=half_to_float_expected(bits))
    out["f16_scales"] = bits.size

    rng = np.random.default_rng(7)
    cases = {}
    for i, (width, rows) in enumerate([(1024, 3), (128, 6), (96, 2), (36, 2)]):
        xx = (rng.standard_normal(width * rows) * rng.choice([1e-3, 1.0, 30.0], width * rows)).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(width)).astype(np.float32)
        cases[f"x{i}"], cases[f"g{i}"], cases[f"w{i}"] = xx, g, np.int32(width)
        cases[f"y{i}"] = rmsnorm_expected(xx, width, g, 1e-6)
    np.savez_compressed(HERE / "rmsnorm.npz", **cases)
    out["rmsnorm"] = 4

    nan, inf = np.nan, np.inf
    gcases = [[1, 3, 3, 2], [nan, 5, 6], [1, nan, 2, nan], [-0.0, 0.0], [-inf, -inf, -1e30], [inf, 1, inf], [0.5],
              [2, 2, 2, 2, 2, 2, 2, 2, 2, 3, 3]]
    expected = []
    for c in gcases:
        a = np.array(c, np.float32)
        best = 0
        for i in range(1, a.size):
            if a[i] > a[best]:
                best = i
        expected.append(best)
    flat = np.concatenate([np.array(c, np.float32) for c in gcases])
    np.savez_compressed(HERE / "greedy.npz", flat=flat, lens=np.array([len(c) for c in gcases], np.int32),
                        expected=np.array(expected, np.int32))
    out["greedy"] = len(gcases)

    xs = np.concatenate([np.linspace(-110, 110, 4001, dtype=np.float32),
                         rng.standard_normal(4000).astype(np.float32) * 8,
                         np.array([0.0, -0.0, 1e-30, -1e-30, 88.7, -87.3, 104.0, -104.0, 200, -200], np.float32)])
    np.savez_compressed(HERE / "exp_ref.npz", x=xs, y=np.array([exp_ref(v) for v in xs], np.float32))
    out["exp_ref"] = xs.size
    print(out)


if __name__ == "__main__":
    main()
