"""Parity of every decoder kernel with the CPU oracle, through the C ABI.

All of them reproduce the reference's arithmetic order and are compared bit
for bit: quantiser, Q8 GEMV, FP32 GEMV (FloatRows4Avx order), RMSNorm,
binary16 rounding, SiLU*up and paired-GQA attention (both with the
reference's ExpAvx exp), argmax.  SiLU is also held to the reference's own
2e-6 check against double precision (tests/FunAsrNet.Checks/Program.cs:360-363).
"""
import numpy as np
import pytest

from cases import Q8_AVX_GRID, half_rounding_input, q8_avx_case, q8_weight, quantize_rounding_input
from conftest import assert_bits_equal

pytestmark = pytest.mark.gpu


def test_quantize_rounding_exact(ops, oracle):
    x = quantize_rounding_input()
    q, s = ops.quantize(x)
    eq, es = oracle.quantize(x)
    assert np.array_equal(q, eq)
    assert_bits_equal(s, es, "block scales")


def test_quantize_random_exact(ops, oracle):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(1 << 16) * rng.choice([1e-30, 1e-3, 1, 1e3, 1e30], 1 << 16)).astype(np.float32)
    q, s = ops.quantize(x)
    eq, es = oracle.quantize(x)
    assert np.array_equal(q, eq)
    assert_bits_equal(s, es, "block scales")


@pytest.mark.parametrize("frames,width,rows", Q8_AVX_GRID)
def test_q8_linear_extremes_exact(backend, oracle, frames, width, rows):
    from funasrnet_b200.backend import Weight

    x, q, s, bias = q8_avx_case(frames, width, rows)
    w = Weight("avx-extremes", (width, rows), quantized=q, scales=s)
    b = Weight("bias", (rows,), values=bias)
    out = np.full(frames * rows, 123.0, np.float32)
    assert backend.try_quantized_linear(x, frames, w, b, out)
    exp = oracle.q8_linear(x, frames, q, s, rows, width, bias)
    assert_bits_equal(out, exp, "Q8 linear with -128 weights")


@pytest.mark.parametrize("rows,cols", [(2048, 1024), (1024, 1024), (1024, 2048), (3072, 1024), (1024, 3072),
                                       (4096 + 17, 1024), (96, 8192)])
@pytest.mark.parametrize("frames", [1, 2, 5])
def test_q8_linear_model_shapes_exact(backend, oracle, rows, cols, frames):
    from funasrnet_b200.backend import Weight

    rng = np.random.default_rng(rows * 7 + cols + frames)
    q, s = q8_weight(rng, rows, cols)
    x = rng.standard_normal(frames * cols).astype(np.float32)
    w = Weight("w", (cols, rows), quantized=q, scales=s)
    out = np.empty(frames * rows, np.float32)
    assert backend.try_quantized_linear(x, frames, w, None, out)
    assert_bits_equal(out, oracle.q8_linear(x, frames, q, s, rows, cols), f"{rows}x{cols}")


def test_linear_many_matches_separate(backend, oracle):
    from funasrnet_b200.backend import Weight

    rng = np.random.default_rng(3)
    ws = []
    for rows in (2048, 1024, 1024):
        q, s = q8_weight(rng, rows, 1024)
        ws.append(Weight(f"w{rows}", (1024, rows), quantized=q, scales=s))
    x = rng.standard_normal(3 * 1024).astype(np.float32)
    ok, outs = backend.try_linear_many(x, 3, ws)
    assert ok
    for w, o in zip(ws, outs):
        assert_bits_equal(o, oracle.q8_linear(x, 3, w.quantized, w.scales, w.rows, w.columns), w.name)


def test_linear_declines_and_keeps_output(backend):
    from funasrnet_b200.backend import Weight

    rng = np.random.default_rng(4)
    q, s = q8_weight(rng, 64, 64)
    w = Weight("w", (64, 64), quantized=q, scales=s)
    out = np.full(64, 7.0, np.float32)
    assert not backend.try_quantized_linear(np.zeros(64, np.float32), 0, w, None, out)
    assert not backend.try_linear(np.zeros(64, np.float32), 1, w, None, out)  # Q8 goes to TryQuantizedLinear
    assert np.all(out == 7.0)
    with pytest.raises(ValueError):
        backend.try_quantized_linear(np.zeros(63, np.float32), 1, w, None, out)


@pytest.mark.parametrize("frames", [1, 2, 3, 4, 7, 15, 16, 33])
def test_f32_linear(backend, oracle, frames):
    """FP32 projections in the order the reference picks for the call's frame
    count (TensorMath.cs:106-176): FloatRows4Avx below 4 frames, Dot4x4 groups
    of four plus Dot for the rest up to 15, the fused-segment packed kernels
    from 16 (33 frames: two frame tiles; 1003 rows: a partial row block)."""
    from funasrnet_b200.backend import Weight

    rng = np.random.default_rng(frames)
    rows, cols = 1003, 1024
    wv = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    x = rng.standard_normal(frames * cols).astype(np.float32)
    bias = rng.standard_normal(rows).astype(np.float32)
    w = Weight("f", (cols, rows), values=wv)
    out = np.empty(frames * rows, np.float32)
    assert backend.try_linear(x, frames, w, Weight("b", (rows,), values=bias), out)
    exp = oracle.f32_linear(x, frames, wv, rows, cols, bias)
    assert_bits_equal(out, exp, f"FP32 GEMV, {frames} frames")


@pytest.mark.parametrize("width,rows", [(1024, 5), (128, 24), (96, 3), (3072, 2)])
def test_rmsnorm_exact(ops, oracle, width, rows):
    rng = np.random.default_rng(width + rows)
    x = (rng.standard_normal(width * rows) * rng.choice([1e-3, 1, 50], width * rows)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(width)).astype(np.float32)
    assert_bits_equal(ops.rmsnorm(x, width, g), oracle.rmsnorm(x, width, g), "RMSNorm")


def test_round_half_exhaustive(ops, oracle):
    x = half_rounding_input()
    assert_bits_equal(ops.round_half(x), oracle.round_half(x), "binary16 rounding")


def test_silu_mul_exact(ops, oracle):
    rng = np.random.default_rng(9)
    g = (rng.standard_normal(3072 * 4) * 4).astype(np.float32)
    u = rng.standard_normal(g.size).astype(np.float32)
    got, exp = ops.silu_mul(g, u), oracle.silu_mul(g, u)
    ref = g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64))) * u
    assert np.all(np.abs(got - ref) <= 2e-6 * np.maximum(1, np.abs(ref)))
    assert_bits_equal(got, exp, "SiLU*up")


def test_greedy_edge_cases(ops, oracle):
    nan, inf = np.float32(np.nan), np.float32(np.inf)
    cases = [
        [1, 3, 3, 2],                 # ties keep the first index
        [nan, 5, 6],                  # NaN first -> 0
        [1, nan, 2, nan],             # NaN elsewhere never wins
        [-0.0, 0.0],                  # -0 == +0 keeps index 0
        [-inf, -inf, -1e30],
        [inf, 1, inf],
        [0.5],
    ]
    rng = np.random.default_rng(1)
    big = rng.standard_normal(151936).astype(np.float32)
    big[[77, 150000]] = big.max() + 1
    cases.append(big.tolist())
    for c in cases:
        a = np.array(c, np.float32)
        assert ops.greedy(a) == oracle.greedy(a), c


@pytest.mark.parametrize("frames", [1, 3, 4, 17, 73, 129])
@pytest.mark.parametrize("kv_heads", [1, 3, 8])
def test_attention_pair(ops, oracle, frames, kv_heads):
    rng = np.random.default_rng(frames * 10 + kv_heads)
    size = 128
    stride = kv_heads * size
    q = (rng.random(2 * stride) - 0.5).astype(np.float32)
    k = oracle.round_half((rng.random(stride * (frames + 3)) - 0.5).astype(np.float32))
    v = oracle.round_half((rng.random(stride * (frames + 3)) - 0.5).astype(np.float32))
    ok, got = ops.attention_pair(q, k, v, frames, kv_heads, size)
    assert ok
    exp = oracle.attention_pair(q, k, v, frames, kv_heads, size)
    assert_bits_equal(got, exp, "paired GQA attention")


def test_attention_pair_declines_other_sizes(ops):
    q = np.zeros(2 * 3 * 65, np.float32)
    out = np.full(q.size, 123.0, np.float32)
    ok, out = ops.attention_pair(q, np.zeros(65 * 3 * 4, np.float32), np.zeros(65 * 3 * 4, np.float32), 4, 3, 65, out)
    assert not ok and np.all(out == 123.0)
