"""fa_lm_head_argmax_noalloc: RMSNorm + Q8 projection + greedy argmax of one
frame on caller-owned device memory, with the argmax scratch in module memory.

Each case makes two calls in a row and compares both with the existing entry
points (fa_op_rmsnorm, fa_try_quantized_linear, fa_op_greedy).  Both routes
sum the block products in the reference's order, so the tolerance is exact
bits.  The file runs last so that it also sees the state the earlier GPU tests
leave behind."""
import numpy as np
import pytest

from conftest import assert_bits_equal

pytestmark = pytest.mark.gpu

MAX_ROWS = 262144  # FA_NOALLOC_MAX_ROWS


def q8_weight(name, rows, cols, seed, f16_scales=True):
    from funasrnet_b200.backend import Weight

    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
    s = rng.uniform(1e-4, 3e-3, size=(rows, cols // 32)).astype(np.float32)
    if f16_scales:
        s = s.astype(np.float16).astype(np.float32)
    else:
        s[0, 0] = np.float32(1.0e-9)  # below binary16's range: the f32-scale layout
    return Weight(name, (cols, rows), quantized=q, scales=s)


def existing_route(backend, ops, w, x, gamma):
    y = ops.rmsnorm(x, w.columns, gamma) if gamma is not None else x
    out = np.empty(w.rows, np.float32)
    assert backend.try_quantized_linear(y, 1, w, None, out)
    return out, ops.greedy(out)


def noalloc_route(backend, w, x, gamma, eps=1e-6):
    import torch

    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(x).to(dev)
    gd = torch.from_numpy(gamma).to(dev) if gamma is not None else None
    logits = torch.full((w.rows,), float("nan"), dtype=torch.float32, device=dev)
    token = torch.full((1,), -7, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    ok = backend.lm_head_argmax_noalloc(w, xd.data_ptr(), gd.data_ptr() if gd is not None else None, eps,
                                        logits.data_ptr(), token.data_ptr(), stream)
    torch.cuda.synchronize(dev)
    return ok, logits.cpu().numpy(), int(token.cpu().item())


@pytest.mark.parametrize("f16_scales", [True, False])
def test_two_calls_match_existing_entry_points(backend, ops, f16_scales):
    w = q8_weight("lm_head", 5000, 1024, seed=71, f16_scales=f16_scales)  # 625 tiles: a ragged last CTA
    backend.make_resident(w)
    rng = np.random.default_rng(72)
    gamma = rng.uniform(0.5, 1.5, 1024).astype(np.float32)
    inputs = [(rng.normal(0, 1, 1024).astype(np.float32), gamma),
              (rng.normal(0, 2, 1024).astype(np.float32), None)]
    for i, (x, g) in enumerate(inputs):
        ok, logits, token = noalloc_route(backend, w, x, g)
        assert ok
        exp_logits, exp_token = existing_route(backend, ops, w, x, g)
        assert_bits_equal(logits, exp_logits, f"call {i} logits")
        assert token == exp_token, f"call {i}"


def test_no_device_memory_taken_after_setup(backend):
    import torch

    w = q8_weight("lm_head_mem", 4096, 1024, seed=73)
    backend.make_resident(w)
    x = np.random.default_rng(74).normal(0, 1, 1024).astype(np.float32)
    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(x).to(dev)
    token = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    tokens, free = [], []
    for _ in range(2):
        assert backend.lm_head_argmax_noalloc(w, xd.data_ptr(), None, 1e-6, None, token.data_ptr(), stream)
        torch.cuda.synchronize(dev)
        tokens.append(int(token.item()))
        free.append(torch.cuda.mem_get_info(dev)[0])
    assert tokens[0] == tokens[1]
    assert free[1] == free[0]


def test_first_index_wins_a_tie(backend, ops):
    w = q8_weight("lm_head_tie", 4104, 1024, seed=75)
    w.quantized[4100] = 127
    w.scales[4100] = np.float32(np.float16(2e-3))
    w.quantized[301] = w.quantized[4100]
    w.scales[301] = w.scales[4100]
    backend.make_resident(w)
    x = np.abs(np.random.default_rng(76).normal(0, 1, 1024)).astype(np.float32)
    for _ in range(2):
        ok, logits, token = noalloc_route(backend, w, x, None)
        assert ok and token == 301
        exp_logits, exp_token = existing_route(backend, ops, w, x, None)
        assert_bits_equal(logits, exp_logits, "tie logits")
        assert exp_token == 301


def test_largest_row_count_and_one_tile_beyond(backend, ops):
    from funasrnet_b200._lib import FaError

    w = q8_weight("lm_head_max", MAX_ROWS, 32, seed=77)
    backend.make_resident(w)
    x = np.random.default_rng(78).normal(0, 1, 32).astype(np.float32)
    for _ in range(2):
        ok, logits, token = noalloc_route(backend, w, x, None)
        assert ok
        exp_logits, exp_token = existing_route(backend, ops, w, x, None)
        assert_bits_equal(logits, exp_logits, "largest size logits")
        assert token == exp_token
    over = q8_weight("lm_head_over", MAX_ROWS + 8, 32, seed=79)
    backend.make_resident(over)
    with pytest.raises(FaError) as e:
        noalloc_route(backend, over, x, None)
    assert e.value.code == -2


def test_fp32_weight_is_declined(backend):
    import torch

    from funasrnet_b200.backend import Weight

    w = Weight("lm_head_f32", (64, 16), values=np.ones((16, 64), np.float32))
    backend.make_resident(w)
    dev = torch.device("cuda", 0)
    xd = torch.ones(64, dtype=torch.float32, device=dev)
    token = torch.full((1,), -7, dtype=torch.int32, device=dev)
    assert not backend.lm_head_argmax_noalloc(w, xd.data_ptr(), None, 1e-6, None, token.data_ptr(), None)
    torch.cuda.synchronize(dev)
    assert int(token.item()) == -7


def test_weight_must_be_resident(backend):
    w = q8_weight("lm_head_cold", 64, 32, seed=80)
    with pytest.raises(ValueError):
        backend.lm_head_argmax_noalloc(w, 0, None, 1e-6, None, 0, None)
