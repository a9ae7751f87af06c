"""Full-size Qwen3-0.6B (28 layers, vocab 151936) parity with the oracle on the
benchmark configs' shapes: config 1's 100+8-frame prefix, config 2's 400+8
prefix with decode steps at positions 408..420 and 650..664, config 3's FP32
weights, and a ragged batch of 16 sessions (prefixes U[50, 400] + 8) stepped
together.  Logits are compared bit for bit and against the north-star
tolerance (2e-2 absolute + 1e-3 relative; argmax equal where the top-2 margin
exceeds 1e-2)."""
import numpy as np
import pytest

from test_gpu_decoder import check_logits, prefix_embeddings

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def full_gguf(tmp_path_factory, built_lib):
    from funasrnet_b200._lib import check, lib

    p = tmp_path_factory.mktemp("full") / "qwen3_0p6b_q8_seed1234.gguf"
    check(lib().fa_synth_write_gguf(str(p).encode(), 1234, 0, 0, 0, 0, 1))
    return p


@pytest.fixture(scope="module")
def full_gguf_f32(tmp_path_factory, built_lib):
    from funasrnet_b200._lib import check, lib

    p = tmp_path_factory.mktemp("full") / "qwen3_0p6b_f32_seed1234.gguf"
    check(lib().fa_synth_write_gguf(str(p).encode(), 1234, 0, 0, 0, 0, 0))
    yield p
    p.unlink()


def teacher_forced(d, os_, om, tok, steps, what):
    """`steps` decode steps on both sides, each fed the oracle's greedy token."""
    errs = []
    for i in range(steps):
        nxt, lg = d.step(tok, want_logits=True)
        exp = os_.decode(om.embed([tok]), 1)
        errs.append(check_logits(lg, exp, f"{what} step {i}"))
        tok = oracle_greedy(exp)
        assert nxt == tok, f"{what} step {i}: token {nxt} vs {tok}"
    return errs, tok


def oracle_greedy(logits):
    from oracle import oracle as O

    return O.greedy(logits)


def test_full_model_prefill_and_steps(backend, oracle, full_gguf):
    from funasrnet_b200.decoder import CudaModel, QwenDecoder

    with CudaModel(backend, full_gguf, capacity=512) as cm:
        om = oracle.Model(full_gguf, 512)
        assert (cm.layers, cm.vocab, cm.width, cm.ffn) == (28, 151936, 1024, 3072)
        emb, frames = prefix_embeddings(om, 100, 8, seed=21)
        with QwenDecoder(cm) as d:
            os_ = oracle.Session(om)
            lg, arg = d.decode(emb, frames)
            exp = os_.decode(emb, frames)
            errs = [check_logits(lg, exp, "prefill")]
            tok = oracle.greedy(exp)
            for i in range(12):
                nxt, lg = d.step(tok, want_logits=True)
                exp = os_.decode(om.embed([tok]), 1)
                errs.append(check_logits(lg, exp, f"step {i}"))
                tok = oracle.greedy(exp)
            print("max |logit error| per step:", " ".join(f"{e:.2e}" for e in errs))
            os_.close()
        om.close()


def test_full_model_batch_matches_single_sessions(backend, oracle, full_gguf):
    """The batched path on the full model: 5 ragged sessions stepped together give
    each session's own persistent-kernel logits and tokens bit for bit (those are
    pinned to the oracle above), including the tensor-core prefill."""
    from conftest import assert_bits_equal
    from funasrnet_b200.decoder import BatchDecoder, CudaModel, QwenDecoder

    with CudaModel(backend, full_gguf, capacity=512) as cm:
        om = oracle.Model(full_gguf, 512)
        lengths = [100, 3, 57, 250, 18]
        prefixes = [prefix_embeddings(om, a, 8, seed=300 + i) for i, a in enumerate(lengths)]
        batch_sessions = [QwenDecoder(cm) for _ in lengths]
        solo_sessions = [QwenDecoder(cm) for _ in lengths]
        try:
            toks = []
            for d, s, (emb, frames) in zip(batch_sessions, solo_sessions, prefixes):
                la, a = d.decode(emb, frames)
                lb, b = s.decode(emb, frames)
                assert_bits_equal(la, lb, "prefill")
                toks.append(a)
            with BatchDecoder(batch_sessions) as b:
                for step in range(4):
                    nxt, lg = b.step(want_logits=True)
                    for i, s in enumerate(solo_sessions):
                        tok, ls = s.step(toks[i], want_logits=True)
                        assert_bits_equal(lg[i], ls, f"session {i} step {step}")
                        assert int(nxt[i]) == tok
                        toks[i] = tok
        finally:
            for d in batch_sessions + solo_sessions:
                d.close()
        om.close()


def test_config2_positions_408_to_664(backend, oracle, full_gguf):
    """Config 2 (the benchmark's headline workload): the 400+8-frame prefix,
    steps at positions 408..420, then a 650-frame prefix (the same 408 frames
    followed by 242 further embeddings) and steps at positions 650..664, the
    end of config 2's 256-token decode."""
    from funasrnet_b200.decoder import CudaModel, QwenDecoder

    with CudaModel(backend, full_gguf, capacity=2048) as cm:
        om = oracle.Model(full_gguf, 2048)
        emb, frames = prefix_embeddings(om, 400, 8, seed=1234)
        more = np.random.default_rng(77).standard_normal(242 * om.width).astype(np.float32) * np.float32(0.05)
        for name, e, n, steps in (("prefix 408", emb, frames, 12), ("prefix 650", np.concatenate([emb, more]), 650, 14)):
            with QwenDecoder(cm) as d:
                assert d.persistent_grid() > 0
                os_ = oracle.Session(om)
                lg, arg = d.decode(e, n)
                exp = os_.decode(e, n)
                errs = [check_logits(lg, exp, f"{name} prefill")]
                tok = oracle.greedy(exp)
                assert arg == tok
                more_errs, _ = teacher_forced(d, os_, om, tok, steps, name)
                assert d.position == n + steps
                print(name, "max |logit error| per step:", " ".join(f"{x:.2e}" for x in errs + more_errs))
                os_.close()
        om.close()


def test_config3_fp32_full_model(backend, oracle, full_gguf_f32):
    """Config 3: FP32 (unquantised) weights at full size, 100+8-frame prefix and
    8 teacher-forced steps (the CUDA-graph step with the FP32 GEMV)."""
    from funasrnet_b200.decoder import CudaModel, QwenDecoder

    with CudaModel(backend, full_gguf_f32, capacity=512) as cm:
        om = oracle.Model(full_gguf_f32, 512)
        assert (cm.layers, cm.vocab, om.quantized) == (28, 151936, 0)
        emb, frames = prefix_embeddings(om, 100, 8, seed=23)
        with QwenDecoder(cm) as d:
            os_ = oracle.Session(om)
            lg, arg = d.decode(emb, frames)
            exp = os_.decode(emb, frames)
            errs = [check_logits(lg, exp, "fp32 prefill")]
            more, _ = teacher_forced(d, os_, om, oracle.greedy(exp), 8, "fp32")
            print("fp32 max |logit error| per step:", " ".join(f"{x:.2e}" for x in errs + more))
            os_.close()
        om.close()


def test_ragged_batch_of_16_against_oracle(backend, oracle, full_gguf):
    """Config 4's shape at 16 sessions: prefixes U[50, 400] audio vectors + 8
    prompt ids, prefilled one by one, then two batched steps (tcgen05
    projections, per-session attention) compared with the oracle decoding each
    session alone."""
    from funasrnet_b200.decoder import BatchDecoder, CudaModel, QwenDecoder

    rng = np.random.default_rng(404)
    lengths = [int(a) for a in rng.integers(50, 401, 16)]
    with CudaModel(backend, full_gguf, capacity=512) as cm:
        om = oracle.Model(full_gguf, 512)
        sessions = [QwenDecoder(cm) for _ in lengths]
        refs = [oracle.Session(om) for _ in lengths]
        try:
            toks = []
            for i, (d, r, a) in enumerate(zip(sessions, refs, lengths)):
                emb, frames = prefix_embeddings(om, a, 8, seed=500 + i)
                _, arg = d.decode(emb, frames, want_logits=False)
                exp = r.decode(emb, frames)
                toks.append(oracle.greedy(exp))
                assert arg == toks[-1], f"session {i} prefill argmax"
            with BatchDecoder(sessions) as b:
                for step in range(2):
                    nxt, lg = b.step(want_logits=True)
                    for i, r in enumerate(refs):
                        exp = r.decode(om.embed([toks[i]]), 1)
                        check_logits(lg[i], exp, f"session {i} (prefix {lengths[i] + 8}) step {step}")
                        toks[i] = oracle.greedy(exp)
                        assert int(nxt[i]) == toks[i]
        finally:
            for d in sessions:
                d.close()
            for r in refs:
                r.close()
        om.close()
