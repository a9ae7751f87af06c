"""Full-size Qwen3-0.6B Q8_0 (28 layers, vocab 151936) parity with the oracle:
the BASELINE configs' decoder at its real size, a 100+8-frame prefix and
teacher-forced greedy steps, logits within the north-star tolerance."""
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
