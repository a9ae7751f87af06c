"""The persistent decode kernel (one cooperative launch per generate/step call)
against the CPU oracle and against the CUDA-graph step path: bit-identical
logits and tokens."""
import numpy as np
import pytest

from conftest import assert_bits_equal
from test_gpu_decoder import check_logits, prefix_embeddings

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small(backend, oracle, small_gguf):
    from funasrnet_b200.decoder import CudaModel

    cm = CudaModel(backend, small_gguf, capacity=512)
    om = oracle.Model(small_gguf, 512)
    yield cm, om
    cm.close()
    om.close()


def test_persistent_kernel_is_used(small):
    from funasrnet_b200.decoder import QwenDecoder

    cm, _ = small
    with QwenDecoder(cm) as d:
        assert d.persistent_grid() >= 32


def test_step_matches_oracle_bit_for_bit(small, oracle):
    from funasrnet_b200.decoder import QwenDecoder

    cm, om = small
    emb, frames = prefix_embeddings(om, 11, 8, seed=31)
    with QwenDecoder(cm) as d:
        os_ = oracle.Session(om)
        _, arg = d.decode(emb, frames)
        exp = os_.decode(emb, frames)
        tok = oracle.greedy(exp)
        assert arg == tok
        for i in range(16):
            nxt, lg = d.step(tok, want_logits=True)
            exp = os_.decode(om.embed([tok]), 1)
            check_logits(lg, exp, f"persistent step {i}")
            assert nxt == oracle.greedy(exp)
            tok = nxt
        k, v = d.kv(1)
        ek, ev = os_.kv(1)
        assert_bits_equal(k, ek, "layer-1 keys")
        assert_bits_equal(v, ev, "layer-1 values")
        os_.close()


def test_generate_matches_graph_path(small):
    from funasrnet_b200.decoder import QwenDecoder

    cm, om = small
    emb, frames = prefix_embeddings(om, 40, 8, seed=32)
    with QwenDecoder(cm) as a, QwenDecoder(cm) as b:
        assert b.set_persistent(False)
        for d in (a, b):
            d.decode(emb, frames, want_logits=False)
        ta = a.generate(48, end_ids=())
        tb = b.generate(48, end_ids=())
        assert ta == tb and len(ta) == 48
        assert a.position == b.position == frames + 48
        # continue both with a host-driven step: identical state
        na, la = a.step(ta[-1], want_logits=True)
        nb, lb = b.step(tb[-1], want_logits=True)
        assert na == nb
        assert_bits_equal(la, lb, "persistent vs graph step logits")


def test_generate_in_pieces_equals_one_launch(small):
    from funasrnet_b200.decoder import QwenDecoder

    cm, om = small
    emb, frames = prefix_embeddings(om, 20, 8, seed=33)
    with QwenDecoder(cm) as a, QwenDecoder(cm) as b:
        a.decode(emb, frames, want_logits=False)
        b.decode(emb, frames, want_logits=False)
        one = a.generate(30, end_ids=())
        pieces = b.generate(7, end_ids=()) + b.generate(1, end_ids=()) + b.generate(22, end_ids=())
        assert one == pieces


def test_generate_stops_before_end_token(small):
    from funasrnet_b200.decoder import QwenDecoder

    cm, om = small
    emb, frames = prefix_embeddings(om, 12, 8, seed=34)
    with QwenDecoder(cm) as d:
        d.decode(emb, frames, want_logits=False)
        full = d.generate(16, end_ids=())
        d.reset()
        d.decode(emb, frames, want_logits=False)
        cut = d.generate(16, end_ids=(full[9],))
        assert cut == full[:full.index(full[9])]
        assert d.position == frames + len(cut)


def test_reset_and_reuse(small):
    from funasrnet_b200.decoder import QwenDecoder

    cm, om = small
    emb, frames = prefix_embeddings(om, 9, 8, seed=35)
    with QwenDecoder(cm) as d:
        runs = []
        for _ in range(3):
            d.reset()
            d.decode(emb, frames, want_logits=False)
            runs.append(d.generate(12, end_ids=()))
        assert runs[0] == runs[1] == runs[2]


def test_bounded_wait_gives_up_and_session_recovers(small):
    """The failure path of the persistent kernel's bounded waits, without a GPU
    fault: one GEMV CTA leaves its first q/k/v rows unpublished and the wait
    limit is short, so the attention CTAs' waits run out.  The call returns
    FA_ERR_TIMEOUT naming the wait, the kernel has returned (the context stays
    usable), the session keeps its position, and the next calls on it give the
    same tokens and bit-identical logits as a session that never failed."""
    from funasrnet_b200._lib import FaError
    from funasrnet_b200.decoder import QwenDecoder

    cm, om = small
    emb, frames = prefix_embeddings(om, 30, 8, seed=61)
    with QwenDecoder(cm) as d, QwenDecoder(cm) as ref:
        grid = d.persistent_grid()
        d.decode(emb, frames, want_logits=False)
        ref.decode(emb, frames, want_logits=False)
        d.set_fault_test(wait_limit=100000, withhold_cta=grid - 1)
        with pytest.raises(FaError) as err:
            d.generate(3, end_ids=())
        assert err.value.code == -6  # FA_ERR_TIMEOUT
        assert "bounded wait gave up" in str(err.value)
        assert d.position == frames
        # the hooks held for one launch: the same session decodes normally again
        assert d.generate(6, end_ids=()) == ref.generate(6, end_ids=())
        assert d.position == ref.position
        nxt, lg = d.step(7, want_logits=True)
        nref, lref = ref.step(7, want_logits=True)
        assert nxt == nref
        assert_bits_equal(lg, lref, "after recovery")
        # and after a reset it matches a fresh decode bit for bit
        d.reset()
        ref.reset()
        la, _ = d.decode(emb, frames)
        lb, _ = ref.decode(emb, frames)
        assert_bits_equal(la, lb, "fresh decode after the failure")


def test_fault_test_hook_rejects_attention_ctas(small):
    from funasrnet_b200._lib import FaError
    from funasrnet_b200.decoder import QwenDecoder

    cm, _ = small
    with QwenDecoder(cm) as d:
        with pytest.raises(FaError):
            d.set_fault_test(withhold_cta=3)
        with pytest.raises(FaError):
            d.set_fault_test(withhold_cta=d.persistent_grid())


def test_persistent_kernel_at_large_capacity(backend, small, small_gguf):
    """At a cache capacity of 4,096 positions (a 16 KB score row per attention
    CTA on top of the GEMV staging) the persistent kernel still launches, and
    its tokens and logits equal the CUDA-graph path's."""
    from funasrnet_b200.decoder import CudaModel, QwenDecoder

    _, om = small
    cm = CudaModel(backend, small_gguf, capacity=4096)
    try:
        emb, frames = prefix_embeddings(om, 30, 8, seed=35)
        with QwenDecoder(cm) as a, QwenDecoder(cm) as b:
            assert a.persistent_grid() > 0
            assert b.set_persistent(False)
            for d in (a, b):
                d.decode(emb, frames, want_logits=False)
            ta = a.generate(12, end_ids=())
            tb = b.generate(12, end_ids=())
            assert ta == tb
            na, la = a.step(ta[-1], want_logits=True)
            nb, lb = b.step(tb[-1], want_logits=True)
            assert na == nb
            assert_bits_equal(la, lb, "persistent vs graph step logits at capacity 4096")
    finally:
        cm.close()
