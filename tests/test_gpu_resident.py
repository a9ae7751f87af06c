"""Resident serving (fa_session_set_resident): fa_session_step posts each token
to one persistent launch that stays running between calls.  Its tokens and
the session state it leaves are bit-identical to the per-call persistent
launch, which the other persistent-kernel tests pin to the oracle."""
import time

import numpy as np
import pytest

from conftest import assert_bits_equal
from test_gpu_decoder import prefix_embeddings

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small(backend, oracle, small_gguf):
    from funasrnet_b200.decoder import CudaModel

    cm = CudaModel(backend, small_gguf, capacity=512)
    om = oracle.Model(small_gguf, 512)
    yield cm, om
    cm.close()
    om.close()


def _pair(cm, om, prefix, seed):
    from funasrnet_b200.decoder import QwenDecoder

    emb, frames = prefix_embeddings(om, prefix, 8, seed=seed)
    a, b = QwenDecoder(cm), QwenDecoder(cm)
    _, ta = a.decode(emb, frames)
    _, tb = b.decode(emb, frames)
    assert ta == tb
    assert b.set_resident(True)
    return a, b, ta


def test_resident_steps_match_per_call_steps(small):
    cm, om = small
    a, b, tok = _pair(cm, om, 30, 41)
    with a, b:
        ta = tb = tok
        for i in range(24):
            ta, _ = a.step(ta)
            tb, _ = b.step(tb)
            assert ta == tb, f"step {i}"
        assert a.position == b.position
        # reading the cache stops the resident launch first: identical state
        for layer in (0, cm.layers - 1):
            ka, va = a.kv(layer)
            kb, vb = b.kv(layer)
            assert_bits_equal(kb, ka, f"layer-{layer} keys")
            assert_bits_equal(vb, va, f"layer-{layer} values")
        # a step with logits runs the per-call launch; then resident again
        na, la = a.step(ta, want_logits=True)
        nb, lb = b.step(tb, want_logits=True)
        assert na == nb
        assert_bits_equal(lb, la, "logits after the resident launch stopped")
        for i in range(8):
            na, _ = a.step(na)
            nb, _ = b.step(nb)
            assert na == nb, f"step {i} after restart"


def test_resident_teacher_forced_tokens(small):
    """Tokens the host chooses (not the argmax) are decoded as posted."""
    cm, om = small
    a, b, _ = _pair(cm, om, 17, 42)
    rng = np.random.default_rng(5)
    with a, b:
        for t in rng.integers(0, cm.vocab, 20):
            na, _ = a.step(int(t))
            nb, _ = b.step(int(t))
            assert na == nb


def test_resident_relaunch_after_idle_limit(small):
    """A launch that waited longer than its idle limit has ended; the next step
    starts a new one and the results do not change."""
    cm, om = small
    a, b, tok = _pair(cm, om, 25, 43)
    with a, b:
        assert b.set_resident(True, idle_us=300)
        ta = tb = tok
        for i in range(12):
            ta, _ = a.step(ta)
            tb, _ = b.step(tb)
            assert ta == tb, f"step {i}"
            if i % 3 == 2:
                time.sleep(0.01)  # beyond the idle limit
        assert a.position == b.position


def test_other_session_runs_while_one_is_resident(small):
    """Another session's launch waits for the resident launch's idle limit, then
    runs; the resident session relaunches at its next step."""
    from funasrnet_b200.decoder import QwenDecoder

    cm, om = small
    a, b, tok = _pair(cm, om, 21, 44)
    emb, frames = prefix_embeddings(om, 21, 8, seed=44)
    with a, b, QwenDecoder(cm) as c:
        assert b.set_resident(True, idle_us=2000)
        _, tc = c.decode(emb, frames)
        ta = tb = tok
        for i in range(6):
            ta, _ = a.step(ta)
            tb, _ = b.step(tb)
            tc, _ = c.step(tc)
            assert ta == tb == tc, f"step {i}"
        toks_a = a.generate(10, end_ids=())
        toks_b = b.generate(10, end_ids=())  # stops the resident launch first
        assert toks_a == toks_b


def test_batch_ends_a_members_resident_launch(small):
    """A batch call stops a member's resident launch first; the batch's tokens
    equal the per-session tokens, and the member then steps resident again."""
    from funasrnet_b200.decoder import BatchDecoder

    cm, om = small
    a, b, tok = _pair(cm, om, 23, 45)
    with a, b:
        ta = tb = tok
        for i in range(5):
            ta, _ = a.step(ta)
            tb, _ = b.step(tb)
            assert ta == tb, f"step {i}"
        ga = a.generate(6, end_ids=())
        with BatchDecoder([b]) as g:
            gb = g.generate(6)[:, 0].tolist()
        assert ga == gb
        na, nb = ga[-1], gb[-1]
        for i in range(4):
            na, _ = a.step(na)
            nb, _ = b.step(nb)
            assert na == nb, f"step {i} after the batch"
