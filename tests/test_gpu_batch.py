"""Batched decode (fa_batch_*) and the tensor-core multi-frame projections
behind it, against the CPU oracle through the C ABI.

The tensor-core path keeps the reference's arithmetic (one K = 32 int8 MMA per
Q8 block, then ((float)dot * ws) * xs summed in block order), so projections,
prefill logits and every session's batched logits are compared bit for bit,
and a batch's greedy tokens must equal each session decoding alone.
"""
import contextlib

import numpy as np
import pytest

from cases import q8_avx_case, q8_weight
from conftest import assert_bits_equal
from test_gpu_decoder import check_logits, prefix_embeddings

pytestmark = pytest.mark.gpu


# ------------------------------------------------ multi-frame projections ----

@pytest.mark.parametrize("rows,cols", [(128, 256), (4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072)])
@pytest.mark.parametrize("frames", [16, 17, 64, 129, 300])
def test_tensor_core_linear_exact(backend, oracle, rows, cols, frames):
    from funasrnet_b200.backend import Weight

    rng = np.random.default_rng(rows + 3 * cols + frames)
    q, s = q8_weight(rng, rows, cols)
    x = (rng.standard_normal(frames * cols) * rng.choice([1e-3, 1.0, 50.0], frames * cols)).astype(np.float32)
    bias = rng.standard_normal(rows).astype(np.float32)
    w = Weight("w", (cols, rows), quantized=q, scales=s)
    out = np.full(frames * rows, 7.0, np.float32)
    assert backend.try_quantized_linear(x, frames, w, Weight("b", (rows,), values=bias), out)
    assert_bits_equal(out, oracle.q8_linear(x, frames, q, s, rows, cols, bias), f"{rows}x{cols}x{frames}")


@pytest.mark.parametrize("frames", [16, 40])
def test_tensor_core_linear_extremes_f32_scales(backend, oracle, frames):
    """QuantizedAvxChecks' pattern (-128 weights, f32 scales that binary16
    cannot hold) at a shape the tensor-core path takes."""
    from funasrnet_b200.backend import Weight

    x, q, s, bias = q8_avx_case(frames, 1024, 256)
    w = Weight("avx-extremes", (1024, 256), quantized=q, scales=s)
    out = np.empty(frames * 256, np.float32)
    assert backend.try_quantized_linear(x, frames, w, Weight("b", (256,), values=bias), out)
    assert_bits_equal(out, oracle.q8_linear(x, frames, q, s, 256, 1024, bias), "extremes")


def test_tensor_core_linear_non_finite(backend, oracle):
    """Infinite / NaN weight scales and activation blocks follow the
    reference's IEEE arithmetic (inf * 0 = NaN, NaN propagates)."""
    from funasrnet_b200.backend import Weight

    rows, cols, frames = 256, 512, 20
    rng = np.random.default_rng(9)
    q, s = q8_weight(rng, rows, cols)
    s[3, 2] = np.inf
    s[7, 0] = -np.inf
    s[130, 5] = np.nan
    q[3, 64:96] = 0  # inf scale over an all-zero block: 0 * inf = NaN
    x = rng.standard_normal(frames * cols).astype(np.float32)
    x[5 * cols + 40] = np.inf
    x[9 * cols + 300] = np.nan
    w = Weight("w", (cols, rows), quantized=q, scales=s)
    out = np.empty(frames * rows, np.float32)
    assert backend.try_quantized_linear(x, frames, w, None, out)
    assert_bits_equal(out, oracle.q8_linear(x, frames, q, s, rows, cols), "non-finite")


# ------------------------------------------------------- batched decode ----

@pytest.fixture(scope="module")
def small(backend, oracle, small_gguf):
    from funasrnet_b200.decoder import CudaModel

    cm = CudaModel(backend, small_gguf, capacity=512)
    om = oracle.Model(small_gguf, 512)
    yield cm, om
    cm.close()
    om.close()


@contextlib.contextmanager
def prefilled(cm, om, oracle, audio_lengths, seed, with_oracle=True):
    """Sessions (and oracle twins) prefilled with ragged prefixes; yields
    (decoders, oracle sessions or None, each session's first greedy token)."""
    from funasrnet_b200.decoder import QwenDecoder

    decs, oss, first = [], [], []
    try:
        for i, audio in enumerate(audio_lengths):
            emb, frames = prefix_embeddings(om, audio, 8, seed=seed + i)
            d = QwenDecoder(cm)
            decs.append(d)
            _, arg = d.decode(emb, frames, want_logits=False)
            first.append(arg)
            if with_oracle:
                o = oracle.Session(om)
                oss.append(o)
                assert arg == oracle.greedy(o.decode(emb, frames)), f"prefill argmax of session {i}"
        yield decs, (oss if with_oracle else None), first
    finally:
        for o in oss:
            o.close()
        for d in decs:
            d.close()


def test_prefill_on_tensor_cores_exact(small, oracle):
    """A 77-frame prefill: chunks of 64 and 13 frames, the first on the tensor cores."""
    from funasrnet_b200.decoder import QwenDecoder

    cm, om = small
    emb, frames = prefix_embeddings(om, 69, 8, seed=41)
    with QwenDecoder(cm) as d:
        o = oracle.Session(om)
        lg, arg = d.decode(emb, frames)
        exp = o.decode(emb, frames)
        check_logits(lg, exp, "77-frame prefill")
        assert arg == oracle.greedy(exp)
        for layer in range(2):
            k, v = d.kv(layer)
            ek, ev = o.kv(layer)
            assert_bits_equal(k, ek, f"layer-{layer} keys")
            assert_bits_equal(v, ev, f"layer-{layer} values")
        o.close()


def test_batch_step_matches_oracle(small, oracle):
    from funasrnet_b200.decoder import BatchDecoder

    cm, om = small
    with prefilled(cm, om, oracle, [5, 40, 17, 0, 60], seed=50) as (decs, oss, toks):
        with BatchDecoder(decs) as b:
            for step in range(5):
                nxt, lg = b.step(want_logits=True)
                for i, o in enumerate(oss):
                    exp = o.decode(om.embed([toks[i]]), 1)
                    check_logits(lg[i], exp, f"session {i} step {step}")
                    assert nxt[i] == oracle.greedy(exp)
                    toks[i] = int(nxt[i])
        for d, o in zip(decs, oss):
            assert d.position == o.position
            k, v = d.kv(1)
            ek, ev = o.kv(1)
            assert_bits_equal(k, ek, "layer-1 keys")
            assert_bits_equal(v, ev, "layer-1 values")


def test_batch_host_tokens(small, oracle):
    """step(tokens) feeds given tokens instead of the sessions' argmaxes."""
    from funasrnet_b200.decoder import BatchDecoder

    cm, om = small
    with prefilled(cm, om, oracle, [3, 9, 30], seed=60) as (decs, oss, _):
        feed = np.array([11, 4095, 0], np.int32)
        with BatchDecoder(decs) as b:
            nxt, lg = b.step(feed, want_logits=True)
        for i, o in enumerate(oss):
            exp = o.decode(om.embed([int(feed[i])]), 1)
            check_logits(lg[i], exp, f"session {i}")
            assert nxt[i] == oracle.greedy(exp)


def test_batch_generate_equals_single_sessions(small, oracle):
    """Each session's batched greedy tokens equal its own generate()."""
    from funasrnet_b200.decoder import BatchDecoder

    cm, om = small
    lengths = [12, 1, 33, 7, 50, 20, 2]
    with prefilled(cm, om, oracle, lengths, seed=70, with_oracle=False) as (a, _, _):
        with BatchDecoder(a) as b:
            got = b.generate(24)
        with prefilled(cm, om, oracle, lengths, seed=70, with_oracle=False) as (s, _, _):
            for i, d in enumerate(s):
                alone = d.generate(24, end_ids=())
                assert got[:, i].tolist() == alone, f"session {i}"
                assert a[i].position == d.position


@pytest.mark.parametrize("n", [1, 16, 33, 128, 256])
def test_batch_sizes(small, oracle, n):
    """Frame tiles of 16, 32 and 64 sessions and padded batches."""
    from funasrnet_b200.decoder import BatchDecoder

    cm, om = small
    rng = np.random.default_rng(n)
    lengths = rng.integers(0, 24, n).tolist()
    with prefilled(cm, om, oracle, lengths, seed=1000 + n, with_oracle=False) as (decs, _, toks):
        check = sorted(set([0, n - 1, n // 2, n // 3]))
        oss = []
        try:
            for i in check:
                o = oracle.Session(om)
                emb, frames = prefix_embeddings(om, lengths[i], 8, seed=1000 + n + i)
                o.decode(emb, frames)
                oss.append(o)
            with BatchDecoder(decs) as b:
                for step in range(2):
                    nxt, lg = b.step(want_logits=True)
                    for i, o in zip(check, oss):
                        exp = o.decode(om.embed([toks[i]]), 1)
                        check_logits(lg[i], exp, f"n={n} session {i} step {step}")
                        assert nxt[i] == oracle.greedy(exp)
                    toks = [int(t) for t in nxt]
        finally:
            for o in oss:
                o.close()


def test_session_continues_alone_after_batch(small, oracle):
    """After a batched step a session steps on its own (persistent kernel) from
    the position and token the batch left."""
    from funasrnet_b200.decoder import BatchDecoder

    cm, om = small
    with prefilled(cm, om, oracle, [4, 25], seed=80) as (decs, oss, toks):
        with BatchDecoder(decs) as b:
            nxt, _ = b.step()
        for i, (d, o) in enumerate(zip(decs, oss)):
            assert int(nxt[i]) == oracle.greedy(o.decode(om.embed([toks[i]]), 1))
            tok = int(nxt[i])
            for step in range(3):
                nx, lg = d.step(tok, want_logits=True)
                exp = o.decode(om.embed([tok]), 1)
                check_logits(lg, exp, f"session {i} solo step {step}")
                assert nx == oracle.greedy(exp)
                tok = nx
            assert d.position == o.position


def test_batch_capacity_and_arguments(small, oracle):
    from funasrnet_b200._lib import FaError
    from funasrnet_b200.decoder import BatchDecoder, QwenDecoder

    cm, om = small
    with prefilled(cm, om, oracle, [2, 3], seed=90, with_oracle=False) as (decs, _, _):
        with pytest.raises(FaError):
            BatchDecoder([decs[0], decs[0]])  # a session twice
        with QwenDecoder(cm) as fresh:  # no Decode yet: no token to continue from
            with BatchDecoder([decs[0], fresh]) as b:
                with pytest.raises(FaError):
                    b.generate(2)
        with BatchDecoder(decs) as b:
            with pytest.raises(FaError):
                b.generate(cm.capacity)  # past the KV capacity
            assert [d.position for d in decs] == [10, 11]


def test_batch_generate_until_end_tokens(small, oracle):
    """The end-token stop: each session's tokens equal its own generate(end_ids)
    and a stopped session keeps its position."""
    from funasrnet_b200.decoder import BatchDecoder

    cm, om = small
    lengths = [6, 30, 2, 18]
    with prefilled(cm, om, oracle, lengths, seed=110, with_oracle=False) as (probe, _, _):
        with BatchDecoder(probe) as b:
            seqs = b.generate(20)
    # an end id that occurs early in session 0's sequence and one that never occurs
    ends = [int(seqs[5, 0]), 4095 if 4095 not in seqs else 4094]
    with prefilled(cm, om, oracle, lengths, seed=110, with_oracle=False) as (a, _, _):
        with BatchDecoder(a) as b:
            got = b.generate_until(20, ends)
        with prefilled(cm, om, oracle, lengths, seed=110, with_oracle=False) as (s, _, _):
            for i, d in enumerate(s):
                alone = d.generate(20, end_ids=ends)
                assert got[i] == alone, f"session {i}"
                assert a[i].position == d.position
    assert len(got[0]) <= 5
