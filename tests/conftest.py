import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device; runs through the C ABI")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.build()
    O.set_threads(min(8, os.cpu_count() or 1))
    return O


@pytest.fixture(scope="session")
def built_lib():
    from funasrnet_b200 import build

    return build.build_library()


@pytest.fixture(scope="session")
def backend(built_lib):
    from funasrnet_b200.backend import CudaFloatBackend

    b = CudaFloatBackend(0)
    yield b


@pytest.fixture(scope="session")
def ops(backend):
    from funasrnet_b200.backend import Ops

    return Ops(backend)


@pytest.fixture(scope="session")
def small_gguf(tmp_path_factory, built_lib):
    """2-layer full-width Qwen3 with a 4096-token vocabulary (seed 11)."""
    from funasrnet_b200._lib import check, lib

    p = tmp_path_factory.mktemp("models") / "small_q8.gguf"
    check(lib().fa_synth_write_gguf(str(p).encode(), 11, 2, 4096, 0, 0, 1))
    return p


@pytest.fixture(scope="session")
def small_gguf_f32(tmp_path_factory, built_lib):
    from funasrnet_b200._lib import check, lib

    p = tmp_path_factory.mktemp("models") / "small_f32.gguf"
    check(lib().fa_synth_write_gguf(str(p).encode(), 12, 2, 4096, 0, 0, 0))
    return p


def f32_bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def assert_bits_equal(actual, expected, what=""):
    a, e = f32_bits(actual), f32_bits(expected)
    both_nan = np.isnan(np.asarray(actual, np.float32)) & np.isnan(np.asarray(expected, np.float32))
    bad = (a != e) & ~both_nan
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(f"{what}: {int(bad.sum())} of {a.size} values differ; first at {i}: "
                             f"{np.asarray(actual).reshape(-1)[i]!r} vs {np.asarray(expected).reshape(-1)[i]!r}")
