"""B200-native (sm_100a) Qwen3 decoder token loop for FunAsrNet.

The compute lives in libfunasr_cuda.so (C ABI: include/funasr_cuda.h); this
package is the host-side mirror of the reference's backend and decoder
interfaces used by the tests and the benchmark.
"""
from ._lib import FA_DECLINED, FA_OK, FaError, lib

__all__ = ["FA_OK", "FA_DECLINED", "FaError", "lib"]
