"""Builds libfunasr_cuda.so in-tree for sm_100a with nvcc.

    python -m funasrnet_b200.build            # library only
    python -m funasrnet_b200.build --oracle   # also the CPU oracle (test infrastructure)
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libfunasr_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fmad=false: every a*b+c stays two roundings unless a kernel asks for an FMA
# explicitly, matching the reference's RyuJIT evaluation.
# Calls from device code into host-only functions (diagnostics 20011-20015)
# are errors: nvcc only warns, and the device compiler then treats the calling
# path as unreachable and drops it.
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC,-O3,-ffp-contract=off",
                     "-Xptxas", "-v", "-diag-error", "20011,20012,20013,20014,20015"]
SOURCES = ["decoder_kernels.cu", "mega.cu", "batch.cu", "f32_stream.cu", "runtime.cu", "host_util.cpp"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def host_compiler() -> list[str]:
    # The image's default CXX can point at a toolchain without libgomp specs;
    # the system g++ is the one nvcc supports.
    gxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else shutil.which("g++")
    return ["-ccbin", gxx] if gxx else []


def _compile(src: Path, obj: Path) -> str:
    cmd = [nvcc(), *host_compiler(), *NVCC_FLAGS, "-x", "cu" if src.suffix == ".cu" else "c++", "-c", str(src),
           "-o", str(obj)]
    if src.suffix != ".cu":
        cmd = [nvcc(), *host_compiler(), "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3,-ffp-contract=off", "-c",
               str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build_library(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    deps = sorted(CSRC.glob("*")) + [ROOT / "include" / "funasr_cuda.h"]
    newest = max(p.stat().st_mtime for p in deps)
    if LIB.exists() and LIB.stat().st_mtime >= newest and os.environ.get("FA_FORCE_BUILD") != "1":
        return LIB
    objs = []
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        futs = {}
        for name in SOURCES:
            src = CSRC / name
            obj = BUILD / (src.stem + ".o")
            objs.append(obj)
            futs[ex.submit(_compile, src, obj)] = name
        for f in cf.as_completed(futs):
            log = f.result()
            if verbose:
                print(f"--- {futs[f]}\n{log}")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *host_compiler(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    tmp.replace(LIB)
    return LIB


def build_oracle() -> Path:
    """The CPU oracle is test infrastructure (tests/, smoke(), bench cpu_baseline)."""
    oracle = ROOT / "oracle"
    r = subprocess.run(["make", "-C", str(oracle)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed\n{r.stdout}\n{r.stderr}")
    return oracle / "liboracle.so"


if __name__ == "__main__":
    print(build_library(verbose="-v" in sys.argv))
    if "--oracle" in sys.argv:
        print(build_oracle())
