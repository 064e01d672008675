"""Build libfp4gemm.so in place (sm_100a only).

``python fp4-gemm-blackwell_b200/build.py`` compiles every CUDA source in
``csrc/`` with nvcc for ``sm_100a`` into ``libfp4gemm.so`` beside
``fp4_gemm.py`` (the layout fp4_gemm.py:26-27 of the reference expects).
nvcc cross-compiles without a GPU.  The CUDA runtime is linked statically, so
the library only needs the driver at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libfp4gemm.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = ["capi.cu", "quantize.cu", "quantize_units.cu", "gemm_sm100.cu", "noalloc.cu", "selftest.cu", "peak.cu", "peer_barrier.cu"]
HEADERS = ["fp4b_internal.h", "nvfp4_codec.cuh", "ptx_sm100.cuh", "quantize_core.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-shared",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise FileNotFoundError("nvcc not found")


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(INCLUDE, "fp4gemm.h"), __file__]
    return all(os.path.getmtime(d) <= t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and up_to_date():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, *(extra or []), f"-I{CSRC}", f"-I{INCLUDE}",
           *[os.path.join(CSRC, f) for f in SOURCES], "-o", tmp]
    if verbose:
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    extra = [a for a in sys.argv[1:] if a.startswith("-X") or a.startswith("--")]
    extra = [a for a in extra if a not in ("--force", "--verbose")]
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv, extra=extra))
