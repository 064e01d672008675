"""Build recipes for the test oracle (TEST INFRASTRUCTURE ONLY).

* ``build_oracle()`` compiles ``nvfp4_oracle.c`` (the C restatement of the
  reference quantizer) into ``oracle/libnvfp4_oracle.so``.
* ``build_ref()`` compiles the reference's OWN quantizer source for the host
  into ``oracle/_ref/libref_quant.so``.  It reads
  ``fp4_gemm_lib.cu`` of VincentKaufmann/fp4-gemm-blackwell where it lies,
  takes the section from the E2M1 constant table through the end of
  ``quantize_bf16_to_fp4_kernel`` (fp4_gemm_lib.cu:106-286) into a temporary
  directory, and compiles it with ``ref_shim.h`` + ``ref_driver.cpp``.  Nothing
  from the reference is written into the repository; only the ``.so`` lands in
  ``oracle/_ref/`` (git-ignored).  The CUTLASS GEMM half of that file needs an
  external library (CUTLASS 3.8, fetched over the network by the reference's
  build.sh) and an SM120 GPU, so it is not built.

Where the reference's source is read from: the path in the environment
variable ``FP4_REFERENCE_LIB_CU`` (the reference's ``fp4_gemm_lib.cu``), else
``<reference_path>/fp4_gemm_lib.cu`` with ``reference_path`` taken from this
repository's ``BASELINE.json`` (the build's own record of where the reference
checkout was surveyed).  When neither exists -- e.g. on a GPU box, which only
uses the prebuilt files -- the reference step is skipped and a library built
earlier is kept.

Run ``python oracle/build.py`` to build both.
"""
from __future__ import annotations

import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libnvfp4_oracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_SO = os.path.join(REF_DIR, "libref_quant.so")


def reference_lib_cu() -> str | None:
    """Location of the reference's fp4_gemm_lib.cu (see the module docstring), or None."""
    env = os.environ.get("FP4_REFERENCE_LIB_CU")
    if env:
        return env
    baseline = os.path.join(os.path.dirname(HERE), "BASELINE.json")
    try:
        import json
        with open(baseline, encoding="utf-8") as f:
            root = json.load(f).get("reference_path")
    except (OSError, ValueError):
        return None
    return os.path.join(root, "fp4_gemm_lib.cu") if root else None


# Both compiles keep IEEE fp32 semantics: no contraction, no fast-math.
_FP_FLAGS = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared"]


def _newer(target: str, *deps: str) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps if os.path.exists(d))


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "nvfp4_oracle.c")
    if force or not _newer(ORACLE_SO, src):
        cmd = ["gcc", "-std=c11", *_FP_FLAGS, src, "-o", ORACLE_SO, "-lm"]
        subprocess.check_call(cmd)
    return ORACLE_SO


def extract_reference_quantizer(lib_cu: str) -> str:
    """Return the quantizer section of the reference's fp4_gemm_lib.cu.

    Starts at the line declaring the E2M1 constant table and ends at the
    closing brace of ``quantize_bf16_to_fp4_kernel``.  Raises if the markers
    are not found exactly once, so a changed reference fails loudly.
    """
    with open(lib_cu, "r", encoding="utf-8") as f:
        lines = f.read().splitlines()
    starts = [i for i, l in enumerate(lines) if l.startswith("__constant__ float c_fp4_values")]
    kern = [i for i, l in enumerate(lines) if l.startswith("__global__ void quantize_bf16_to_fp4_kernel(")]
    if len(starts) != 1 or len(kern) != 1 or kern[0] < starts[0]:
        raise RuntimeError(f"quantizer markers not found in {lib_cu}")
    end = next(i for i in range(kern[0], len(lines)) if lines[i] == "}")
    return "\n".join(lines[starts[0]: end + 1]) + "\n"


def build_ref(force: bool = False) -> str | None:
    """Compile the reference quantizer for the host; None when the reference is absent."""
    lib_cu = reference_lib_cu()
    if not lib_cu or not os.path.exists(lib_cu):
        return REF_SO if os.path.exists(REF_SO) else None
    deps = (lib_cu, os.path.join(HERE, "ref_shim.h"), os.path.join(HERE, "ref_driver.cpp"))
    if not force and _newer(REF_SO, *deps):
        return REF_SO
    os.makedirs(REF_DIR, exist_ok=True)
    section = extract_reference_quantizer(lib_cu)
    with tempfile.TemporaryDirectory() as tmp:
        inc = os.path.join(tmp, "ref_quant_section.inc")
        with open(inc, "w", encoding="utf-8") as f:
            f.write(section)
        cmd = ["g++", "-std=c++17", *_FP_FLAGS, "-Wno-unknown-pragmas", f"-I{HERE}",
               f'-DREF_QUANT_SOURCE="{inc}"', os.path.join(HERE, "ref_driver.cpp"), "-o", REF_SO]
        subprocess.check_call(cmd)
    return REF_SO


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build_oracle(force))
    print(build_ref(force))
