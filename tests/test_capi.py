"""The C ABI library loads, exports every declared symbol, and rejects bad
arguments on the host (no GPU work is issued by these tests)."""
import ctypes
import os
import re

import pytest

from tests.conftest import PKG, ROOT

HEADER = os.path.join(ROOT, "include", "fp4gemm.h")
LIB = os.path.join(PKG, "libfp4gemm.so")

# The symbols the reference library exports (fp4_gemm_lib.cu:401-842).
REFERENCE_SYMBOLS = [
    "fp4_gemm_sf_vec_size", "fp4_gemm_init", "fp4_gemm_prealloc", "fp4_gemm_run", "fp4_gemm_run_host",
    "fp4_gemm_cleanup", "fp4_gemm_sync", "fp4_quantize_weights", "fp4_weight_cache_fp4_ptr",
    "fp4_weight_cache_sf_ptr", "fp4_weight_cache_N", "fp4_weight_cache_K", "fp4_weight_cache_free",
    "fp4_gemm_run_cached",
]


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(fp4[A-Za-z0-9_]*)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    assert os.path.exists(LIB), "libfp4gemm.so not built"
    return ctypes.CDLL(LIB)


def test_header_declares_reference_abi():
    decl = declared_functions()
    assert set(REFERENCE_SYMBOLS) <= set(decl)


def test_every_declared_symbol_is_exported(lib):
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, f"not exported: {missing}"


def test_host_side_contract(lib):
    lib.fp4_quantize_weights.restype = ctypes.c_void_p
    lib.fp4b_weight_cache_slice.restype = ctypes.c_void_p
    lib.fp4_weight_cache_fp4_ptr.restype = ctypes.c_void_p
    lib.fp4b_last_error.restype = ctypes.c_char_p
    assert lib.fp4_gemm_sf_vec_size() == 16
    assert lib.fp4b_version() == 1
    # shape errors are reported before any device work (fp4_gemm_lib.cu:673-676, 762-774)
    assert lib.fp4_quantize_weights(None, 100, 128) is None
    assert b"multiples of 128" in lib.fp4b_last_error()
    assert lib.fp4_gemm_run_cached(None, None, None, None, 128, ctypes.c_float(1.0), ctypes.c_float(0.0)) == -1
    assert lib.fp4_gemm_init(100, 128, 128) == -1
    assert lib.fp4_gemm_run_host(None, None, None, None, 128, 128, 128, ctypes.c_float(1.0), ctypes.c_float(0.0)) == -2
    # NULL handles: getters return 0 / NULL, free is NULL-safe (fp4_gemm_lib.cu:723-750)
    assert lib.fp4_weight_cache_N(None) == 0 and lib.fp4_weight_cache_K(None) == 0
    assert lib.fp4_weight_cache_fp4_ptr(None) is None
    lib.fp4_weight_cache_free(None)
    assert lib.fp4b_weight_cache_slice(None, 0, 128) is None


def test_python_module_imports_without_gpu():
    import fp4_gemm
    assert fp4_gemm.SF_VEC_SIZE == 16
    assert fp4_gemm._pad_to_multiple(2880, 128) == 2944
    for name in ["fp4_matmul", "fp4_linear", "FP4WeightCache", "fp4_quantize", "fp4_cached_matmul",
                 "fp4_cached_linear", "sync", "prealloc", "cleanup"]:
        assert callable(getattr(fp4_gemm, name))


def test_python_argument_errors_match_reference():
    import torch

    import fp4_gemm
    w = torch.zeros(128, 128, dtype=torch.bfloat16)
    with pytest.raises(AssertionError, match="Weight must be on CUDA"):
        fp4_gemm.FP4WeightCache(w)
    with pytest.raises(AssertionError, match="Weight must be 2D"):
        fp4_gemm.FP4WeightCache(torch.zeros(4, dtype=torch.bfloat16))
    with pytest.raises(AssertionError, match="K mismatch"):
        fp4_gemm.fp4_matmul(torch.zeros(4, 8), torch.zeros(4, 16))
    with pytest.raises(AssertionError, match="Both tensors must be on CUDA"):
        fp4_gemm.fp4_matmul(torch.zeros(4, 8), torch.zeros(4, 8))


_ALLOC_FAILURE_SCRIPT = r"""
import ctypes, sys
lib = ctypes.CDLL(sys.argv[1])
lib.fp4_quantize_weights.restype = ctypes.c_void_p
lib.fp4b_last_error.restype = ctypes.c_char_p
buf = ctypes.create_string_buffer(128 * 128 * 2)
p = ctypes.cast(buf, ctypes.c_void_p)
one, zero = ctypes.c_float(1.0), ctypes.c_float(0.0)
res = [lib.fp4_quantize_weights(p, 128, 128) is None, lib.fp4b_last_error()]
res += [lib.fp4_gemm_init(128, 128, 128), lib.fp4b_last_error()]
res += [lib.fp4_gemm_prealloc(128, 128, 128), lib.fp4_gemm_run(p, p, None, p, 128, 128, 128, one, zero)]
lib.fp4_gemm_cleanup()
print(repr(res))
"""


def test_allocation_failures_return_errors():
    # Host-side fault injection: with no device visible every cudaMalloc the
    # library makes fails.  The calls that allocate must return their error
    # value with a message (where the reference leaves cudaMalloc unchecked,
    # fp4_gemm_lib.cu:467-470) and leave the process usable.
    import ast
    import subprocess
    import sys
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, "-c", _ALLOC_FAILURE_SCRIPT, LIB], env=env, capture_output=True, text=True,
                         timeout=120)
    assert out.returncode == 0, out.stderr[-2000:]
    null_cache, msg_q, rc_init, msg_init, rc_pre, rc_run = ast.literal_eval(out.stdout.strip().splitlines()[-1])
    assert null_cache and b"cudaMalloc" in msg_q
    assert rc_init == -1 and b"cudaMalloc" in msg_init
    assert rc_pre == -1 and rc_run == -1


def test_peer_outputs_must_be_16_byte_aligned(lib):
    # The column-parallel epilogue stores 16 bytes at a time into D and into
    # every peer buffer; a misaligned address or row stride is refused with -2
    # on the host, before the cache handle is even looked up, so no kernel can
    # fault on it.  (Fake addresses: nothing is dereferenced.)
    lib.fp4b_last_error.restype = ctypes.c_char_p
    fn = lib.fp4b_run_cached_peers
    fn.restype = ctypes.c_int
    vp = ctypes.c_void_p
    fn.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, ctypes.c_int, vp, ctypes.c_int,
                   ctypes.POINTER(vp), ctypes.c_int, vp, vp]

    def call(d, ldd, peers):
        arr = (vp * len(peers))(*peers)
        return fn(0x10000, 256, 512, 512, None, 512, d, ldd, arr, len(peers), None, None)

    assert call(0x20000, 512, [0x30008]) == -2
    assert b"16-byte aligned" in lib.fp4b_last_error()
    assert call(0x20000, 512, [0x30000, 0x40004]) == -2   # the second peer is off
    assert call(0x20008, 512, [0x30000]) == -2            # D itself
    assert call(0x20000, 508, [0x30000]) == -2            # row stride not a multiple of 8 elements
    assert call(0x20000, 512, [0x30000, None]) == -2      # NULL peer
    # aligned everything: the call goes on to the handle check (NULL here) and fails there instead
    assert call(0x20000, 512, [0x30000, 0x40000]) == -1
    assert b"cache handle" in lib.fp4b_last_error()


def test_peer_barrier_rejects_bad_arguments(lib):
    # fp4b_peer_barrier checks its arguments on the host before any launch.
    lib.fp4b_last_error.restype = ctypes.c_char_p
    fn = lib.fp4b_peer_barrier
    fn.restype = ctypes.c_int
    vp = ctypes.c_void_p
    fn.argtypes = [vp, ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int,
                   ctypes.c_ulonglong, vp]

    def call(mine, peers, ranks, my_rank, epoch):
        p = (vp * max(1, len(peers)))(*peers)
        r = (ctypes.c_int * max(1, len(ranks)))(*ranks)
        return fn(mine, p, r, len(peers), my_rank, epoch, None)

    assert call(None, [0x1000], [1], 0, 1) == -1            # no flag array
    assert call(0x2000, [], [], 0, 1) == -1                 # no peers
    assert call(0x2000, [0x1000], [1], 0, 0) == -1          # epochs start at 1
    assert call(0x2004, [0x1000], [1], 0, 1) == -1          # misaligned own array
    assert call(0x2000, [0x1004], [1], 0, 1) == -1          # misaligned peer array
    assert call(0x2000, [0x1000], [0], 0, 1) == -1          # a peer with this rank's own rank
    assert call(0x2000, [0x1000] * 8, list(range(1, 9)), 0, 1) == -1  # at most 7 peers
    assert b"fp4b_peer_barrier" in lib.fp4b_last_error()
