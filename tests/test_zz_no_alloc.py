"""fp4b_run_cached_noalloc: the cached linear for callers that cannot let a
library allocate device memory (a serving engine whose own allocator owns
nearly all of HBM, or a pipeline that cannot take the device-wide wait of a
cudaFree).  It keeps the quantized activations in a fixed array compiled into
the library instead of a cudaMalloc'd scratch buffer.

Checked through the C ABI against fp4b_run_cached_ex, the allocating entry
point it mirrors, on two calls in a row (the second must not see anything left
over from the first), plus the size limit.  This file is named to be collected
last, so a failure here leaves the rest of a stop-at-first-failure run intact.
"""
import ctypes

import pytest
import torch

from tests import workloads as W
from tests.gpu_helpers import assert_gemm_close

pytestmark = pytest.mark.gpu

_vp, _i, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
MAX_ELEMENTS = 16 << 20  # the fixed scratch holds this many padded activation elements


def _bind(lib):
    fn = lib.fp4b_run_cached_noalloc
    fn.restype = _i
    fn.argtypes = [_vp, _i, _i, _i, _vp, _i, _vp, _i, _vp, _i, _vp, _f, _f, _vp]
    return fn


def test_noalloc_matches_allocating_entry_point(cuda, fp4):
    lib = fp4._lib
    noalloc = _bind(lib)
    m, n, k = 300, 640, 1152
    _, w, b = W.cached_linear_inputs(m, n, k, seed=41)
    cache = fp4.FP4WeightCache(w.to(cuda))
    bias = b.to(cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for call, seed in enumerate((42, 43)):
        x = W.normal_bf16((m, k), 1.0, seed).to(cuda)
        got = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        want = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        rc = noalloc(x.data_ptr(), m, k, k, cache._handle, n, None, 0, got.data_ptr(), n, bias.data_ptr(), 1.0, 0.0,
                     stream)
        assert rc == 0, fp4._last_error()
        rc = lib.fp4b_run_cached_ex(x.data_ptr(), m, k, k, cache._handle, n, None, 0, want.data_ptr(), n,
                                    bias.data_ptr(), 1.0, 0.0, stream)
        assert rc == 0, fp4._last_error()
        torch.cuda.synchronize()
        assert_gemm_close(got, want.float(), f"no-alloc call {call + 1}")
    assert fp4.device_error() == 0
    cache.free()


def test_noalloc_rejects_inputs_beyond_its_scratch(cuda, fp4):
    noalloc = _bind(fp4._lib)
    k = 4096
    m = MAX_ELEMENTS // k + 128  # one 128-row tile more than fits
    _, w, _ = W.cached_linear_inputs(128, 128, k, seed=5, bias=False)
    cache = fp4.FP4WeightCache(w.to(cuda))
    x = torch.zeros(m, k, dtype=torch.bfloat16, device=cuda)
    d = torch.empty(m, 128, dtype=torch.bfloat16, device=cuda)
    rc = noalloc(x.data_ptr(), m, k, k, cache._handle, 128, None, 0, d.data_ptr(), 128, None, 1.0, 0.0, None)
    assert rc == -1
    assert "exceed the fixed scratch" in fp4._last_error()
    cache.free()
