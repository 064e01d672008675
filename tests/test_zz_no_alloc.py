"""fp4b_run_cached_noalloc: the cached linear for callers that cannot let a
library allocate device memory (a serving engine whose own allocator owns
nearly all of HBM, or a pipeline that cannot take the device-wide wait of a
cudaFree).  It keeps the quantized activations in a fixed array compiled into
the library instead of a cudaMalloc'd scratch buffer.

Checked through the C ABI against fp4b_run_cached_ex, the allocating entry
point it mirrors.  Both run the same kernels on the same bytes, so their
outputs must be identical, bit for bit:
  * two calls in a row on the CTA-pair kernel (the second must not see
    anything left over from the first);
  * a call of at most 128 rows (the one-CTA kernel);
  * a call that fills the array almost completely (2048 x 7680);
  * a large call followed by a smaller one whose input is narrower than the
    cache's K, on the same cache, so that the second call reads a region the
    first one wrote: every byte it reads must be rewritten, zero padding
    included;
plus the size limit.  This file is named to be collected last, so a failure
here leaves the rest of a stop-at-first-failure run intact.
"""
import ctypes

import pytest
import torch

from tests import workloads as W

pytestmark = pytest.mark.gpu

_vp, _i, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
MAX_ELEMENTS = 16 << 20  # the fixed scratch holds this many padded activation elements


def _bind(lib):
    fn = lib.fp4b_run_cached_noalloc
    fn.restype = _i
    fn.argtypes = [_vp, _i, _i, _i, _vp, _i, _vp, _i, _vp, _i, _vp, _f, _f, _vp]
    return fn


def _both(fp4, cuda, x, m, k_in, lda, cache, n, bias):
    """(no-alloc output, allocating output) of the same call."""
    lib = fp4._lib
    noalloc = _bind(lib)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    b_ptr = bias.data_ptr() if bias is not None else None
    got = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    want = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    rc = noalloc(x.data_ptr(), m, k_in, lda, cache._handle, n, None, 0, got.data_ptr(), n, b_ptr, 1.0, 0.0, stream)
    assert rc == 0, fp4._last_error()
    rc = lib.fp4b_run_cached_ex(x.data_ptr(), m, k_in, lda, cache._handle, n, None, 0, want.data_ptr(), n, b_ptr,
                                1.0, 0.0, stream)
    assert rc == 0, fp4._last_error()
    torch.cuda.synchronize()
    return got, want


def test_noalloc_matches_allocating_entry_point(cuda, fp4):
    m, n, k = 300, 640, 1152
    _, w, b = W.cached_linear_inputs(m, n, k, seed=41)
    cache = fp4.FP4WeightCache(w.to(cuda))
    bias = b.to(cuda)
    for call, seed in enumerate((42, 43)):
        x = W.normal_bf16((m, k), 1.0, seed).to(cuda)
        got, want = _both(fp4, cuda, x, m, k, k, cache, n, bias)
        assert torch.equal(got, want), f"no-alloc call {call + 1} differs"
    assert fp4.device_error() == 0
    cache.free()


def test_noalloc_one_cta_kernel(cuda, fp4):
    m, n, k = 100, 384, 512
    x, w, b = W.cached_linear_inputs(m, n, k, seed=44)
    cache = fp4.FP4WeightCache(w.to(cuda))
    got, want = _both(fp4, cuda, x.to(cuda), m, k, k, cache, n, b.to(cuda))
    assert torch.equal(got, want)
    cache.free()


def test_noalloc_near_the_size_limit(cuda, fp4):
    m, n, k = 2048, 512, 7680  # 2048 x 7680 = 15.7 Mi of the 16 Mi padded elements
    assert m * k <= MAX_ELEMENTS
    x, w, b = W.cached_linear_inputs(m, n, k, seed=45)
    cache = fp4.FP4WeightCache(w.to(cuda))
    got, want = _both(fp4, cuda, x.to(cuda), m, k, k, cache, n, b.to(cuda))
    assert torch.equal(got, want)
    cache.free()


def test_noalloc_smaller_narrower_call_after_a_large_one(cuda, fp4):
    n, k = 512, 4096
    _, w, b = W.cached_linear_inputs(128, n, k, seed=46)
    cache = fp4.FP4WeightCache(w.to(cuda))
    bias = b.to(cuda)
    big = W.normal_bf16((1024, k), 1.0, 47).to(cuda)
    got, want = _both(fp4, cuda, big, 1024, k, k, cache, n, bias)
    assert torch.equal(got, want)
    # 200 rows of only 3000 columns (row stride 4096): the quantizer must write
    # zeros for columns 3000..4095 and for rows 200..255 of the padded tile,
    # over what the large call left in the shared array.
    small = W.normal_bf16((200, k), 1.0, 48).to(cuda)
    got, want = _both(fp4, cuda, small, 200, 3000, k, cache, n, bias)
    assert torch.equal(got, want)
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
