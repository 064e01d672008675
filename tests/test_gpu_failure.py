"""The kernels' failure path on the GPU, without a fault: a bounded wait on
something that never completes gives up after its limit, its code reaches the
host through the device error word, and the context stays usable."""
import time

import pytest
import torch

from tests import workloads as W
from tests.gpu_helpers import assert_gemm_close, oracle_linear

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("which,code", [(0, 7), (1, 8)])
def test_bounded_wait_gives_up_and_the_context_stays_usable(cuda, fp4, which, code):
    assert fp4.device_error(clear=True) == 0
    stream = torch.cuda.current_stream(cuda).cuda_stream
    t0 = time.monotonic()
    assert fp4._lib.fp4b_selftest_bounded_wait(which, stream) == 0, fp4._last_error()
    got = fp4.device_error(clear=True)  # synchronises
    elapsed = time.monotonic() - t0
    assert got == code
    assert 1.5 < elapsed < 60  # the 2 s bound, not an endless spin
    assert fp4.device_error(clear=False) == 0
    # later work on the same context runs and is right
    x, w, b = W.cached_linear_inputs(256, 384, 512, seed=91)
    with fp4.FP4WeightCache(w.to(cuda), b.to(cuda)) as cache:
        y = cache.forward(x.to(cuda))
    assert_gemm_close(y, oracle_linear(x, w, bias=b), "after a timed-out wait")
    assert fp4.device_error() == 0


def test_selftest_rejects_unknown_kind(fp4):
    assert fp4._lib.fp4b_selftest_bounded_wait(2, None) == -1
    assert "which must be" in fp4._last_error()
