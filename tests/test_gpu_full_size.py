"""Every configuration that bench.py times, checked at its full size through
the default dispatch (the GEMM's width model picks the tile, as in the bench).

* config 2 (the cached-linear sweep; fp4_gemm.py:324-394 of the reference
  with bias): 512x2880x2880, 2048x7680x2880 and 4096x2880x2880 against the
  CPU oracle end to end (the reference quantizer's semantics for both
  operands, fp32 matmul of the dequantized values, the BF16 bias add).  The
  headline 2048x2880x7680 and config 1 are covered in test_gpu_api.py.
* config 3 (fp4_matmul, both operands quantized per call; fp4_gemm_lib.cu:
  508-585): 16384^3 against a GPU fp32 matmul (TF32 off) of the dequantized
  operands, plus a row sample of both operands' quantized bytes against the
  CPU oracle.
* config 5 (the decoder stack's four linears at M = 8192): the cached linear
  against a GPU fp32 matmul (TF32 off) of the dequantized activation and
  cached weight bytes, the activation bytes checked against the CPU oracle on
  a row sample.

Tolerance: the GEMM contract of tests/gpu_helpers.py (max rel-err 1e-2).
"""
import numpy as np
import pytest
import torch

from tests import workloads as W
from tests.gpu_helpers import (assert_gemm_close, assert_gemm_close_device, dequant_torch, fp32_reference_no_tf32,
                               oracle_linear, oracle_quantize)

pytestmark = pytest.mark.gpu

STACK_SHAPES = [(8192, 5120, 2880), (8192, 2880, 4096), (8192, 15360, 2880), (8192, 2880, 7680)]


def _sf_rows(sf: np.ndarray, k_pad: int, tiles: int) -> np.ndarray:
    """Scale bytes of the first `tiles` 128-row tiles (contiguous in the 128x4-atom layout)."""
    return sf.reshape(-1)[: tiles * 128 * k_pad // 16]


def _check_rows_against_oracle(x_rows: torch.Tensor, fp4: torch.Tensor, sf: torch.Tensor, k_pad: int):
    """The quantized bytes of the first 128*t rows equal the CPU oracle's."""
    rows = x_rows.shape[0]
    assert rows % 128 == 0
    q, s = oracle_quantize(x_rows, rows, k_pad)
    assert np.array_equal(fp4[:rows].cpu().numpy().reshape(-1), q.reshape(-1)), "packed E2M1 bytes differ"
    assert np.array_equal(_sf_rows(sf.cpu().numpy(), k_pad, rows // 128), s.reshape(-1)), "scale bytes differ"


@pytest.mark.parametrize("m,n,k", [(512, 2880, 2880), (2048, 7680, 2880), (4096, 2880, 2880)])
def test_config2_sweep_against_oracle(cuda, fp4, m, n, k):
    x, w, b = W.cached_linear_inputs(m, n, k, seed=2000)
    cache = fp4.FP4WeightCache(w.to(cuda), b.to(cuda))
    y = cache.forward(x.to(cuda))
    assert_gemm_close(y, oracle_linear(x, w, bias=b), f"cached {m}x{n}x{k} (tile {fp4.gemm_tile_width(m, n, k)})")
    assert fp4.device_error() == 0
    cache.free()


def test_config3_dynamic_16384_cubed(cuda, fp4):
    n = 16384
    g = torch.Generator(device=cuda).manual_seed(3)
    a = torch.randn(n, n, generator=g, device=cuda).to(torch.bfloat16)
    b = torch.randn(n, n, generator=g, device=cuda).to(torch.bfloat16)
    d = fp4.fp4_matmul(a, b)  # the timed path: quantize A, quantize B, GEMM
    aq, asf = fp4.quantize_to_buffers(a, None, n)
    bq, bsf = fp4.quantize_to_buffers(b, None, n)
    torch.cuda.synchronize()
    for src, q, s in ((a, aq, asf), (b, bq, bsf)):
        _check_rows_against_oracle(src[:256].cpu(), q, s, n)
    ref = fp32_reference_no_tf32(dequant_torch(aq, asf, n, n), dequant_torch(bq, bsf, n, n))
    del aq, asf, bq, bsf
    assert_gemm_close_device(d, ref, "dynamic 16384^3")
    assert fp4.device_error() == 0


@pytest.mark.parametrize("m,n,k", STACK_SHAPES)
def test_config5_stack_linears(cuda, fp4, m, n, k):
    g = torch.Generator(device=cuda).manual_seed(n + k)
    w = (torch.randn(n, k, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
    cache = fp4.FP4WeightCache(w)
    y = cache.forward(x)
    kp = cache.K
    aq, asf = fp4.quantize_to_buffers(x, None, kp)
    sd = cache.state_dict()
    torch.cuda.synchronize()
    _check_rows_against_oracle(x[:256].cpu(), aq, asf, kp)
    ref = fp32_reference_no_tf32(dequant_torch(aq, asf, aq.shape[0], kp)[:m],
                                 dequant_torch(sd["fp4"], sd["sf"], cache.N, kp)[:n])
    assert_gemm_close_device(y, ref, f"stack linear {m}x{n}x{k} (tile {fp4.gemm_tile_width(m, n, k)})")
    assert fp4.device_error() == 0
    cache.free()
