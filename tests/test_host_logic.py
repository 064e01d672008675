"""Host-side logic of the Python layer that needs no GPU."""
import fp4_gemm


def test_forward_host_chunk_schedule():
    for m in (1, 60, 127, 128, 129, 700, 2048, 4096, 5000):
        for chunk in (128, 256, 512):
            sizes = fp4_gemm._chunk_schedule(m, chunk)
            assert sum(sizes) == m
            assert all(0 < s <= chunk for s in sizes)
            assert all(s == chunk for s in sizes[:-1])
    assert fp4_gemm._chunk_schedule(2048, 512) == [512] * 4
    assert fp4_gemm._chunk_schedule(700, 256) == [256, 256, 188]


def test_global_weight_scale_is_largest_fitting_power_of_two():
    import math
    for amax in (0.05, 0.02, 1.0, 6.0, 2879.0, 2880.0, 3000.0, 1e-6, 7.3e4):
        s = fp4_gemm.global_weight_scale(amax)
        assert s == 2.0 ** round(math.log2(s))            # a power of two
        assert amax * s / 6.0 <= 480.0                     # largest block scale fits UE4M3
        assert amax * (2 * s) / 6.0 > 480.0                # and no larger power of two does
    for bad in (0.0, float("nan"), float("inf"), -1.0):
        assert fp4_gemm.global_weight_scale(bad) == 1.0


def test_global_scale_reduces_error_of_small_weights_in_the_oracle():
    # N(0, 0.02) weights: their block scales (|w|max / 6 ~ 0.01) are UE4M3
    # subnormals, truncated to multiples of 2^-9.  Scaling by the global power
    # of two moves them into the normal range; the oracle (the reference's
    # quantizer) shows the reconstruction error drop.
    import numpy as np
    import torch
    from oracle import nvfp4_oracle as O
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(256, 1024, generator=g) * 0.02).to(torch.bfloat16)
    s = fp4_gemm.global_weight_scale(float(w.abs().max()))
    ws = (w.float() * s).to(torch.bfloat16)
    assert torch.equal(ws.float() / s, w.float())        # the scaling is exact
    ref = w.float().numpy()
    q0, f0 = O.quantize(w)
    q1, f1 = O.quantize(ws)
    rms = lambda d: float(np.sqrt(((d - ref) ** 2).mean() / (ref ** 2).mean()))
    e0 = rms(O.dequantize(q0, f0, 256, 1024))
    e1 = rms(O.dequantize(q1, f1, 256, 1024) / s)
    assert e1 < 0.85 * e0, (e0, e1)  # measured 0.129 -> 0.095


def test_gemm_tile_width_model_decisions():
    # The tile width the GEMM picks from its time model (host only), for the
    # shapes it was fitted on, with B200's 148 SMs: the 320-wide two-MMA tile
    # for the headline (72 tiles on 74 CTA pairs), the 384-wide one for wide-N
    # short-K shapes (config-5 gate_up) and 8192^3, the 192-wide one (two K
    # chunks per stage) for most other multi-round shapes, narrower tiles for
    # small M (CTA pairs at every M, a pair's second CTA all padding at M <= 128).
    import pytest

    import fp4_gemm
    want = {(2048, 2880, 7680): 320, (4096, 2880, 7680): 320, (8192, 15360, 2880): 384, (8192, 5120, 2880): 192,
            (8192, 8192, 8192): 384, (16384, 16384, 16384): 384, (2048, 5120, 2880): 192, (1024, 2880, 7680): 192,
            (512, 2880, 2880): 128, (256, 2880, 2880): 128}
    got = {s: fp4_gemm.gemm_tile_width(*s) for s in want}
    assert got == want
    assert fp4_gemm.gemm_tile_width(128, 2880, 2880) == 128  # the same model as M = 256: one row of pair tiles
    assert fp4_gemm.gemm_tile_width(1, 8, 128) in (128, 192, 256, 320, 384)
    with pytest.raises(ValueError):
        fp4_gemm.gemm_tile_width(0, 128, 128)
