"""Guard bytes around every output: each kernel writes exactly its outputs.

The GEMM's output D goes into the middle of a larger buffer filled with a
sentinel (rows above and below, and columns past N when the row stride is
larger than N); the quantizer's packed E2M1 and scale outputs go between 4 KB
guard zones.  After the call, every guard element must still hold its sentinel
and the output must equal the same call into a plain buffer.  Both GEMM kernels
and every tile width are forced in turn, with row strides that take the
TMA-store epilogue (16-byte aligned rows) and the plain-store one (odd
stride), one and several tiles per CTA (pair).
"""
import pytest
import torch

from tests import workloads as W

pytestmark = pytest.mark.gpu

SENTINEL = -12288.0  # exact in BF16, never produced by these inputs
GUARD = 4096


@pytest.mark.parametrize("pair,bn,m,n", [(0, 128, 100, 1000), (0, 256, 128, 1000), (1, 192, 300, 1000),
                                         (1, 256, 300, 1000), (1, 320, 300, 1000), (1, 384, 300, 1000),
                                         (1, 128, 4096, 1000), (1, 384, 8192, 1000),
                                         # CTA pairs at M <= 128 (the default): the second CTA's rows are padding
                                         (1, 128, 100, 1000), (1, 320, 1, 1000), (1, 192, 128, 1000),
                                         # more column tiles than CTA pairs: the ragged last row tile is
                                         # stored by the per-tile epilogue too, not only the last-tile team
                                         (1, 128, 300, 10000), (1, 192, 300, 14500), (1, 320, 300, 24000)])
@pytest.mark.parametrize("ldd_extra", [24, 3])
def test_gemm_writes_only_its_output(cuda, fp4, monkeypatch, pair, bn, m, n, ldd_extra):
    k = 640
    monkeypatch.setenv("FP4B_PAIR", str(pair))
    monkeypatch.setenv("FP4B_FORCE_BN", str(bn))
    x, w, b = W.cached_linear_inputs(m, n, k, seed=61)
    bias = b.to(cuda)
    cache = fp4.FP4WeightCache(w.to(cuda), bias)
    xd = x.to(cuda)
    want = cache.forward(xd)
    ldd = n + ldd_extra
    top, bottom = 4, 5
    buf = torch.full((top + m + bottom, ldd), SENTINEL, dtype=torch.bfloat16, device=cuda)
    d = buf[top:top + m]
    stream = torch.cuda.current_stream(cuda).cuda_stream
    rc = fp4._lib.fp4b_run_cached_ex(xd.data_ptr(), m, k, k, cache._handle, n, None, 0, d.data_ptr(), ldd,
                                     bias.data_ptr(), 1.0, 0.0, stream)
    assert rc == 0, fp4._last_error()
    torch.cuda.synchronize()
    assert torch.equal(buf[top:top + m, :n], want)
    guard = torch.ones(buf.shape, dtype=torch.bool, device=cuda)
    guard[top:top + m, :n] = False
    assert bool((buf[guard] == SENTINEL).all())
    assert fp4.device_error() == 0
    cache.free()


@pytest.mark.parametrize("rows,cols", [(300, 2880), (128, 640), (200, 300), (5, 7680)])
def test_quantizer_writes_only_its_output(cuda, fp4, rows, cols):
    # Staged kernel (row length a multiple of 64) and register kernel (300),
    # with padding rows and K padding written as zeros inside the outputs.
    rows_pad, k_pad = (rows + 127) // 128 * 128, (cols + 127) // 128 * 128
    n_fp4, n_sf = rows_pad * k_pad // 2, rows_pad * k_pad // 16
    x = W.normal_bf16((rows, cols), 1.0, 71).to(cuda)
    want_q, want_s = fp4.quantize_to_buffers(x, rows_pad, k_pad)
    qbuf = torch.full((GUARD + n_fp4 + GUARD,), 0xA5, dtype=torch.uint8, device=cuda)
    sbuf = torch.full((GUARD + n_sf + GUARD,), 0x5A, dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    rc = fp4._lib.fp4b_quantize(x.data_ptr(), rows, cols, cols, qbuf[GUARD:].data_ptr(), sbuf[GUARD:].data_ptr(),
                                rows_pad, k_pad, stream)
    assert rc == 0, fp4._last_error()
    torch.cuda.synchronize()
    assert torch.equal(qbuf[GUARD:GUARD + n_fp4], want_q.reshape(-1))
    assert torch.equal(sbuf[GUARD:GUARD + n_sf], want_s.reshape(-1))
    assert bool((qbuf[:GUARD] == 0xA5).all()) and bool((qbuf[GUARD + n_fp4:] == 0xA5).all())
    assert bool((sbuf[:GUARD] == 0x5A).all()) and bool((sbuf[GUARD + n_sf:] == 0x5A).all())
