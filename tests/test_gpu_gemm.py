"""tcgen05 block-scaled GEMM vs the fp32 matmul of the oracle-dequantized operands.

The reference GEMM (CUTLASS SM120, fp4_gemm_lib.cu:540-580) is pinned only by
this tolerance: D must match alpha * dq(A) @ dq(B)^T + beta*C (+ bias) in fp32
within max rel-err 1e-2 (tests/gpu_helpers.py).  Both kernels (one CTA per
128-row tile, and CTA pairs on 256-row tiles) are forced in turn with every
tile width they have; ragged M/N/K, K tails of half a stage, C/alpha/beta and
bias are covered, and the headline shape runs at full size.
"""
import numpy as np
import pytest
import torch

from tests import workloads as W
from tests.gpu_helpers import assert_gemm_close, oracle_dequant, oracle_linear, oracle_quantize, pearson

pytestmark = pytest.mark.gpu

TILES = [128, 192, 256]


def run_prequant(fp4mod, x, w, bias=None, C=None, alpha=1.0, beta=0.0):
    dev = torch.device("cuda:0")
    m, k = x.shape
    n = w.shape[0]
    kp = fp4mod._pad_to_multiple(k, 128)
    aq, asf = fp4mod.quantize_to_buffers(x.to(dev), None, kp)
    bq, bsf = fp4mod.quantize_to_buffers(w.to(dev), None, kp)
    d = fp4mod.gemm_prequantized(aq, asf, m, bq, bsf, n, kp, bias=None if bias is None else bias.to(dev),
                                 C=None if C is None else C.to(dev), alpha=alpha, beta=beta)
    torch.cuda.synchronize()
    return d


@pytest.mark.parametrize("pair", [0, 1])
@pytest.mark.parametrize("bn", TILES)
@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (256, 512, 1024), (200, 300, 384), (1, 8, 128),
                                   (384, 1000, 640)])
def test_tile_widths(cuda, fp4, monkeypatch, pair, bn, m, n, k):
    monkeypatch.setenv("FP4B_FORCE_BN", str(bn))
    monkeypatch.setenv("FP4B_PAIR", str(pair))
    x = W.normal_bf16((m, k), 1.0, m + n)
    w = W.normal_bf16((n, k), 1.0, k)
    d = run_prequant(fp4, x, w)
    assert_gemm_close(d, oracle_linear(x, w), f"pair={pair} bn={bn} {m}x{n}x{k}")
    assert fp4.device_error() == 0


@pytest.mark.parametrize("deep", ["1", "0"])
@pytest.mark.parametrize("m,n,k", [(1, 8, 128), (100, 1000, 640), (300, 200, 384), (128, 2880, 2880)])
def test_one_cta_64_wide_tile(cuda, fp4, monkeypatch, deep, m, n, k):
    # The one-CTA kernel's 128 x 64 tile (FP4B_PAIR=0 FP4B_FORCE_BN=64; half of
    # its tiles start 64 rows into a scale-B atom) gives the default's bytes.
    x = W.normal_bf16((m, k), 1.0, 5 * m + n)
    w = W.normal_bf16((n, k), 1.0, k + 1)
    want = run_prequant(fp4, x, w)
    monkeypatch.setenv("FP4B_PAIR", "0")
    monkeypatch.setenv("FP4B_FORCE_BN", "64")
    monkeypatch.setenv("FP4B_DEEP", deep)
    d = run_prequant(fp4, x, w)
    assert torch.equal(d, want)
    assert_gemm_close(d, oracle_linear(x, w), f"one-CTA bn=64 {m}x{n}x{k}")
    assert fp4.device_error() == 0


def test_alpha_beta_c_bias(cuda, fp4):
    m, n, k = 256, 384, 512
    x = W.normal_bf16((m, k), 1.0, 1)
    w = W.normal_bf16((n, k), 0.02, 2)
    c = W.normal_bf16((m, n), 1.0, 3)
    b = W.normal_bf16((n,), 0.01, 4)
    for alpha, beta in ((1.0, 0.0), (0.5, 1.0), (2.0, -0.25)):
        d = run_prequant(fp4, x, w, bias=b, C=c, alpha=alpha, beta=beta)
        ref = oracle_linear(x, w, bias=b, alpha=alpha, beta=beta, c=c)
        assert_gemm_close(d, ref, f"alpha={alpha} beta={beta}")


def test_n_not_multiple_of_8(cuda, fp4):
    x = W.normal_bf16((130, 256), 1.0, 5)
    w = W.normal_bf16((37, 256), 1.0, 6)
    d = run_prequant(fp4, x, w)
    assert_gemm_close(d, oracle_linear(x, w), "n=37")


def test_headline_shape_full_size(cuda, fp4):
    m, n, k = W.HEADLINE_SHAPE
    x, w, b = W.cached_linear_inputs(m, n, k, seed=0)
    d = run_prequant(fp4, x, w, bias=b)
    ref = oracle_linear(x, w, bias=b)
    assert_gemm_close(d, ref, "2048x2880x7680")
    # accuracy vs unquantized fp32 is a property of NVFP4 with the reference's
    # scale rounding, not of the kernel: it must equal the oracle's own value.
    exact = x.float() @ w.float().t() + b.float()
    assert abs(pearson(d.cpu(), exact) - pearson(ref, exact)) < 2e-4


@pytest.mark.parametrize("m", [128, 512])
def test_accumulation_over_long_k(cuda, fp4, m):
    # K = 16384 exercises many pipeline wraps of the smem ring (m=512: CTA pairs).
    x = W.normal_bf16((m, 16384), 1.0, 8)
    w = W.normal_bf16((256, 16384), 1.0, 9)
    d = run_prequant(fp4, x, w)
    assert_gemm_close(d, oracle_linear(x, w), f"{m}x256xK=16384")


@pytest.mark.parametrize("pair", [0, 1])
def test_many_tiles_per_cta(cuda, fp4, monkeypatch, pair):
    # More tiles than SMs (pairs): every CTA walks several tiles, reusing
    # both TMEM accumulators and the smem ring across tiles.
    monkeypatch.setenv("FP4B_PAIR", str(pair))
    m, n, k = 2304, 3200, 512
    x = W.normal_bf16((m, k), 1.0, 21)
    w = W.normal_bf16((n, k), 1.0, 22)
    d = run_prequant(fp4, x, w)
    assert_gemm_close(d, oracle_linear(x, w), f"pair={pair} {m}x{n}x{k}")


def test_exact_small_integers(cuda, fp4):
    # Operands that quantize exactly (values in E2M1 x power-of-two scales):
    # the product is exact in fp32, so the result must equal the oracle bit for bit.
    g = torch.Generator().manual_seed(3)
    vals = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
    x = vals[torch.randint(0, 8, (128, 256), generator=g)] * torch.where(torch.rand(128, 256, generator=g) < .5, -1, 1)
    w = vals[torch.randint(0, 8, (128, 256), generator=g)]
    x[:, ::16] = 6.0
    w[:, ::16] = 6.0
    x, w = x.to(torch.bfloat16), w.to(torch.bfloat16)
    d = run_prequant(fp4, x, w)
    ref = (x.float() @ w.float().t())
    assert torch.equal(d.float().cpu(), ref.to(torch.bfloat16).float())
    aq, asf = oracle_quantize(x)
    assert torch.equal(oracle_dequant(aq, asf, 128, 256), x.float())


def test_dynamic_8192_cubed_against_torch_fp32(cuda, fp4):
    # Config 3 at full size: both operands quantized on the GPU (bytes pinned
    # elsewhere against the oracle), the GEMM checked against torch fp32 (no
    # TF32) on the dequantized operands.
    from tests.gpu_helpers import dequant_torch
    n = 8192
    g = torch.Generator(device=cuda).manual_seed(5)
    a = torch.randn(n, n, generator=g, device=cuda).to(torch.bfloat16)
    b = torch.randn(n, n, generator=g, device=cuda).to(torch.bfloat16)
    aq, asf = fp4.quantize_to_buffers(a, None, n)
    bq, bsf = fp4.quantize_to_buffers(b, None, n)
    d = fp4.gemm_prequantized(aq, asf, n, bq, bsf, n, n)
    torch.cuda.synchronize()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = dequant_torch(aq, asf, n, n) @ dequant_torch(bq, bsf, n, n).t()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    err = (d.float() - ref).abs()
    scale = ref.abs().max()
    assert err.max() <= 1e-2 * scale, (err.max().item(), scale.item())
    assert not (err > 1e-2 * ref.abs() + 1e-3 * scale).any()
    # and the dynamic API gives the same bytes
    assert torch.equal(fp4.fp4_matmul(a, b), d)


def test_dequant_torch_matches_oracle(cuda, fp4):
    from tests.gpu_helpers import dequant_torch, oracle_dequant
    x = W.normal_bf16((256, 384), 1.0, 31)
    aq, asf = fp4.quantize_to_buffers(x.to(cuda), None, 384)
    torch.cuda.synchronize()
    got = dequant_torch(aq, asf, 256, 384).cpu()
    want = oracle_dequant(aq.cpu().numpy().reshape(-1), asf.cpu().numpy().reshape(-1), 256, 384)
    assert torch.equal(got, want)


@pytest.mark.parametrize("m,n,k", [(256, 384, 512), (300, 1000, 640), (257, 769, 256), (2304, 3200, 512),
                                   (2048, 2880, 7680)])
@pytest.mark.parametrize("width", ["384", "320"])
def test_wide_pair_tile_equals_default(cuda, fp4, monkeypatch, m, n, k, width):
    # The 256 x 384 and 256 x 320 pair tiles (two MMAs per k-block on one A
    # tile, N = 192 + 192 or 128 + 192, one TMEM accumulator) run the same K
    # sequence per output element as the other widths, so their bytes equal
    # theirs; also close to the oracle, and several tiles per pair
    # (2304 x 3200) reuse the single accumulator.  320-wide tiles start 0 or
    # 64 rows into a 128-row scale atom.
    x = W.normal_bf16((m, k), 1.0, 71)
    w = W.normal_bf16((n, k), 1.0, 72)
    b = W.normal_bf16((n,), 1.0, 73)
    monkeypatch.setenv("FP4B_PAIR", "1")
    monkeypatch.setenv("FP4B_FORCE_BN", "192")
    narrow = run_prequant(fp4, x, w, bias=b)
    monkeypatch.setenv("FP4B_FORCE_BN", width)
    wide = run_prequant(fp4, x, w, bias=b)
    assert torch.equal(wide, narrow)
    if m * n * k < 1e9:
        assert_gemm_close(wide, oracle_linear(x, w, bias=b), f"{width}-wide {m}x{n}x{k}")
    assert fp4.device_error() == 0


@pytest.mark.parametrize("pair,bn", [(0, 128), (1, 128), (1, 192), (1, 256), (1, 320), (1, 384)])
@pytest.mark.parametrize("m,n,k,alpha", [(2048, 2880, 7680, 1.0), (300, 1000, 640, 0.37), (4096, 640, 1024, 1.0)])
def test_bias_add_equals_bf16_add_of_unbiased_output(cuda, fp4, monkeypatch, pair, bn, m, n, k, alpha):
    # The reference adds the bias to the BF16 GEMM output in BF16 (fp32 sum,
    # one rounding).  Every epilogue must give exactly torch's BF16 add of its
    # own unbiased output and the bias, for biases over 80 binades (sums that
    # are exact in fp32, and ones where the smaller operand vanishes), zeros
    # and +-inf.
    if pair == 0 and m > 128 and bn == 128:
        m = 128  # the one-CTA kernel's own shape range
    monkeypatch.setenv("FP4B_PAIR", str(pair))
    monkeypatch.setenv("FP4B_FORCE_BN", str(bn))
    x = W.normal_bf16((m, k), 1.0, 81)
    w = W.normal_bf16((n, k), 1.0, 82)
    g = torch.Generator().manual_seed(83)
    b = torch.randn(n, generator=g) * torch.exp2(torch.randint(-40, 41, (n,), generator=g).float())
    b[::97] = 0.0
    b[5], b[6] = float("inf"), float("-inf")
    b = b.to(torch.bfloat16)
    plain = run_prequant(fp4, x, w, alpha=alpha)
    biased = run_prequant(fp4, x, w, bias=b, alpha=alpha)
    want = (plain.float() + b.to(plain.device).float()).to(torch.bfloat16)
    assert torch.equal(biased, want)
    assert fp4.device_error() == 0


@pytest.mark.parametrize("bn", ["128", "192"])
@pytest.mark.parametrize("m,n,k", [(1, 2880, 2880), (300, 1000, 640), (256, 384, 128), (2304, 3200, 2944),
                                   (512, 2880, 7680)])
def test_two_k_chunks_per_stage_equal_one(cuda, fp4, monkeypatch, bn, m, n, k):
    # The 128- and 192-wide pair tiles load two 128-byte K chunks per stage by
    # default (a K of 512 per stage; the last stage may hold 1-7 of its 8
    # k-blocks); the MMAs run in the same K order, so the bytes equal one chunk
    # per stage, including multi-round shapes that reuse both accumulators.
    x = W.normal_bf16((m, k), 1.0, 3 * m + k)
    w = W.normal_bf16((n, k), 1.0, n + 7)
    b = W.normal_bf16((n,), 1.0, 11)
    monkeypatch.setenv("FP4B_FORCE_BN", bn)
    monkeypatch.setenv("FP4B_KCHUNKS", "1")
    one = run_prequant(fp4, x, w, bias=b)
    monkeypatch.setenv("FP4B_KCHUNKS", "2")
    two = run_prequant(fp4, x, w, bias=b)
    assert torch.equal(two, one)
    if m * n * k < 2e9:
        assert_gemm_close(two, oracle_linear(x, w, bias=b), f"2 K chunks bn={bn} {m}x{n}x{k}")
    assert fp4.device_error() == 0
