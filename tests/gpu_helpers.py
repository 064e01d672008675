"""Helpers shared by the GPU parity tests: oracle references and tolerances.

GEMM tolerance: BF16 output of an fp32-accumulated
product must match the fp32 matmul of the dequantized operands within a max
relative error of 1e-2: max|D - ref| <= 1e-2 * max|ref|, and elementwise
|D - ref| <= 1e-2 * |ref| + 1e-3 * max|ref| (BF16 rounding alone is 2^-9).
Quantized bytes must be bit-exact.
"""
import numpy as np
import torch

from oracle import nvfp4_oracle as O

REL_TOL = 1e-2
ABS_FRAC = 1e-3


def assert_gemm_close(d: torch.Tensor, ref: torch.Tensor, what: str = ""):
    d = d.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert d.shape == ref.shape, (d.shape, ref.shape)
    assert torch.isfinite(d).all(), f"{what}: non-finite output"
    scale = ref.abs().max().item()
    err = (d - ref).abs()
    assert err.max().item() <= REL_TOL * scale + 1e-30, f"{what}: max err {err.max().item()} vs scale {scale}"
    bad = err > REL_TOL * ref.abs() + ABS_FRAC * scale
    assert not bad.any(), f"{what}: {int(bad.sum())} elements out of tolerance, worst {err.max().item()}"


def oracle_quantize(x_bf16: torch.Tensor, rows_pad=None, k_pad=None):
    return O.quantize(O.bf16_bits(x_bf16.cpu()), rows_pad, k_pad)


def oracle_dequant(fp4: np.ndarray, sf: np.ndarray, rows_pad: int, k_pad: int) -> torch.Tensor:
    return torch.from_numpy(O.dequantize(fp4, sf, rows_pad, k_pad))


def oracle_linear(x: torch.Tensor, w: torch.Tensor, bias=None, alpha=1.0, beta=0.0, c=None) -> torch.Tensor:
    """Reference cached/dynamic linear in fp32: pad to 128, quantize both, dequantize, matmul."""
    x = x.cpu()
    w = w.cpu()
    m, k = x.shape
    n = w.shape[0]
    kp = O.round_up(k, 128)
    mp, npad = O.round_up(m, 128), O.round_up(n, 128)
    a = oracle_dequant(*oracle_quantize(x, mp, kp), mp, kp)[:m]
    b = oracle_dequant(*oracle_quantize(w, npad, kp), npad, kp)[:n]
    out = alpha * (a @ b.t())
    if c is not None and beta != 0.0:
        out = out + beta * c.cpu().float()
    if bias is not None:
        out = out.to(torch.bfloat16).float() + bias.cpu().float()
    return out


def to_numpy_u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().astype(np.uint8, copy=False)


def pearson(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().cpu().double().flatten()
    b = b.detach().cpu().double().flatten()
    a = a - a.mean()
    b = b - b.mean()
    return float((a @ b) / (a.norm() * b.norm()))
