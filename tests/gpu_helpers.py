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


def assert_gemm_close_device(d: torch.Tensor, ref: torch.Tensor, what: str = ""):
    """assert_gemm_close evaluated where the tensors are (for outputs of
    hundreds of millions of elements, which are slow to copy to the host)."""
    assert d.shape == ref.shape, (d.shape, ref.shape)
    d = d.float()
    assert bool(torch.isfinite(d).all()), f"{what}: non-finite output"
    scale = ref.abs().max()
    err = (d - ref).abs()
    worst = err.max()
    assert bool(worst <= REL_TOL * scale + 1e-30), f"{what}: max err {worst.item()} vs scale {scale.item()}"
    bad = int((err > REL_TOL * ref.abs() + ABS_FRAC * scale).sum())
    assert bad == 0, f"{what}: {bad} elements out of tolerance, worst {worst.item()}"


def fp32_reference_no_tf32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a @ b^T in fp32 on the tensors' device with TF32 disabled."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return a @ b.t()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def to_numpy_u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().astype(np.uint8, copy=False)


def pearson(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().cpu().double().flatten()
    b = b.detach().cpu().double().flatten()
    a = a - a.mean()
    b = b - b.mean()
    return float((a @ b) / (a.norm() * b.norm()))


_E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


def dequant_torch(fp4: torch.Tensor, sf: torch.Tensor, rows_pad: int, k_pad: int) -> torch.Tensor:
    """fp32 [rows_pad, k_pad] from packed E2M1 bytes and 128x4-atom UE4M3 scales,
    on the tensors' device (a torch restatement of oracle.dequantize for sizes
    the CPU oracle cannot finish quickly)."""
    dev = fp4.device
    lut = torch.tensor(_E2M1, dtype=torch.float32, device=dev)
    b = fp4.reshape(rows_pad, k_pad // 2).to(torch.int64)
    vals = torch.stack([lut[b & 0xF], lut[b >> 4]], dim=-1).reshape(rows_pad, k_pad)
    # UE4M3 decode of all 256 byte values: (8 + m) * 2^(e - 10), subnormal m * 2^-9
    codes = torch.arange(256, device=dev)
    e, m = (codes >> 3) & 0xF, (codes & 7).to(torch.float32)
    dec = torch.where(e == 0, m * 2.0 ** -9, (8 + m) * torch.pow(2.0, (e - 10).to(torch.float32)))
    nsb = k_pad // 16
    r = torch.arange(rows_pad, device=dev).unsqueeze(1)
    kb = torch.arange(nsb, device=dev).unsqueeze(0)
    off = (r % 32) * 16 + ((r // 32) % 4) * 4 + (kb % 4) + (kb // 4) * 512 + (r // 128) * 512 * (nsb // 4)
    scale = dec[sf.reshape(-1).to(torch.int64)[off]]  # [rows_pad, nsb]
    return vals * scale.repeat_interleave(16, dim=1)
