"""sm_100a quantizer vs the golden vectors and the oracle: bit-exact bytes.

Covers the reference kernel's semantics (fp4_gemm_lib.cu:241-286) on hand-built
corner blocks, seeded tensors, ragged and unaligned inputs, and the full-size
config-4 stress tensor (16384 x 16384, compared by SHA-256 with the bytes the
reference's own quantizer produced).
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from tests import workloads as W
from tests.gpu_helpers import oracle_quantize, to_numpy_u8

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def bits_to_cuda_bf16(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(dev)


def gpu_quantize(fp4mod, x, rows_pad=None, k_pad=None):
    fp4, sf = fp4mod.quantize_to_buffers(x, rows_pad, k_pad)
    torch.cuda.synchronize()
    return to_numpy_u8(fp4), to_numpy_u8(sf)


def test_block_kats(cuda, fp4):
    k = np.load(os.path.join(GOLDEN, "kat_blocks.npz"))
    q, s = gpu_quantize(fp4, bits_to_cuda_bf16(k["x_bits"], cuda))
    assert np.array_equal(s, k["sf"]), f"scale bytes differ at {np.nonzero(s != k['sf'])[0][:10]}"
    assert np.array_equal(q, k["fp4"]), f"fp4 bytes differ at {np.argwhere(q != k['fp4'])[:10]}"


@pytest.mark.parametrize("name", ["normal", "weight", "stress", "subnormal", "ragged"])
def test_tensor_fixtures(cuda, fp4, name):
    t = np.load(os.path.join(GOLDEN, "tensors.npz"))
    x = bits_to_cuda_bf16(t[f"{name}_x"], cuda)  # unpadded: the kernel zero-pads itself
    q, s = gpu_quantize(fp4, x)
    assert np.array_equal(q, t[f"{name}_fp4"])
    assert np.array_equal(s, t[f"{name}_sf"])


@pytest.mark.parametrize("rows,cols", [(1, 16), (1, 7), (127, 128), (128, 100), (300, 2880), (129, 7680),
                                       (256, 4), (200, 1000)])
def test_random_shapes_vs_oracle(cuda, fp4, rows, cols):
    g = torch.Generator().manual_seed(rows * 7919 + cols)
    x = (torch.randn(rows, cols, generator=g) * torch.logspace(-3, 3, rows).unsqueeze(1)).to(torch.bfloat16)
    q, s = gpu_quantize(fp4, x.to(cuda))
    rq, rs = oracle_quantize(x)
    assert np.array_equal(q, rq) and np.array_equal(s, rs)


def test_strided_and_unaligned_rows(cuda, fp4):
    # Row stride 1000 elements; column offsets 8 (16-byte aligned), 1 and 5 (unaligned).
    g = torch.Generator().manual_seed(5)
    big = torch.randn(256, 1000, generator=g).to(torch.bfloat16)
    big_d = big.to(cuda)
    for rs_, cs_ in ((slice(0, 256), slice(8, 520)), (slice(0, 256), slice(1, 513)), (slice(3, 200), slice(5, 700))):
        q, s = gpu_quantize(fp4, big_d[rs_, cs_])
        rq, rsf = oracle_quantize(big[rs_, cs_].contiguous())
        assert np.array_equal(q, rq) and np.array_equal(s, rsf)


def test_explicit_padding(cuda, fp4):
    x = W.normal_bf16((100, 200), 1.0, 11)
    q, s = gpu_quantize(fp4, x.to(cuda), 384, 512)
    rq, rs = oracle_quantize(x, 384, 512)
    assert np.array_equal(q, rq) and np.array_equal(s, rs)
    assert np.all(rs[O.sf_index(300, 20, 32)] == 0x01)  # zero padding -> scale 0x01


def test_config4_full_size_digest(cuda, fp4):
    want = json.load(open(os.path.join(GOLDEN, "digests.json")))["cfg4_stress_16384x16384_seed0"]
    x = W.quantizer_stress(16384, 16384, seed=0).to(cuda)
    fq, fs = fp4.quantize_to_buffers(x)
    torch.cuda.synchronize()
    got_q = hashlib.sha256(fq.cpu().numpy().tobytes()).hexdigest()
    got_s = hashlib.sha256(fs.cpu().numpy().tobytes()).hexdigest()
    assert got_s == want["sf"], "config-4 scale bytes differ from the reference's"
    assert got_q == want["fp4"], "config-4 fp4 bytes differ from the reference's"


def test_idempotent_and_deterministic(cuda, fp4):
    x = W.quantizer_stress(512, 2048, seed=3).to(cuda)
    a = fp4.quantize_to_buffers(x)
    b = fp4.quantize_to_buffers(x)
    torch.cuda.synchronize()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
