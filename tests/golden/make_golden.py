"""Generate the golden vectors in tests/golden/ from the reference's own code.

Run in a container that has the reference checkout (it is not needed on the GPU
box, which only reads the committed fixtures):

    python oracle/build.py            # builds oracle/_ref/libref_quant.so
    python tests/golden/make_golden.py

Every output here is produced by ``oracle/_ref/libref_quant.so``, i.e. by the
reference's quantizer source (fp4_gemm_lib.cu:106-286 of
VincentKaufmann/fp4-gemm-blackwell) compiled for the host, never by this
project's code.  Files:

* ``kat_scalars.npz``  -- E2M1 codes, UE4M3 encodes/decodes and scale-layout
  offsets for hand-picked and random inputs (d_float_to_fp4,
  d_float_to_ue4m3, d_ue4m3_to_float, compute_sf_index);
* ``kat_blocks.npz``   -- a 128 x 256 BF16 matrix of hand-built 16-element
  blocks (ties, zero / subnormal / saturated / carried scales, negative zero,
  tiny negatives, NaN / Inf, huge values) with the quantized bytes;
* ``tensors.npz``      -- seeded matrices (normal activations, N(0,0.02)
  weights, the config-4 stress distribution, truncated-subnormal scales, and
  a ragged 200 x 300 matrix zero-padded to 256 x 384 as fp4_gemm.py pads it);
* ``digests.json``     -- SHA-256 of the reference quantizer's bytes on
  full-size inputs from tests/workloads.py (config 4: 16384 x 16384; the
  padded 2944-row weights of configs 1 and 2).
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import build as oracle_build  # noqa: E402
from oracle import nvfp4_oracle as O  # noqa: E402
from tests import workloads as W  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def scalar_kats(R):
    rng = np.random.default_rng(1234)
    special = np.array([0.0, -0.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 6.5, 7.0, 12.0,
                        0.2499999, 0.2500001, 0.7499999, 0.7500001, 1.2499999, 1.2500001, 1.7499999, 1.7500001,
                        2.4999998, 2.5000002, 3.4999998, 3.5000002, 4.9999995, 5.0000005,
                        1e-30, -1e-30, -1e-5, 1e-45, -1e-45, np.inf, -np.inf, np.nan, -np.nan,
                        2.0 ** 22, 2.0 ** 23, 2.0 ** 23 + 1, 2.0 ** 24, 2.0 ** 24 + 2, 2.0 ** 26 + 4, 2.0 ** 26 + 8,
                        2.0 ** 27, 3e38, -3e38, 1e35], dtype=np.float32)
    rnd = np.concatenate([rng.standard_normal(4000) * 3, rng.uniform(-8, 8, 4000),
                          np.sign(rng.standard_normal(500)) * 10.0 ** rng.uniform(-8, 12, 500)]).astype(np.float32)
    e2m1_in = np.concatenate([special, -special, rnd]).astype(np.float32)
    e2m1_out = np.array([R.ref_float_to_fp4(float(v)) for v in e2m1_in], dtype=np.uint8)

    s_special = np.array([0.0, 1e-10, 1.953125e-3, 1.9e-3, 2.0e-3, 0.0039, 0.015625, 0.0156, 0.0157, 0.5, 1.0,
                          1.0625, 1.0624, 1.9375, 1.96875, 1.99, 15.9, 31.5, 127.9, 255.0, 255.9, 256.0, 300.0,
                          448.0, 480.0, 481.0, 1e6, np.inf, 2.0 ** -7, 2.0 ** -8, 3 * 2.0 ** -9,
                          7.5 * 2.0 ** -9], dtype=np.float32)
    s_rnd = (np.abs(rng.standard_normal(3000)) * 10.0 ** rng.uniform(-4, 3, 3000)).astype(np.float32)
    ue_in = np.concatenate([s_special, s_rnd]).astype(np.float32)
    ue_out = np.array([R.ref_float_to_ue4m3(float(v)) for v in ue_in], dtype=np.uint8)
    dec_out = np.array([R.ref_ue4m3_to_float(b) for b in range(256)], dtype=np.float32)

    sf_cases = []
    for nsb in (8, 16, 24, 184, 480):
        for r in list(range(0, 300, 7)) + [127, 128, 129, 255, 256]:
            for kb in sorted({0, 1, 3, 4, 5, 7, nsb - 1}):
                sf_cases.append((r, kb, 512, nsb))
    sf_cases = np.array(sf_cases, dtype=np.int64)
    sf_out = np.array([R.ref_sf_index(int(r), int(kb), int(rows), int(nsb)) for r, kb, rows, nsb in sf_cases],
                      dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "kat_scalars.npz"), e2m1_in=e2m1_in, e2m1_out=e2m1_out, ue4m3_in=ue_in,
                        ue4m3_out=ue_out, ue4m3_decode=dec_out, sf_cases=sf_cases, sf_out=sf_out)


def designed_blocks() -> list[np.ndarray]:
    """16-element blocks that hit every rounding and scale corner of the reference."""
    ties = np.array([6, .25, .75, 1.25, 1.75, 2.5, 3.5, 5, -.25, -.75, -1.25, -1.75, -2.5, -3.5, -5, -6], np.float32)
    b = [ties, ties * 2, ties * 0.5, ties * 4, ties * 0.125,
         np.zeros(16, np.float32), np.full(16, -0.0, np.float32),
         np.concatenate([[0.05], np.linspace(-0.05, 0.04, 15)]).astype(np.float32),   # subnormal scale
         np.concatenate([[0.0117], np.linspace(-0.01, 0.011, 15)]).astype(np.float32),
         np.full(16, 0.01171875, np.float32),                                        # 6 * 2^-9 exactly
         np.concatenate([[2000.0], np.linspace(-1900, 1500, 15)]).astype(np.float32),  # scale >= 256 -> 0x7F
         np.concatenate([[2880.0], np.linspace(-2000, 100, 15)]).astype(np.float32),
         np.concatenate([[1535.0], np.linspace(-1000, 1000, 15)]).astype(np.float32),
         np.concatenate([[6.0], np.full(15, -1e-5)]).astype(np.float32),               # tiny negatives
         np.concatenate([[11.76], np.linspace(-11, 11, 15)]).astype(np.float32),       # mantissa carry
         np.concatenate([[1535.9], np.linspace(-11, 11, 15)]).astype(np.float32),      # carry into 0x78
         np.array([1.0, np.nan, 2.0, -np.nan, 3.0, 0.5, -0.5, 1.5] * 2, np.float32),
         np.array([1.0, np.inf, 2.0, -3.0, 4.0, -np.inf, 0.25, 1.0] * 2, np.float32),
         np.array([1e35, -1e35, 1e30, 3e9, -3e9, 1.0, 2.0 ** 31, 2.0 ** 30] * 2, np.float32),
         np.array([3.3e38, -3.3e38, 1.0, -1.0, 1e38, 0.0, 5e37, -2e38] * 2, np.float32),
         np.array([2.0 ** 30, 2.0 ** 30 - 1e3, 1.0, -1.0, 2.0 ** 29, 5e8, -6e8, 7e8] * 2, np.float32),
         np.array([4.5, 0.375, 0.5625, 0.9375, 1.3125, 1.875, 2.625, 3.75] * 2, np.float32),  # scale 0.75
         np.full(16, 1.0, np.float32), np.full(16, -7.0, np.float32),
         (np.arange(16, dtype=np.float32) - 8) * 1e-39,                               # bf16 subnormals
         np.array([1e-38, -2e-38, 3e-39, 0.0] * 4, np.float32)]
    return b


def block_kats():
    rng = np.random.default_rng(99)
    rows, cols = 128, 256
    nb = rows * cols // 16
    designed = designed_blocks()
    blocks = []
    for i in range(nb):
        if i < len(designed) * 4:
            base = designed[i % len(designed)]
            scale = [1.0, 2.0 ** rng.integers(-6, 7), -1.0, float(rng.uniform(0.1, 10))][i // len(designed)]
            with np.errstate(over="ignore"):  # scaled huge values may become +-Inf on purpose
                blocks.append((base * np.float32(scale)).astype(np.float32))
        else:
            sigma = 10.0 ** rng.uniform(-4, 4)
            blocks.append((rng.standard_normal(16) * sigma).astype(np.float32))
    x = np.stack(blocks).reshape(rows, cols)
    bits = O.f32_to_bf16_bits(x)
    fp4, sf = O.ref_quantize(bits)
    np.savez_compressed(os.path.join(HERE, "kat_blocks.npz"), x_bits=bits, fp4=fp4, sf=sf)


def tensor_fixtures():
    out = {}

    def add(name, t, rows_pad=None, k_pad=None):
        bits = O.bf16_bits(t)
        rows, cols = bits.shape
        rp = rows_pad or O.round_up(rows, 128)
        kp = k_pad or O.round_up(cols, 128)
        padded = np.zeros((rp, kp), dtype=np.uint16)  # torch.zeros padding of fp4_gemm.py:296-309
        padded[:rows, :cols] = bits
        fp4, sf = O.ref_quantize(padded)
        out[f"{name}_x"] = bits
        out[f"{name}_fp4"] = fp4
        out[f"{name}_sf"] = sf

    add("normal", W.normal_bf16((256, 512), 1.0, 0))
    add("weight", W.normal_bf16((128, 256), 0.02, 1))
    add("stress", W.quantizer_stress(256, 1024, seed=2, outlier_frac=1e-2, zero_block_frac=5e-2))
    add("subnormal", W.subnormal_scale_rows(128, 512, seed=3))
    add("ragged", W.normal_bf16((200, 300), 1.0, 4))
    np.savez_compressed(os.path.join(HERE, "tensors.npz"), **out)


def digests():
    d = {}
    x = W.quantizer_stress(16384, 16384, seed=0)
    fp4, sf = O.ref_quantize(x)
    d["cfg4_stress_16384x16384_seed0"] = {"fp4": sha(fp4), "sf": sha(sf)}
    for name, (n, k) in {"cfg1_weight_2880x2880_seed1": (2880, 2880),
                         "cfg2_weight_2880x7680_seed1": (2880, 7680)}.items():
        w = W.normal_bf16((n, k), 0.02, 1)
        padded = np.zeros((O.round_up(n, 128), O.round_up(k, 128)), dtype=np.uint16)
        padded[:n, :k] = O.bf16_bits(w)
        fp4, sf = O.ref_quantize(padded)
        d[name] = {"fp4": sha(fp4), "sf": sha(sf)}
    with open(os.path.join(HERE, "digests.json"), "w") as f:
        json.dump(d, f, indent=1, sort_keys=True)


def main():
    if oracle_build.build_ref() is None:
        raise SystemExit("reference checkout not found; cannot generate golden vectors")
    R = O.ref_lib()
    torch.manual_seed(0)
    scalar_kats(R)
    block_kats()
    tensor_fixtures()
    digests()
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
