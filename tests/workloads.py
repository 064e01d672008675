"""Seeded synthetic inputs shared by the tests and bench.py.

The reference measures on no public dataset; these generators produce the
shapes and value distributions BASELINE.json names for each config, on the
CPU from fixed seeds, so the oracle and the GPU see identical BF16 bytes.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch

# (M, N, K) of the cached-linear sweep; the metric is quoted on 2048x2880x7680.
CACHED_SHAPES = [(512, 2880, 2880), (2048, 2880, 7680), (2048, 7680, 2880), (4096, 2880, 2880)]
HEADLINE_SHAPE = (2048, 2880, 7680)
CFG1_SHAPE = (256, 2880, 2880)


def normal_bf16(shape, std: float, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g, dtype=torch.float32) * std).to(torch.bfloat16)


def cached_linear_inputs(m: int, n: int, k: int, seed: int = 0, bias: bool = True):
    """Activations ~N(0,1) [m,k], weights ~N(0,0.02) [n,k], bias ~N(0,0.01) [n] (CPU, bf16)."""
    x = normal_bf16((m, k), 1.0, seed)
    w = normal_bf16((n, k), 0.02, seed + 1)
    b = normal_bf16((n,), 0.01, seed + 2) if bias else None
    return x, w, b


def quantizer_stress(rows: int, cols: int, seed: int = 0, outlier_frac: float = 1e-3,
                     zero_block_frac: float = 1e-2, chunk_rows: int = 512) -> torch.Tensor:
    """Config 4 input: 0.5 * Student-t(df=3), then +-400 at `outlier_frac` of the
    positions and all-zero 16-element blocks at `zero_block_frac` of the blocks
    (positions sampled without replacement; zero blocks applied last).

    Row chunks draw from independent child generators of SeedSequence(seed), so
    the result does not depend on how many threads fill them."""
    assert cols % 16 == 0
    n_chunks = (rows + chunk_rows - 1) // chunk_rows
    children = np.random.SeedSequence(seed).spawn(n_chunks + 1)
    x = np.empty((rows, cols), dtype=np.float32)

    def fill(i):
        r0, r1 = i * chunk_rows, min(rows, (i + 1) * chunk_rows)
        x[r0:r1] = 0.5 * np.random.default_rng(children[i]).standard_t(3, size=(r1 - r0, cols))

    with ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 1)) as ex:
        list(ex.map(fill, range(n_chunks)))
    rng = np.random.default_rng(children[-1])
    flat = x.reshape(-1)
    n_out = int(round(outlier_frac * flat.size))
    if n_out:
        pos = rng.choice(flat.size, size=n_out, replace=False)
        flat[pos] = np.where(rng.random(n_out) < 0.5, -400.0, 400.0).astype(np.float32)
    blocks = flat.reshape(-1, 16)
    n_zero = int(round(zero_block_frac * blocks.shape[0]))
    if n_zero:
        blocks[rng.choice(blocks.shape[0], size=n_zero, replace=False)] = 0.0
    return torch.from_numpy(x).to(torch.bfloat16)


def subnormal_scale_rows(rows: int, cols: int, seed: int = 0) -> torch.Tensor:
    """Blocks whose |x|max lies in [0.0117, 0.094): UE4M3 scales in the truncated subnormal range."""
    rng = np.random.default_rng(seed)
    amax = rng.uniform(0.0117, 0.094, size=(rows, cols // 16, 1)).astype(np.float32)
    v = rng.uniform(-1.0, 1.0, size=(rows, cols // 16, 16)).astype(np.float32)
    v /= np.maximum(np.abs(v).max(axis=2, keepdims=True), 1e-30)
    return torch.from_numpy((v * amax).reshape(rows, cols)).to(torch.bfloat16)
