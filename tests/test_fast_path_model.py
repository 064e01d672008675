"""CPU checks of the arithmetic the GPU quantizer relies on (no GPU needed).

The sm_100a quantizer replaces the reference's per-element nearest-value scan
(fp4_gemm_lib.cu:110-124) with a lookup on the fp32 bit pattern, and divides
by the row length with a multiply-shift.  These tests restate both in numpy
and compare them with the oracle on many inputs.
"""
import numpy as np

from oracle import nvfp4_oracle as O

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def scan_np(v: np.ndarray) -> np.ndarray:
    """Vectorised restatement of the reference scan in float32 arithmetic."""
    v = v.astype(np.float32)
    a = np.abs(v)
    best = a.copy()
    code = np.zeros(v.shape, dtype=np.uint8)
    with np.errstate(invalid="ignore"):
        for i in range(1, 8):
            d = np.abs(a - E2M1[i])
            better = d < best
            best = np.where(better, d, best)
            code = np.where(better, np.uint8(i), code)
        sign = np.where(v < 0, np.uint8(8), np.uint8(0))
    return (code | sign).astype(np.uint8)


def table_np() -> np.ndarray:
    """The 2048-entry table of the GPU kernel: code of the top pattern of each 2^21 slot."""
    tops = ((np.arange(2048, dtype=np.uint64) + 1) << 21).astype(np.uint32)
    return scan_np(tops.view(np.float32))


def test_scan_restatement_matches_oracle():
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(3000) * 4, [0.25, 0.75, 1.75, 3.5, 5.0, -0.0, np.inf, np.nan, 1e30]])
    v = v.astype(np.float32)
    assert np.array_equal(scan_np(v), np.array([O.e2m1_code(float(x)) for x in v], dtype=np.uint8))


def test_slot_table_equals_scan_below_2p23():
    tab = table_np()
    rng = np.random.default_rng(1)
    # every slot boundary +-1 ulp and random patterns, both signs, |v| < 2^23
    limit = np.uint32(0x4B000000)
    edges = (np.arange(1, int(limit >> 21) + 1, dtype=np.uint64) << 21).astype(np.uint32)
    pats = np.concatenate([edges, edges - 1, edges + 1, rng.integers(0, int(limit), 2_000_000, dtype=np.uint32),
                           np.array([0, 1, 2], dtype=np.uint32)])
    pats = pats[pats < limit]
    pats = np.concatenate([pats, pats | np.uint32(0x80000000)])
    v = pats.view(np.float32)
    idx = ((pats.astype(np.uint64) + 0xFFFFFFFF) & 0xFFFFFFFF) >> 21  # (bits - 1) >> 21 in uint32
    assert np.array_equal(tab[idx.astype(np.int64)], scan_np(v))


def test_fast_path_bound_keeps_scaled_values_below_2p23():
    # Blocks with |x|max < 2^30 (bf16 0x4E80) never produce |x * inv| >= 2^23.
    rng = np.random.default_rng(2)
    amax = np.concatenate([10.0 ** rng.uniform(-45, 9.03, 200000), [2.0 ** 30 - 2.0 ** 22, 1536.0, 2880.0, 0.0]])
    bits = O.f32_to_bf16_bits(amax.astype(np.float32))
    bits = bits[bits < 0x4E80]
    a = O.bits_to_f32(bits)
    s = np.maximum(a / np.float32(6.0), np.float32(2.0 ** -9)).astype(np.float32)
    inv = np.array([np.float32(1.0) / np.float32(O.ue4m3_decode(O.ue4m3_encode(float(x)))) for x in s[:20000]])
    assert np.all(a[:20000] * inv < 2.0 ** 23)


def fast_div(n: np.ndarray, d: int) -> np.ndarray:
    s = 0
    while (1 << s) < d:
        s += 1
    mul = ((1 << 32) * ((1 << s) - d)) // d + 1
    hi = (n.astype(np.uint64) * np.uint64(mul)) >> np.uint64(32)
    return ((hi + n.astype(np.uint64)) >> np.uint64(s)).astype(np.int64)


def test_fast_division_exact():
    rng = np.random.default_rng(3)
    for d in [8, 16, 24, 184, 480, 1024, 7, 1, 3 * 5 * 7 * 11, 65536, 123457]:
        n = np.concatenate([rng.integers(0, 2 ** 31 - 1, 100000), np.arange(0, 4 * d), [2 ** 31 - 1]])
        assert np.array_equal(fast_div(n, d), n // d), d


def test_scale_layout_is_bijective():
    for rows, k in [(128, 128), (256, 384), (384, 2944)]:
        nsb = k // 16
        offs = {O.sf_index(r, kb, nsb) for r in range(rows) for kb in range(nsb)}
        assert offs == set(range(rows * nsb))


def test_division_table_matches_ieee_for_every_bf16_absmax():
    # The GPU kernel forms RN(absmax / 6) as RN((128 + m) / 6) * 2^(E - 134) for
    # every fast-path |x|max (bf16 bits below 0x4E80) at or above 6 * 2^-9, and
    # uses scale byte 0x01 below; the reference divides in IEEE fp32.
    bits = np.arange(0, 0x4E80, dtype=np.uint32)
    amax = (bits << 16).view(np.float32)
    div6 = (np.arange(128, dtype=np.float32) + np.float32(128)) / np.float32(6)
    hi = bits >= 0x3C40
    e = (bits >> 7).astype(np.int64)
    table = (div6.view(np.uint32)[bits & 0x7F].astype(np.int64) + ((e - 134) << 23)).astype(np.uint32)
    ieee = (amax / np.float32(6)).astype(np.float32)
    assert np.array_equal(table[hi].view(np.float32), ieee[hi])
    assert np.all(ieee[~hi] <= np.float32(2.0 ** -9))
    # and the resulting scale bytes, through the oracle's encoder
    s_ref = np.maximum(ieee, np.float32(2.0 ** -9))
    sample = np.concatenate([np.arange(0, 0x4E80, 7), [0x3C3F, 0x3C40, 0x3C41, 0x4E7F]])
    for b in sample:
        want = O.ue4m3_encode(float(s_ref[b]))
        got = 0x01 if b < 0x3C40 else O.ue4m3_encode(float(table[b].view(np.float32)))
        assert got == want, hex(b)
