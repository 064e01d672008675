"""CPU checks of the arithmetic the GPU quantizer relies on (no GPU needed).

The sm_100a quantizer replaces the reference's per-element nearest-value scan
(fp4_gemm_lib.cu:110-124) with a lookup on the fp32 bit pattern (of 16 * v,
with the slot index of negative values moved to other shared-memory banks),
reads the scale byte from a table over the block |x|max, and divides by the
row length with a multiply-shift.  These tests
restate each in numpy and compare them with the oracle / IEEE results.
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


def banked_index_np(bits16: np.ndarray) -> np.ndarray:
    t = (bits16.astype(np.uint64) + 0xFFFFFFFF) & 0xFFFFFFFF  # bits - 1 in uint32
    return ((t ^ ((t >> 4) & 0x08000000)) >> 21).astype(np.int64)


def banked_table_np() -> np.ndarray:
    i = np.arange(2048, dtype=np.uint64)
    t = i ^ ((i >> 10) << 6)
    tops = ((t + 1) << 21).astype(np.uint32)  # (2047 + 1) << 21 wraps to +0
    with np.errstate(invalid="ignore"):  # the NaN slots (exponent 255) stay NaN
        return scan_np(tops.view(np.float32) * np.float32(0.03125))


def test_banked_table_of_32v_equals_scan_below_2p23():
    tab = banked_table_np()
    rng = np.random.default_rng(11)
    limit = np.uint32(0x4B000000)  # 2^23
    edges = (np.arange(1, int(limit >> 21) + 1, dtype=np.uint64) << 21).astype(np.uint32)
    pats = np.concatenate([edges, edges - 1, edges + 1, rng.integers(0, int(limit), 2_000_000, dtype=np.uint32),
                           np.array([0, 1, 2, 0x00800000, 0x007FFFFF], dtype=np.uint32)])
    pats = pats[pats < limit]
    pats = np.concatenate([pats, pats | np.uint32(0x80000000)])
    v = pats.view(np.float32)
    with np.errstate(over="ignore"):
        v32 = (v * np.float32(32)).astype(np.float32)  # exact: a power-of-two factor, no overflow
    assert np.array_equal(v32 / np.float32(32), v)
    got = tab[banked_index_np(v32.view(np.uint32))]
    assert np.array_equal(got, scan_np(v))
    # +0 -> 0, -0 -> 0, tiny negative -> 8 (sign for any value < 0)
    special = np.array([0.0, -0.0, -1e-30, 1e-30, -2.0 ** -140], dtype=np.float32)
    got = tab[banked_index_np((special * np.float32(32)).view(np.uint32))]
    assert got.tolist() == [0, 0, 8, 0, 8]


def test_banked_index_spreads_active_slots_over_banks():
    # the slots of |v| in (2^-4, 8) (every nonzero code and the band below),
    # both signs, and +-0 lie in pairwise distinct 4-byte words on distinct banks
    vals = np.array([s * m * 2.0 ** e for s in (1, -1) for e in range(-4, 3) for m in (1.0, 1.25, 1.5, 1.75)]
                    + [0.0, -0.0], dtype=np.float32)
    vals = vals[np.abs(vals) != 2.0 ** -4]
    words = banked_index_np((vals * np.float32(32)).view(np.uint32)) >> 2
    uniq = np.unique(words)
    assert len(np.unique(uniq % 32)) == len(uniq)


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


def test_scale_table_matches_oracle_for_every_fast_path_absmax():
    # The GPU kernel reads the scale byte from a table over the |x|max bit
    # patterns [0x3C40, 0x4E80) built as ue4m3(absmax / 6) in IEEE fp32, and
    # uses 0x01 below 0x3C40.  Check both against the oracle quantizer on
    # blocks whose largest element is each of those values.
    bits = np.arange(0, 0x4E80, dtype=np.uint32)
    amax = (bits << 16).view(np.float32)
    ieee = (amax / np.float32(6)).astype(np.float32)
    assert np.all(ieee[bits < 0x3C40] <= np.float32(2.0 ** -9))
    table = np.array([O.ue4m3_encode(float(x)) for x in ieee[0x3C40:]], dtype=np.uint8)
    rows = O.round_up(len(bits), 128)
    x = np.zeros((rows, 128), dtype=np.float32)
    x[: len(bits), 0] = amax
    x[: len(bits), 5] = -amax / 3  # another element, smaller in magnitude
    fp4, sf = O.quantize(O.f32_to_bf16_bits(x), rows, 128)
    got = np.array([sf[O.sf_index(r, 0, 8)] for r in range(len(bits))], dtype=np.uint8)
    assert np.all(got[:0x3C40] == 0x01)
    assert np.array_equal(got[0x3C40:], table)
