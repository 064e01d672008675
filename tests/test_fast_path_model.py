"""CPU checks of the arithmetic the GPU quantizer relies on (no GPU needed).

The sm_100a quantizer replaces the reference's per-element nearest-value scan
(fp4_gemm_lib.cu:110-124) with the hardware round-to-nearest-even conversion
applied to a stand-in for each scaled value, reads the scale byte from a table
over the block |x|max, and divides by the row length with a multiply-shift.
These tests restate each in numpy and compare them with the oracle / IEEE
results.
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


def test_scan_restatement_matches_oracle():
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(3000) * 4, [0.25, 0.75, 1.75, 3.5, 5.0, -0.0, np.inf, np.nan, 1e30]])
    v = v.astype(np.float32)
    assert np.array_equal(scan_np(v), np.array([O.e2m1_code(float(x)) for x in v], dtype=np.uint8))


TINY = np.float32(2.0 ** -149)


def stand_in_bits(v: np.ndarray) -> np.ndarray:
    """The GPU quantizer's stand-in for an already rounded v = RN(x * inv):
    v' = RN(v + 2^-149) (the kernel forms RN(x * inv + 2^-149) in one fma; for a
    v that is not a zero nor within 2^-142 of one, adding 2^-149 to v or to the
    exact product rounds alike except at exact midpoints, which
    test_denormal_addend_changes_no_code covers), then (b - 1) | 1 on the bits."""
    with np.errstate(over="ignore"):
        vp = (v.astype(np.float32) + TINY).astype(np.float32)
    b = vp.view(np.uint32).copy()
    return ((b - np.uint32(1)) | np.uint32(1)).astype(np.uint32)


def reachable(pats: np.ndarray) -> np.ndarray:
    """Scaled values the fast path can produce: zeros and |v| >= 2^-142 (a BF16
    x is 0 or at least 2^-133 in magnitude, 1 / scale at least 1/480)."""
    mag = pats & np.uint32(0x7FFFFFFF)
    return pats[(mag == 0) | (mag >= np.float32(2.0 ** -142).view(np.uint32))]


def e2m1_rne_np(bits: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even onto E2M1 with saturation, as cvt.rn.satfinite.e2m1x2
    does, for inputs that are never exactly halfway (asserted): the sign bit of
    the input and the nearest magnitude code."""
    v = bits.view(np.float32).astype(np.float64)
    a = np.abs(v)
    d = np.abs(a[:, None] - E2M1.astype(np.float64)[None, :])
    code = np.argmin(d, axis=1)
    srt = np.sort(d, axis=1)
    assert np.all(srt[:, 0] < srt[:, 1]), "a stand-in is halfway between two E2M1 values"
    sign = np.where(bits >= np.uint32(0x80000000), 8, 0)
    return (code | sign).astype(np.uint8)


def test_hardware_rounding_of_stand_in_equals_scan():
    rng = np.random.default_rng(1)
    limit = np.uint32(0x4B000000)  # 2^23; beyond it every value saturates to code 7
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32).view(np.uint32)
    edges = (np.arange(1, int(limit >> 21) + 1, dtype=np.uint64) << 21).astype(np.uint32)
    pats = np.concatenate([edges, edges - 1, edges + 1, ties, ties - 1, ties + 1,
                           rng.integers(0, int(limit), 1_000_000, dtype=np.uint32),
                           np.array([0, 1, 2, 3, 0x00800000, 0x007FFFFF, 0x4AFFFFFF], dtype=np.uint32)])
    pats = pats[pats < limit]
    pats = reachable(np.concatenate([pats, pats | np.uint32(0x80000000)]))
    v = pats.view(np.float32)
    assert np.array_equal(e2m1_rne_np(stand_in_bits(v)), scan_np(v))


def test_stand_in_special_values():
    # +0 and -0 -> code 0; any value < 0 keeps the sign, even when it rounds to 0;
    # the halfway values go to the lower magnitude (0.75 -> 0.5, 1.75 -> 1.5, 3.5 -> 3).
    v = np.array([0.0, -0.0, 1e-30, -1e-30, -2.0 ** -140, 0.75, -0.75, 1.75, 3.5, -3.5, 5.0, 0.25, 1.25, 2.5,
                  6.0, 7.0, 1e6], dtype=np.float32)
    assert len(reachable(v.view(np.uint32))) == len(v)
    got = e2m1_rne_np(stand_in_bits(v))
    assert got.tolist() == [0, 0, 0, 8, 8, 1, 9, 3, 5, 13, 6, 0, 2, 4, 7, 7, 7]
    assert np.array_equal(got, scan_np(v))


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


def ue4m3_value(b: int) -> float:
    e, m = (b >> 3) & 0xF, b & 7
    return m * 2.0 ** -9 if e == 0 else (8 + m) * 2.0 ** (e - 10)


def test_denormal_addend_changes_no_code():
    # The kernel scales with fma(x, inv, 2^-149) instead of x * inv.  For every
    # fast-path BF16 x (finite, |x| < 2^30, non-zero) and every reciprocal
    # inv = RN(1 / ue4m3(s)), the product x * inv is exact in float64; where it
    # is exactly halfway between two floats, RN(x * inv) picks the even one
    # while the addend pushes positive products to the larger and negative
    # ones to the smaller magnitude.  Both must have the same reference code.
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])

    def code(v):
        return np.searchsorted(mids, np.abs(v), side="left") + np.where(v < 0, 8, 0)

    bits = np.arange(65536, dtype=np.uint32)
    with np.errstate(invalid="ignore"):
        x = (bits << 16).view(np.float32).astype(np.float64)
    x = x[np.isfinite(x) & (np.abs(x) < 2.0 ** 30) & (x != 0)]
    assert np.abs(x).min() * (1.0 / 480.0) >= 2.0 ** -142
    halfway = 0
    for s in range(1, 128):
        inv = np.float64(np.float32(1.0) / np.float32(ue4m3_value(s)))
        p = x * inv
        b = p.view(np.uint64)
        normal = ((b >> np.uint64(52)) & np.uint64(0x7FF)).astype(np.int64) - 1023 >= -126
        mid = normal & ((b & np.uint64((1 << 29) - 1)) == np.uint64(1 << 28))
        if not mid.any():
            continue
        pm = p[mid]
        below = (pm.view(np.uint64) & ~np.uint64((1 << 29) - 1)).view(np.float64)  # toward zero
        above = below + 2 * (pm - below)                                         # away from zero
        with_addend = np.where(pm > 0, above, below)
        rne = pm.astype(np.float32).astype(np.float64)
        assert np.array_equal(code(rne), code(with_addend)), f"scale byte {s}"
        halfway += int(mid.sum())
    assert halfway > 0  # the case does occur
