"""The CPU oracle against the golden vectors made by the reference's own quantizer.

These pin oracle/nvfp4_oracle.c (the checker every GPU parity test uses) to
fp4_gemm_lib.cu:106-286 of the reference: scalar codecs, the scale layout,
hand-built corner blocks, seeded tensors and full-size digests.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import nvfp4_oracle as O
from tests import workloads as W

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_e2m1_codes_match_reference():
    k = _load("kat_scalars.npz")
    got = np.array([O.e2m1_code(float(v)) for v in k["e2m1_in"]], dtype=np.uint8)
    bad = np.nonzero(got != k["e2m1_out"])[0]
    assert bad.size == 0, f"mismatch at inputs {k['e2m1_in'][bad[:8]]}: {got[bad[:8]]} vs {k['e2m1_out'][bad[:8]]}"


def test_e2m1_ties_go_low():
    # fp4_gemm_lib.cu:116-121: strict '<' keeps the lower code on a tie (not RNE).
    assert [O.e2m1_code(v) for v in (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)] == [0, 1, 2, 3, 4, 5, 6]
    assert O.e2m1_code(-1e-5) == 0x8 and O.e2m1_code(-0.0) == 0x0
    assert O.e2m1_code(float("nan")) == 0 and O.e2m1_code(float("inf")) == 0 and O.e2m1_code(7.0) == 7


def test_ue4m3_encode_decode_match_reference():
    k = _load("kat_scalars.npz")
    got = np.array([O.ue4m3_encode(float(v)) for v in k["ue4m3_in"]], dtype=np.uint8)
    assert np.array_equal(got, k["ue4m3_out"])
    dec = np.array([O.ue4m3_decode(b) for b in range(256)], dtype=np.float32)
    assert np.array_equal(dec.view(np.uint32), k["ue4m3_decode"].view(np.uint32))


def test_ue4m3_corners():
    assert O.ue4m3_encode(0.0) == 0x01            # clamp to 2^-9: zero blocks get 0x01, never 0x00
    assert O.ue4m3_encode(300.0) == 0x7F          # exponent >= 15 saturates
    assert O.ue4m3_encode(255.9) == 0x78          # mantissa carry into exponent 15
    assert O.ue4m3_decode(0x7F) == 480.0
    assert O.ue4m3_encode(3.5 * 2 ** -9) == 0x03  # subnormal mantissa truncates


def test_sf_index_matches_reference():
    k = _load("kat_scalars.npz")
    got = np.array([O.sf_index(int(r), int(kb), int(nsb)) for r, kb, _rows, nsb in k["sf_cases"]])
    assert np.array_equal(got, k["sf_out"])


def test_block_kats_match_reference():
    k = _load("kat_blocks.npz")
    fp4, sf = O.quantize(k["x_bits"])
    assert np.array_equal(fp4, k["fp4"])
    assert np.array_equal(sf, k["sf"])


@pytest.mark.parametrize("name", ["normal", "weight", "stress", "subnormal", "ragged"])
def test_tensor_fixtures_match_reference(name):
    t = _load("tensors.npz")
    fp4, sf = O.quantize(t[f"{name}_x"])  # the oracle pads to 128 itself
    assert np.array_equal(fp4, t[f"{name}_fp4"])
    assert np.array_equal(sf, t[f"{name}_sf"])


def test_full_size_digests_match_reference():
    d = json.load(open(os.path.join(GOLDEN, "digests.json")))
    w = W.normal_bf16((2880, 2880), 0.02, 1)
    fp4, sf = O.quantize(w)
    assert (_sha(fp4), _sha(sf)) == (d["cfg1_weight_2880x2880_seed1"]["fp4"], d["cfg1_weight_2880x2880_seed1"]["sf"])
    x = W.quantizer_stress(16384, 16384, seed=0)
    fp4, sf = O.quantize(x)
    want = d["cfg4_stress_16384x16384_seed0"]
    assert (_sha(fp4), _sha(sf)) == (want["fp4"], want["sf"])


def test_dequantize_roundtrip_values():
    t = _load("tensors.npz")
    fp4, sf = t["normal_fp4"], t["normal_sf"]
    dq = O.dequantize(fp4, sf, 256, 512)
    # every dequantized value is an E2M1 magnitude times its block's UE4M3 scale
    x = O.bits_to_f32(t["normal_x"])
    err = np.abs(dq - x)
    scale = np.array([O.ue4m3_decode(sf[O.sf_index(r, kb, 32)]) for r in range(256) for kb in range(32)])
    assert np.all(err.reshape(256, 32, 16).max(axis=2).reshape(-1) <= scale * 1.0 + 1e-6)


@pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) not present")
def test_oracle_matches_reference_on_random_tensors():
    rng = np.random.default_rng(7)
    for i in range(4):
        rows, cols = 128 * (i + 1), 128 * (4 - i)
        x = (rng.standard_normal((rows, cols)) * 10.0 ** rng.uniform(-3, 3, (rows, 1))).astype(np.float32)
        bits = O.f32_to_bf16_bits(x)
        a = O.quantize(bits)
        b = O.ref_quantize(bits)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
