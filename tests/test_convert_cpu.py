"""The CPU checker for state-format conversions (oracle/convert.py) against the reference's own conversions.

The fixture tests/golden/convert/conversions.npz was written by the reference's adambridge/precision.py
(tests/golden/make_reference_states.py): values with zeros of both signs, subnormals, huge values, infinities
and NaNs stored as bf16, FP8 (first and second moment), fp24, an FP8 store moved between roles, and a
64-element-block FP8 store.  Every stored bit must match; values read back must match bit for bit too, NaN
positions compared as positions."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import convert as C

FIX = Path(__file__).resolve().parent / "golden" / "convert" / "conversions.npz"


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(FIX))


def same_floats(a, b) -> bool:
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a)
    return bool(np.array_equal(nan, np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32)))


def test_bf16(gold):
    assert np.array_equal(C.bf16_encode(gold["x_m"]), gold["bf16_data"])
    assert same_floats(C.bf16_decode(gold["bf16_data"]), gold["bf16_read"])


def test_fp24(gold):
    hi, lo = C.fp24_encode(gold["x_m"])
    assert np.array_equal(hi, gold["fp24_hi"]) and np.array_equal(lo, gold["fp24_lo"])
    assert same_floats(C.fp24_decode(hi, lo), gold["fp24_read"])


@pytest.mark.parametrize("role", ["m", "v"])
def test_fp8_roles(gold, role):
    q, s = C.fp8_encode(gold[f"x_{role}"], role)
    assert np.array_equal(s.view(np.uint32), gold[f"fp8_{role}_scale"].view(np.uint32))
    assert np.array_equal(q, gold[f"fp8_{role}_q"])
    n = gold[f"x_{role}"].size
    assert same_floats(C.fp8_decode(q, s, n, role), gold[f"fp8_{role}_read"])


def test_fp8_store_moved_between_roles(gold):
    n = gold["x_v"].size
    src = C.fp8_decode(gold["m_as_v_src_q"], gold["m_as_v_src_scale"], n, "m")
    q, s = C.fp8_encode(src, "v")
    assert np.array_equal(q, gold["m_as_v_q"])
    assert np.array_equal(s.view(np.uint32), gold["m_as_v_scale"].view(np.uint32))


def test_fp8_other_block_decodes(gold):
    n = gold["x_m"].size
    got = C.fp8_decode(gold["fp8_b64_q"], gold["fp8_b64_scale"], n, "m", block=64)
    assert same_floats(got, gold["fp8_b64_read"])


def test_fp8_codes_cover_every_finite_value():
    """Every finite code decodes and re-encodes to itself (scale 1, both formats)."""
    for role in ("m", "v"):
        codes = np.arange(256, dtype=np.uint8)
        vals = C.fp8_value(codes, role)
        finite = np.isfinite(vals)
        assert np.array_equal(C.fp8_code(vals[finite], role), codes[finite])
