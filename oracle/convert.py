"""TEST INFRASTRUCTURE ONLY: a numpy restatement of the reference's state-format conversions.

The reference converts optimizer state between formats with torch operations on the host
(adambridge/precision.py): a bf16 moment is a nearest-even cast (BF16Store.write :319-323), an FP8
moment is written by FP8Store.write without a seed (:383-398) and read by FP8Store.read (:374-381), an
fp24 master by FP24Store.write / read (:448-462, round_to_fp24_nearest_ :185-194).  This module states
the same arithmetic with numpy float32 operations (IEEE round-to-nearest, as torch's CPU kernels) and
integer bit operations, so tests can check libabx's device conversion kernel (abx_convert) against it.
It is pinned to the reference itself by the fixtures in tests/golden/convert/ (made by
tests/golden/make_reference_states.py from the reference's own precision.py).

Only tests import this module.
"""

from __future__ import annotations

import numpy as np

BLOCK = 128
FP8 = {"m": dict(mbits=3, bias=7, fmax=np.float32(448.0)),      # E4M3 (fn): no infinities, 0x7f is NaN
       "v": dict(mbits=2, bias=15, fmax=np.float32(57344.0))}   # E5M2 of sqrt(v): IEEE-style inf and NaN


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


# ---- bf16 ---------------------------------------------------------------------------------------

def bf16_encode(x) -> np.ndarray:
    """Nearest-even bf16 bits (uint16); NaN -> 0x7fc0 (torch's float -> bfloat16 cast)."""
    x = _f32(x)
    b = x.view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), r)


def bf16_decode(h) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- fp24 -----------------------------------------------------------------------------------------

def fp24_encode(x) -> tuple[np.ndarray, np.ndarray]:
    """(hi, lo) planes of the nearest-even top 24 bits; a NaN is quieted and kept whole."""
    x = _f32(x)
    b = x.view(np.uint32).astype(np.uint64)
    r = (b + 0x7F + ((b >> 8) & 1)) & ~np.uint64(0xFF)
    r = np.where(np.isnan(x), b | 0x00400000, r).astype(np.uint32)
    return (r >> 16).astype(np.uint16), ((r >> 8) & 0xFF).astype(np.uint8)


def fp24_decode(hi, lo) -> np.ndarray:
    bits = (np.asarray(hi, np.uint16).astype(np.uint32) << 16) | (np.asarray(lo, np.uint8).astype(np.uint32) << 8)
    return bits.view(np.float32)


# ---- FP8 --------------------------------------------------------------------------------------------

def fp8_code(q, role: str) -> np.ndarray:
    """Codes of values already clamped to the format's range (or NaN), nearest-even; NaN -> 0x7f | sign.

    Below the smallest normal a value is a multiple of the smallest subnormal, rounded half-to-even (np.rint);
    above it the fp32 significand is rounded half-to-even at the format's width by an integer add."""
    f = FP8[role]
    mbits, bias = f["mbits"], f["bias"]
    q = _f32(q)
    b = q.view(np.uint32).astype(np.uint64)
    sign = ((b >> 24) & 0x80).astype(np.uint32)
    a = (b & 0x7FFFFFFF).astype(np.uint32).view(np.float32)
    with np.errstate(invalid="ignore"):
        sub = np.rint(a.astype(np.float64) / 2.0 ** (1 - bias - mbits))
        sub = np.nan_to_num(sub).astype(np.uint32)
    drop = 23 - mbits
    ab = a.view(np.uint32).astype(np.uint64)
    r = ab + ((1 << (drop - 1)) - 1) + ((ab >> drop) & 1)
    exp = (r >> 23).astype(np.int64) - 127 + bias
    mant = ((r >> drop) & ((1 << mbits) - 1)).astype(np.int64)
    normal = np.where(exp > 0, (exp << mbits) | mant, 0).astype(np.uint32)
    code = np.where(a < np.float32(2.0 ** (1 - bias)), sub, normal)
    code = np.where(np.isnan(q), np.uint32(0x7F), code)
    return ((code | sign) & 0xFF).astype(np.uint8)


def fp8_value(codes, role: str) -> np.ndarray:
    """Exact value of every code (E4M3: 0x7f/0xff NaN; E5M2: exponent 31 is inf or NaN).  A NaN code gives the
    quiet NaN the host's conversion gives -- its sign, and E5M2's mantissa bits above the quiet bit."""
    f = FP8[role]
    mbits, bias = f["mbits"], f["bias"]
    c = np.asarray(codes, np.uint8).astype(np.int64)
    e = (c >> mbits) & ((1 << (7 - mbits)) - 1)
    m = c & ((1 << mbits) - 1)
    mag = np.where(e == 0, m * 2.0 ** (1 - bias - mbits), (1.0 + m / 2.0 ** mbits) * 2.0 ** (e - bias))
    if role == "m":
        nan = (c & 0x7F) == 0x7F
        nan_bits = np.full(c.shape, 0x7FE00000, np.int64)
    else:
        top = e == (1 << (7 - mbits)) - 1
        mag = np.where(top & (m == 0), np.inf, mag)
        nan = top & (m != 0)
        nan_bits = 0x7FC00000 | (m << 21)
    val = np.copysign(mag, np.where(c & 0x80, -1.0, 1.0)).astype(np.float32)
    bits = np.where(nan, nan_bits | ((c & 0x80) << 24), val.view(np.uint32).astype(np.int64))
    return bits.astype(np.uint32).view(np.float32)


def fp8_encode(x, role: str) -> tuple[np.ndarray, np.ndarray]:
    """(codes padded to whole blocks, fp32 scales) of the values ``x`` (a second moment v, role 'v', is stored
    as sqrt(max(v, 0))): scale = block absmax / fmax (1 if the absmax is 0 or NaN), x / scale clamped."""
    f = FP8[role]
    x = _f32(x).copy()
    n = x.size
    if role == "v":
        with np.errstate(invalid="ignore"):
            x = np.sqrt(np.where(x < 0, np.float32(0.0), x))
    nb = max(1, -(-n // BLOCK))
    xb = np.zeros(nb * BLOCK, np.float32)
    xb[:n] = x
    xb = xb.reshape(nb, BLOCK)
    with np.errstate(invalid="ignore"):
        amax = np.abs(xb).max(axis=1)
        scale = np.where(amax > 0, amax / f["fmax"], np.float32(1.0)).astype(np.float32)
        q = np.clip(xb / scale[:, None], -f["fmax"], f["fmax"]).astype(np.float32)
    return fp8_code(q.reshape(-1), role), scale


def fp8_decode(codes, scales, n: int, role: str, block: int = BLOCK) -> np.ndarray:
    """Values of the first n elements: code x block scale, squared for a second moment."""
    q = fp8_value(np.asarray(codes)[:n], role)
    sc = np.asarray(scales, np.float32)[np.arange(n) // block]
    with np.errstate(invalid="ignore", over="ignore"):
        x = (q * sc).astype(np.float32)
        return (x * x).astype(np.float32) if role == "v" else x


# ---- one buffer, any format --------------------------------------------------------------------------

def decode(fmt: str, planes: dict, n: int, role: str = "m", block: int = BLOCK) -> np.ndarray:
    if fmt == "fp32":
        return _f32(planes["data"])[:n]
    if fmt == "bf16":
        return bf16_decode(planes["data"])[:n]
    if fmt == "fp24":
        return fp24_decode(planes["hi"], planes["lo"])[:n]
    return fp8_decode(planes["q"], planes["scale"], n, role, block)


def encode(fmt: str, x, role: str = "m") -> dict:
    x = _f32(x)
    if fmt == "fp32":
        return {"data": x.copy()}
    if fmt == "bf16":
        return {"data": bf16_encode(x)}
    if fmt == "fp24":
        hi, lo = fp24_encode(x)
        return {"hi": hi, "lo": lo}
    q, s = fp8_encode(x, role)
    return {"q": q, "scale": s}
