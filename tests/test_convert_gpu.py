"""libabx's state-format conversion kernel (abx_convert) against the reference's own conversions and the CPU
checker (oracle/convert.py), through the product's StateBuffer.

The fixture tests/golden/convert/conversions.npz holds what the reference's adambridge/precision.py stored for
seeded values with every special case (zeros of both signs, subnormals, huge values, infinities, NaNs): every
code, scale and plane must match bit for bit; decoded values must match bit for bit, NaNs as positions."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from adambridge_b200.precision import StateBuffer
from oracle import convert as C

pytestmark = pytest.mark.gpu

FIX = Path(__file__).resolve().parent / "golden" / "convert" / "conversions.npz"
DEV = "cuda"


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(FIX))


def as_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
        return t.view(torch.uint8).numpy()
    return t.numpy()


def same_floats(a, b) -> bool:
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a)
    return bool(np.array_equal(nan, np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32)))


def values(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(DEV)


def test_bf16_matches_reference(gold):
    buf = StateBuffer.converted(values(gold["x_m"]), "bf16", "m", DEV)
    assert np.array_equal(as_np(buf.planes["data"]), gold["bf16_data"])
    assert same_floats(as_np(buf.to_fp32()), gold["bf16_read"])


def test_fp24_matches_reference(gold):
    buf = StateBuffer.converted(values(gold["x_m"]), "fp24", "p", DEV)
    assert np.array_equal(as_np(buf.planes["hi"]), gold["fp24_hi"])
    assert np.array_equal(as_np(buf.planes["lo"]), gold["fp24_lo"])
    assert same_floats(as_np(buf.to_fp32()), gold["fp24_read"])


@pytest.mark.parametrize("role", ["m", "v"])
def test_fp8_matches_reference(gold, role):
    buf = StateBuffer.converted(values(gold[f"x_{role}"]), "fp8", role, DEV)
    assert np.array_equal(as_np(buf.planes["scale"]).view(np.uint32), gold[f"fp8_{role}_scale"].view(np.uint32))
    assert np.array_equal(as_np(buf.planes["q"]), gold[f"fp8_{role}_q"])
    assert same_floats(as_np(buf.to_fp32()), gold[f"fp8_{role}_read"])


def test_fp8_moved_between_roles_matches_reference(gold):
    n = gold["x_v"].size
    src = StateBuffer("fp8", "m", n, {"q": torch.from_numpy(gold["m_as_v_src_q"]).to(DEV),
                                      "scale": torch.from_numpy(gold["m_as_v_src_scale"]).to(DEV)})
    dst = StateBuffer.converted(src, "fp8", "v", DEV)
    assert np.array_equal(as_np(dst.planes["q"]), gold["m_as_v_q"])
    assert np.array_equal(as_np(dst.planes["scale"]).view(np.uint32), gold["m_as_v_scale"].view(np.uint32))


def test_fp8_other_block_decodes_like_reference(gold):
    n = gold["x_m"].size
    src = StateBuffer("fp8", "m", n, {"q": torch.from_numpy(gold["fp8_b64_q"]).to(DEV),
                                      "scale": torch.from_numpy(gold["fp8_b64_scale"]).to(DEV)}, block=64)
    assert same_floats(as_np(src.to_fp32()), gold["fp8_b64_read"])
    # re-encoded in the kernels' 128-element blocks, as the checker re-encodes the same values
    dst = StateBuffer.converted(src, "fp8", "m", DEV)
    q, s = C.fp8_encode(gold["fp8_b64_read"], "m")
    assert np.array_equal(as_np(dst.planes["q"]), q)
    assert np.array_equal(as_np(dst.planes["scale"]).view(np.uint32), s.view(np.uint32))


FORMATS = [("fp32", "m"), ("bf16", "m"), ("fp8", "m"), ("fp8", "v"), ("fp24", "p")]


@pytest.mark.parametrize("n", [1, 127, 128, 129, 100_003])
@pytest.mark.parametrize("src", FORMATS)
@pytest.mark.parametrize("dst", FORMATS)
def test_every_pair_of_formats_matches_the_checker(src, dst, n):
    """Random values through every (source format, destination format) pair, at sizes around the block."""
    rng = np.random.default_rng(n * 31 + len(src[0]) * 7 + len(dst[0]))
    x = (rng.standard_normal(n) * 10.0 ** rng.uniform(-8, 3, n)).astype(np.float32)
    if "v" in (src[1], dst[1]):
        x = np.abs(x)
    src_planes = C.encode(src[0], x, src[1])
    if src == dst or (src[0] == dst[0] and src[0] != "fp8"):
        want = src_planes        # the same layout: the planes are copied as they are
    else:
        want = C.encode(dst[0], C.decode(src[0], src_planes, n, src[1]), dst[1])
    out = StateBuffer.converted(_on_device(src, n, src_planes, misalign=False), dst[0], dst[1], DEV)
    _assert_planes(out, want)


def _on_device(fmt_role, n, planes, misalign: bool) -> StateBuffer:
    """The planes as device tensors; ``misalign`` starts every plane one element into its allocation, so no
    plane is aligned for vector accesses (the conversion's one-value-at-a-time kernel)."""
    tensors = {}
    for k, a in planes.items():
        t = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a)
        if misalign and k != "scale":
            tensors[k] = torch.cat([t[:1], t]).to(DEV)[1:]   # one element into its allocation
        else:
            tensors[k] = t.to(DEV)
    return StateBuffer(fmt_role[0], fmt_role[1], n, tensors)


def _assert_planes(out: StateBuffer, want: dict) -> None:
    for k, a in want.items():
        got = as_np(out.planes[k])
        if a.dtype == np.float32:
            assert same_floats(got, a), k
        else:
            assert np.array_equal(got.view(a.dtype), a), k


@pytest.mark.parametrize("n", [129, 100_003])
@pytest.mark.parametrize("src", FORMATS)
@pytest.mark.parametrize("dst", [f for f in FORMATS if f[0] != "fp8"] + [("fp8", "m")])
def test_unaligned_buffers_take_the_scalar_kernel(src, dst, n):
    """Sources that start one element into their allocation (no vector access possible) convert to the same bits
    as the checker gives."""
    if src[0] == dst[0] and src[0] != "fp8":
        return   # same layout: a plane copy, no kernel
    rng = np.random.default_rng(n + 17)
    x = np.abs((rng.standard_normal(n) * 10.0 ** rng.uniform(-8, 3, n)).astype(np.float32))
    src_planes = C.encode(src[0], x, src[1])
    want = C.encode(dst[0], C.decode(src[0], src_planes, n, src[1]), dst[1])
    out = StateBuffer.converted(_on_device(src, n, src_planes, misalign=True), dst[0], dst[1], DEV)
    _assert_planes(out, want)


@pytest.mark.parametrize("role", ["m", "v"])
def test_every_bf16_value_into_fp8(role):
    """All 65,536 bf16 bit patterns (zeros, subnormals, infinities, NaNs of both signs among them), in 512 blocks
    whose ranges differ, re-encoded as FP8: the kernel's codes and scales are the checker's."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    src_planes = {"data": bits}
    want = C.encode("fp8", C.decode("bf16", src_planes, bits.size, "m"), role)
    out = StateBuffer.converted(_on_device(("bf16", "m"), bits.size, src_planes, misalign=False), "fp8", role, DEV)
    _assert_planes(out, want)


@pytest.mark.parametrize("role", ["m", "v"])
def test_every_fp8_code_decodes(role):
    """Every code under block scales from 2^-126 to 2^126 (and 0, inf, NaN scales) decodes to the checker's
    values, NaN signs and the host's 0 x inf NaN included."""
    scales = np.array([2.0 ** e for e in range(-126, 127, 9)] + [0.0, np.inf, np.nan, 1.0, 3e-45],
                      np.float32)
    codes = np.tile(np.arange(256, dtype=np.uint8), 2 * scales.size)     # two blocks of 128 per scale
    planes = {"q": codes, "scale": np.repeat(scales, 4)}
    n = codes.size
    want = C.decode("fp8", planes, n, role)
    got = StateBuffer("fp8", role, n, {"q": torch.from_numpy(codes).to(DEV),
                                       "scale": torch.from_numpy(planes["scale"]).to(DEV)}).to_fp32()
    g = as_np(got)
    assert same_floats(g, want)
    nan = np.isnan(want)
    assert np.array_equal(g[nan].view(np.uint32) >> 31, want[nan].view(np.uint32) >> 31)   # NaN signs
