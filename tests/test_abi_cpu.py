"""The C ABI boundary without a GPU: libabx loads, exports every function include/abx.h declares, keeps the
reference's struct layouts and codes, computes the reference's coefficients and seeds, and rejects bad
segments with the reference's error codes before touching CUDA (tests/test_hardening.py:91-104 analogue)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from oracle import oracle as O

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> list[str]:
    text = (ROOT / "include" / "abx.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(abx_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_function(kernels):
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(kernels._lib, name), name


def test_struct_layouts_match_reference(kernels, reference):
    from adambridge_b200 import native
    assert kernels._lib.abx_segment_size() == ctypes.sizeof(native.Segment) == ctypes.sizeof(O.Segment) == 128
    assert kernels._lib.abx_group_size() == ctypes.sizeof(native.Group) == 56
    assert kernels._lib.abx_hparams_size() == ctypes.sizeof(native._HParams) == 40
    if reference is not None:   # the reference library's own sizes
        assert reference._lib.adambridge_segment_size() == 128
        assert reference._lib.adambridge_group_size() == 56
        assert reference._lib.adambridge_hparams_size() == 40


def test_codes_match_reference():
    from adambridge_b200 import native
    assert (native.DT_NONE, native.DT_F32, native.DT_BF16, native.DT_FP8, native.DT_F24) == (0, 1, 2, 3, 4)
    assert native.ALGORITHMS == {"adamw": 0, "lion": 1}
    assert native.MOMENT_CODES == {"fp32": 1, "bf16": 2, "fp8": 3}


def test_simd_level_selection(kernels):
    assert kernels.detected_simd_level == "avx512"
    try:
        for name in ("scalar", "avx2", "neon", "avx512"):
            assert kernels.set_simd_level(name) == name
            assert kernels.simd_level == name
        assert kernels._lib.abx_set_simd_level(9) == -22
    finally:
        kernels.set_simd_level(None)
    assert kernels.simd_level == "avx512"


def test_hparams_and_seed_identical_to_oracle(kernels, oracle):
    from adambridge_b200 import native
    for base, index, step in [(0, 0, 1), (5, 290, 17), (2**64 - 1, 2**40, 99999)]:
        assert kernels.step_seed(base, index, step) == oracle.step_seed(base, index, step)
    for lion in (0, 1):
        for step in (1, 3, 50, 10**6):
            grp = dict(lr=2e-5, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, seed=7, stochastic=1)
            ng, og = native.Group(**grp), O.Group(**grp)
            ps = native.Segment(n=1, step=step, index=3, algorithm=lion)
            ps.group = ctypes.pointer(ng)
            os_ = O.Segment(n=1, step=step, index=3, algorithm=lion)
            os_.group = ctypes.pointer(og)
            a, b = kernels.hparams_for(ps), oracle.hparams_for(os_)
            assert bytes(a) == bytes(b)


def _valid_segment():
    from adambridge_b200 import native
    s = native.Segment(p=0x1000, g=0x2000, m=0x3000, v=0x4000, m_scale=0x5000, v_scale=0x6000, out=0x7000,
                       n=256, step=1, index=0, offset=0, g_dtype=2, mv_dtype=3, out_dtype=2, algorithm=0, p_dtype=1)
    return s


@pytest.mark.parametrize("field,value,code", [
    ("n", -1, -1), ("algorithm", 7, -12), ("p_dtype", 9, -13), ("g", None, -2), ("g_dtype", 3, -3),
    ("mv_dtype", 4, -4), ("out_dtype", 3, -5), ("out", None, -6), ("m_scale", None, -7), ("offset", 100, -11),
    ("offset", -128, -11),
])
def test_validation_codes_before_any_cuda_call(kernels, oracle, field, value, code):
    """Each rejection is decided on the host, with the reference's code, before anything is launched (these
    calls never reach CUDA: the pointers are not even valid device addresses)."""
    from adambridge_b200 import native
    grp = native.Group(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, seed=0, stochastic=1)
    s = _valid_segment()
    s.group = ctypes.pointer(grp)
    setattr(s, field, value)
    rc = kernels._lib.abx_multi_step(None, kernels.segment_array([ctypes.pointer(s)]), 1, 0)
    assert rc == code
    o = O.Segment.from_buffer_copy(bytes(s))
    assert oracle.check_segment(o, True) == code


def test_missing_group_and_null_array(kernels):
    s = _valid_segment()
    assert kernels._lib.abx_multi_step(None, kernels.segment_array([ctypes.pointer(s)]), 1, 0) == -8
    assert kernels._lib.abx_multi_step(None, None, 1, 0) == -1
    assert kernels._lib.abx_multi_step(None, None, 0, 0) == 0
    assert kernels._lib.abx_multi_apply(None, kernels.segment_array([ctypes.pointer(s)]), None, 1, 0) == -1


def test_misaligned_pointer_rejected_before_launch(kernels):
    from adambridge_b200 import native
    grp = native.Group(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, seed=0, stochastic=1)
    s = _valid_segment()
    s.group = ctypes.pointer(grp)
    s.p = 0x1002          # fp32 master not 4-byte aligned
    assert kernels._lib.abx_multi_step(None, kernels.segment_array([ctypes.pointer(s)]), 1, 0) == -21
    assert b"aligned" in kernels._lib.abx_last_error()


def test_fused_adamw_argument_codes(kernels):
    """adambridge_fused_adamw's checks (csrc:1518-1535) in order, all before any CUDA call."""
    from adambridge_b200 import native
    hp = native._HParams()
    f = kernels._lib.abx_fused_adamw
    assert f(0x10, 0x20, 1, 0x30, 0x40, 1, None, 0, -1, 0, ctypes.byref(hp), None) == -1
    assert f(0x10, 0x20, 1, 0x30, 0x40, 1, None, 0, 0, 0, ctypes.byref(hp), None) == 0
    assert f(None, 0x20, 1, 0x30, 0x40, 1, None, 0, 8, 0, ctypes.byref(hp), None) == -2
    assert f(0x10, 0x20, 3, 0x30, 0x40, 1, None, 0, 8, 0, ctypes.byref(hp), None) == -3
    assert f(0x10, 0x20, 1, 0x30, 0x40, 3, None, 0, 8, 0, ctypes.byref(hp), None) == -4
    assert f(0x10, 0x20, 1, 0x30, 0x40, 1, None, 4, 8, 0, ctypes.byref(hp), None) == -5
    assert f(0x10, 0x20, 1, 0x30, 0x40, 1, None, 2, 8, 0, ctypes.byref(hp), None) == -6


def test_clip_noalloc_limit_rejected_before_any_cuda_call(kernels):
    """abx_clip_coef_noalloc's static scratch holds 524,288 norm tiles of 16384 elements: gradients needing one
    tile more get ABX_E_SCRATCH (-23) and a message, from host checks made before any CUDA call (here, with no
    GPU, a CUDA call would return -20 instead).  The pointers are never dereferenced."""
    from adambridge_b200 import native
    arr = (native.Tensor * 2)()
    arr[0] = native.Tensor(0x1000, 16384 * 524_288, native.DT_BF16, 0)
    arr[1] = native.Tensor(0x2000, 1, native.DT_BF16, 0)
    f = kernels._lib.abx_clip_coef_noalloc
    assert f(None, arr, 2, 1.0, 0x3000, None, 0x4000) == -23
    assert b"static scratch" in kernels._lib.abx_last_error()
    assert f(None, arr, 0, 1.0, 0x3000, None, 0x4000) == -1
    arr[1] = native.Tensor(0x2000, 1, native.DT_F32, 0)
    assert f(None, arr, 2, 1.0, 0x3000, None, 0x4000) == -3      # one dtype for all gradients


def test_product_loader_fails_loudly_without_library(tmp_path, monkeypatch):
    """No fallback: a missing library raises instead of switching to another implementation."""
    from adambridge_b200 import native
    monkeypatch.setattr(native, "LIBRARY", tmp_path / "libabx.so")
    monkeypatch.setattr(native, "_loaded", None)
    with pytest.raises(native.BuildError):
        native.load()


def test_convert_rejects_bad_arguments_before_touching_the_device(kernels):
    """abx_convert checks formats, roles, blocks, pointers and alignment before any CUDA call (so on a machine
    without a GPU every rejection still comes back; the addresses are never dereferenced)."""
    from adambridge_b200 import native
    vals, codes, scales = 0x10000, 0x20000, 0x30000
    src = native.State(vals, None, native.DT_F32, 0, 1)
    cases = [(native.State(codes, None, native.DT_FP8, 0, 128), -7),         # FP8 without scales
             (native.State(codes, scales, native.DT_FP8, 0, 64), -1),        # a destination block other than 128
             (native.State(codes, scales, native.DT_FP8, 2, 128), -1),       # unknown role
             (native.State(codes, scales, 9, 0, 128), -4),                   # unknown format
             (native.State(None, None, native.DT_F32, 0, 1), -2),            # no values
             (native.State(vals + 2, None, native.DT_F32, 0, 1), -21),       # fp32 values not 4-byte aligned
             (native.State(codes, None, native.DT_F24, 0, 1), -7)]           # fp24 without its lo plane
    for dst, code in cases:
        assert kernels._lib.abx_convert(None, ctypes.byref(src), ctypes.byref(dst), 256) == code
    bad_src = native.State(codes, scales, native.DT_FP8, 0, 0)               # a source block of 0
    ok_dst = native.State(vals, None, native.DT_F32, 0, 1)
    assert kernels._lib.abx_convert(None, ctypes.byref(bad_src), ctypes.byref(ok_dst), 256) == -1
    assert kernels._lib.abx_convert(None, ctypes.byref(src), ctypes.byref(ok_dst), -1) == -1
    assert kernels._lib.abx_convert(None, ctypes.byref(src), ctypes.byref(ok_dst), 0) == 0


def test_replicate_rejects_bad_arguments_before_any_copy(kernels):
    """abx_replicate_async checks sizes, replica counts, pointers and overlap before issuing a copy (the addresses
    are never touched, so every rejection comes back on a machine without a GPU)."""
    lib = kernels._lib
    streams = (ctypes.c_void_p * 8)(*([None] * 8))

    def deltas(*d):
        return (ctypes.c_int64 * max(1, len(d)))(*d)

    src = 0x100000
    assert lib.abx_replicate_async(streams, src, -1, deltas(1 << 20), 1) == -1        # negative size
    assert lib.abx_replicate_async(streams, src, 64, deltas(*[1 << 20] * 8), 8) == -1  # more than 7 replicas
    assert lib.abx_replicate_async(streams, src, 64, deltas(1 << 20), -1) == -1
    assert lib.abx_replicate_async(streams, None, 64, deltas(1 << 20), 1) == -2        # no source
    assert lib.abx_replicate_async(None, src, 64, deltas(1 << 20), 1) == -2            # no streams
    assert lib.abx_replicate_async(streams, src, 64, None, 1) == -2                    # no deltas
    assert lib.abx_replicate_async(streams, src, 64, deltas(1 << 20, 32), 2) == -1     # a replica overlaps src
    assert lib.abx_replicate_async(streams, src, 64, deltas(-63), 1) == -1
    assert lib.abx_replicate_async(streams, src, 0, deltas(1 << 20), 1) == 0           # nothing to copy
    assert lib.abx_replicate_async(streams, src, 64, deltas(), 0) == 0
