"""TEST INFRASTRUCTURE ONLY: ctypes bindings of the CPU checkers for libabx.

Two libraries, both built by ``oracle/Makefile``:

* ``Oracle`` -- ``oracle/_build/libabx_oracle.so``, the plain-C restatement of the
  reference's update arithmetic (``oracle/abx_oracle.c``), parameterised by the SIMD
  level whose rounding pattern it reproduces.
* ``Reference`` -- ``oracle/_ref/libadambridge_ref.so``, the reference's own kernel
  library (adambridge/csrc/adambridge_kernels.c) compiled from its sources with its own
  flags.  It exists where the reference tree was present at build time; it travels
  with the repository snapshot as a prebuilt file.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this
module, and only as the checker or the timed CPU baseline -- never as the product.

``HostSegment`` owns numpy buffers in the reference's segment layout
(adambridge/csrc/adambridge_kernels.c:747-769) so one seeded case can be run
through the oracle, the reference library and the GPU kernels alike.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "libabx_oracle.so"
REF_LIB = HERE / "_ref" / "libadambridge_ref.so"

DT_NONE, DT_F32, DT_BF16, DT_FP8, DT_F24 = 0, 1, 2, 3, 4
ADAMW, LION = 0, 1
SIMD_SCALAR, SIMD_AVX2, SIMD_AVX512, SIMD_NEON = 0, 1, 2, 3
SIMD_NAMES = {0: "scalar", 1: "avx2", 2: "avx512", 3: "neon"}
FP8_BLOCK = 128


class HParams(ctypes.Structure):
    _fields_ = [("beta1", ctypes.c_float), ("beta2", ctypes.c_float), ("one_minus_beta1", ctypes.c_float),
                ("one_minus_beta2", ctypes.c_float), ("decay", ctypes.c_float), ("step_size", ctypes.c_float),
                ("inv_sqrt_bc2", ctypes.c_float), ("eps", ctypes.c_float), ("seed", ctypes.c_uint32),
                ("stochastic", ctypes.c_int32)]


class Group(ctypes.Structure):
    _fields_ = [("lr", ctypes.c_double), ("beta1", ctypes.c_double), ("beta2", ctypes.c_double),
                ("eps", ctypes.c_double), ("weight_decay", ctypes.c_double), ("seed", ctypes.c_uint64),
                ("stochastic", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class Segment(ctypes.Structure):
    _fields_ = [("p", ctypes.c_void_p), ("p_lo", ctypes.c_void_p), ("g", ctypes.c_void_p),
                ("m", ctypes.c_void_p), ("v", ctypes.c_void_p), ("m_scale", ctypes.c_void_p),
                ("v_scale", ctypes.c_void_p), ("out", ctypes.c_void_p), ("group", ctypes.POINTER(Group)),
                ("n", ctypes.c_int64), ("step", ctypes.c_int64), ("index", ctypes.c_uint64),
                ("offset", ctypes.c_int64), ("g_dtype", ctypes.c_int32), ("mv_dtype", ctypes.c_int32),
                ("out_dtype", ctypes.c_int32), ("algorithm", ctypes.c_int32), ("p_dtype", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


def seg_array(segs: list) -> ctypes.Array:
    return (ctypes.POINTER(Segment) * len(segs))(*[ctypes.pointer(s) for s in segs])


_build_lock = threading.Lock()


def build(ref: bool = False) -> None:
    """Build the restatement (and, with ``ref``, the reference library when its sources are present)."""
    with _build_lock:
        targets = ["all"] + (["ref"] if ref else [])
        subprocess.run(["make", "-s", "-C", str(HERE), *targets], check=True)


class Oracle:
    """The C restatement (abx_oracle.c)."""

    def __init__(self, path: Path = ORACLE_LIB):
        if not path.exists():
            build()
        lib = ctypes.CDLL(str(path))
        seg_pp = ctypes.POINTER(ctypes.POINTER(Segment))
        lib.abxo_multi_apply.argtypes = [seg_pp, ctypes.POINTER(HParams), ctypes.c_int32, ctypes.c_int,
                                         ctypes.POINTER(ctypes.c_float)]
        lib.abxo_multi_step.argtypes = [seg_pp, ctypes.c_int32, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]
        lib.abxo_hparams_for.argtypes = [ctypes.POINTER(Segment), ctypes.POINTER(HParams)]
        lib.abxo_hparams_for.restype = None
        lib.abxo_step_seed.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64]
        lib.abxo_step_seed.restype = ctypes.c_uint32
        lib.abxo_hash32.argtypes = [ctypes.c_uint32]
        lib.abxo_hash32.restype = ctypes.c_uint32
        lib.abxo_fp8_encode.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.c_uint32, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_float, ctypes.c_uint32]
        lib.abxo_fp8_encode.restype = ctypes.c_uint32
        lib.abxo_fp8_decode.argtypes = [ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.abxo_fp8_decode.restype = ctypes.c_float
        lib.abxo_check_segment.argtypes = [ctypes.POINTER(Segment), ctypes.c_int]
        if lib.abxo_segment_size() != ctypes.sizeof(Segment):
            raise RuntimeError("oracle segment layout mismatch")
        self._lib = lib

    @staticmethod
    def _scale(g_scale):
        return None if g_scale is None else ctypes.pointer(ctypes.c_float(g_scale))

    def multi_apply(self, segs: list, hps: list, level: int = SIMD_AVX512, g_scale: float | None = None) -> int:
        arr = (HParams * len(hps))(*hps)
        return self._lib.abxo_multi_apply(seg_array(segs), arr, len(segs), level, self._scale(g_scale))

    def multi_step(self, segs: list, level: int = SIMD_AVX512, g_scale: float | None = None) -> int:
        return self._lib.abxo_multi_step(seg_array(segs), len(segs), level, self._scale(g_scale))

    def hparams_for(self, seg: Segment) -> HParams:
        h = HParams()
        self._lib.abxo_hparams_for(ctypes.byref(seg), ctypes.byref(h))
        return h

    def step_seed(self, base: int, index: int, step: int) -> int:
        return self._lib.abxo_step_seed(base, index, step)

    def hash32(self, x: int) -> int:
        return self._lib.abxo_hash32(x)

    def fp8_encode(self, x: float, sr: int, r: int, role: str) -> int:
        if role == "m":
            return self._lib.abxo_fp8_encode(x, sr, r, 3, 7, 448.0, 0x7F)
        return self._lib.abxo_fp8_encode(x, sr, r, 2, 15, 57344.0, 0x7E)

    def fp8_decode(self, code: int, role: str) -> float:
        return self._lib.abxo_fp8_decode(code, 3, 7, 0) if role == "m" else self._lib.abxo_fp8_decode(code, 2, 15, 1)

    def check_segment(self, seg: Segment, need_group: bool = True) -> int:
        return self._lib.abxo_check_segment(ctypes.byref(seg), int(need_group))


class Reference:
    """The reference's own native library, compiled from its sources (oracle/_ref)."""

    def __init__(self, path: Path = REF_LIB):
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (the reference sources were absent at build time)")
        lib = ctypes.CDLL(str(path))
        for fn in ("adambridge_abi_version", "adambridge_simd_level", "adambridge_detected_simd_level",
                   "adambridge_set_simd_level", "adambridge_segment_size", "adambridge_group_size",
                   "adambridge_hparams_size"):
            getattr(lib, fn).restype = ctypes.c_int
        lib.adambridge_set_simd_level.argtypes = [ctypes.c_int]
        seg_pp = ctypes.POINTER(ctypes.POINTER(Segment))
        lib.adambridge_multi_step.argtypes = [ctypes.c_void_p, seg_pp, ctypes.c_int32, ctypes.c_int32]
        lib.adambridge_multi_apply.argtypes = [ctypes.c_void_p, seg_pp, ctypes.POINTER(HParams), ctypes.c_int32,
                                               ctypes.c_int32]
        lib.adambridge_pool_create.restype = ctypes.c_void_p
        lib.adambridge_pool_create.argtypes = [ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32]
        lib.adambridge_pool_destroy.argtypes = [ctypes.c_void_p]
        for fn, cls in (("adambridge_segment_size", Segment), ("adambridge_group_size", Group),
                        ("adambridge_hparams_size", HParams)):
            if getattr(lib, fn)() != ctypes.sizeof(cls):
                raise RuntimeError(f"{fn}: layout mismatch with the reference library")
        self._lib = lib
        self._pools: dict[int, int] = {}

    @property
    def abi_version(self) -> int:
        return self._lib.adambridge_abi_version()

    @property
    def simd_level(self) -> int:
        return self._lib.adambridge_simd_level()

    @property
    def detected_simd_level(self) -> int:
        return self._lib.adambridge_detected_simd_level()

    def set_simd_level(self, level: int | None) -> int:
        return self._lib.adambridge_set_simd_level(-1 if level is None else level)

    def pool(self, threads: int) -> int | None:
        if threads <= 1:
            return None
        if threads not in self._pools:
            self._pools[threads] = self._lib.adambridge_pool_create(threads, None, 0)
        return self._pools[threads]

    def multi_step(self, segs: list, threads: int = 1) -> int:
        return self._lib.adambridge_multi_step(self.pool(threads), seg_array(segs), len(segs), threads)

    def multi_step_array(self, arr: ctypes.Array, threads: int = 1) -> int:
        return self._lib.adambridge_multi_step(self.pool(threads), arr, len(arr), threads)

    def multi_apply(self, segs: list, hps: list, threads: int = 1) -> int:
        arr = (HParams * len(hps))(*hps)
        return self._lib.adambridge_multi_apply(self.pool(threads), seg_array(segs), arr, len(segs), threads)


_oracle: Oracle | None = None
_reference: Reference | None = None


def load_oracle() -> Oracle:
    global _oracle
    if _oracle is None:
        _oracle = Oracle()
    return _oracle


def load_reference() -> Reference | None:
    """The reference library, or None where it was not built."""
    global _reference
    if _reference is None and REF_LIB.exists():
        _reference = Reference()
    return _reference


# --------------------------------------------------------------------------- host buffers

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (NaN made quiet)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((b | 0x00400000) >> 16).astype(np.uint16), r)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def f24_to_f32(hi: np.ndarray, lo: np.ndarray) -> np.ndarray:
    return ((hi.astype(np.uint32) << 16) | (lo.astype(np.uint32) << 8)).view(np.float32)


def f32_to_f24_rne(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (b + 0x7F + ((b >> 8) & 1)) & ~np.uint32(0xFF)
    return (r >> 16).astype(np.uint16), ((r >> 8) & 0xFF).astype(np.uint8)


_ELEM = {DT_F32: np.float32, DT_BF16: np.uint16, DT_FP8: np.uint8}


@dataclass
class HostSegment:
    """Numpy buffers of one segment in the reference's layout, plus its descriptor fields."""

    n: int
    g_dtype: int
    mv_dtype: int
    out_dtype: int
    p_dtype: int = DT_F32
    algorithm: int = ADAMW
    offset: int = 0
    index: int = 0
    step: int = 1
    buffers: dict = field(default_factory=dict)

    BUFFER_NAMES = ("p", "p_lo", "g", "m", "v", "m_scale", "v_scale", "out")

    @property
    def nblocks(self) -> int:
        return max(1, -(-self.n // FP8_BLOCK))

    def moment_len(self) -> int:
        return self.nblocks * FP8_BLOCK if self.mv_dtype == DT_FP8 else self.n

    @classmethod
    def random(cls, n: int, g_dtype: int, mv_dtype: int, out_dtype: int, p_dtype: int = DT_F32,
               algorithm: int = ADAMW, seed: int = 0, offset: int = 0, index: int = 0,
               p_scale: float = 1.0, g_scale: float = 0.1) -> "HostSegment":
        """Seeded buffers: master ~ U(-1,1)*p_scale, grad ~ U(-1,1)*g_scale, zero moments, unit scales."""
        rng = np.random.default_rng(seed)
        s = cls(n, g_dtype, mv_dtype, out_dtype, p_dtype, algorithm, offset, index)
        p = (rng.uniform(-1, 1, n) * p_scale).astype(np.float32)
        if p_dtype == DT_F24:
            s.buffers["p"], s.buffers["p_lo"] = f32_to_f24_rne(p)
        else:
            s.buffers["p"] = p
        g = (rng.uniform(-1, 1, n) * g_scale).astype(np.float32)
        s.buffers["g"] = bf16_bits(g) if g_dtype == DT_BF16 else g
        mlen = s.moment_len()
        s.buffers["m"] = np.zeros(mlen, _ELEM[mv_dtype])
        if algorithm == ADAMW:
            s.buffers["v"] = np.zeros(mlen, _ELEM[mv_dtype])
        if mv_dtype == DT_FP8:
            s.buffers["m_scale"] = np.ones(s.nblocks, np.float32)
            if algorithm == ADAMW:
                s.buffers["v_scale"] = np.ones(s.nblocks, np.float32)
        if out_dtype != DT_NONE:
            s.buffers["out"] = np.zeros(n, np.float32 if out_dtype == DT_F32 else np.uint16)
        return s

    def randomize_moments(self, seed: int) -> "HostSegment":
        """Nonzero moments: m ~ U(-1,1)*1e-2, v ~ U(0,1)*1e-3; FP8: random finite codes, scales in [1e-4, 1]."""
        rng = np.random.default_rng(seed)
        mlen = self.moment_len()
        b = self.buffers
        if self.mv_dtype == DT_FP8:
            m = rng.integers(0, 0x7F, mlen, dtype=np.uint8) | (rng.integers(0, 2, mlen, dtype=np.uint8) << 7)
            b["m"][:] = m
            b["m_scale"][:] = np.exp(rng.uniform(np.log(1e-4), 0, self.nblocks)).astype(np.float32)
            if "v" in b:
                b["v"][:] = rng.integers(0, 0x7C, mlen, dtype=np.uint8)   # sqrt(v) >= 0, finite
                b["v_scale"][:] = np.exp(rng.uniform(np.log(1e-4), 0, self.nblocks)).astype(np.float32)
            pad = self.nblocks * FP8_BLOCK - self.n
            if pad:   # the padding of the last block is zero, as the kernels leave it
                b["m"][self.n:] = 0
                if "v" in b:
                    b["v"][self.n:] = 0
            return self
        m = (rng.uniform(-1, 1, mlen) * 1e-2).astype(np.float32)
        v = (rng.uniform(0, 1, mlen) * 1e-3).astype(np.float32)
        b["m"][:] = bf16_bits(m) if self.mv_dtype == DT_BF16 else m
        if "v" in b:
            b["v"][:] = bf16_bits(v) if self.mv_dtype == DT_BF16 else v
        return self

    def new_grad(self, seed: int, g_scale: float = 0.1) -> None:
        g = (np.random.default_rng(seed).uniform(-1, 1, self.n) * g_scale).astype(np.float32)
        self.buffers["g"][:] = bf16_bits(g) if self.g_dtype == DT_BF16 else g

    def clone(self) -> "HostSegment":
        c = HostSegment(self.n, self.g_dtype, self.mv_dtype, self.out_dtype, self.p_dtype, self.algorithm,
                        self.offset, self.index, self.step)
        c.buffers = {k: v.copy() for k, v in self.buffers.items()}
        return c

    def ctype(self, group: Group | None = None) -> Segment:
        """A Segment pointing at these buffers (keep ``self`` alive while it is used)."""
        b = self.buffers
        ptr = (lambda k: b[k].ctypes.data if k in b else None)
        s = Segment(p=ptr("p"), p_lo=ptr("p_lo"), g=ptr("g"), m=ptr("m"), v=ptr("v"), m_scale=ptr("m_scale"),
                    v_scale=ptr("v_scale"), out=ptr("out"), n=self.n, step=self.step, index=self.index,
                    offset=self.offset, g_dtype=self.g_dtype, mv_dtype=self.mv_dtype, out_dtype=self.out_dtype,
                    algorithm=self.algorithm, p_dtype=self.p_dtype)
        if group is not None:
            s.group = ctypes.pointer(group)
        return s

    def master_f32(self) -> np.ndarray:
        b = self.buffers
        return f24_to_f32(b["p"], b["p_lo"]) if self.p_dtype == DT_F24 else b["p"]

    def mismatches(self, other: "HostSegment") -> dict[str, int]:
        """Per-buffer count of elements whose bits differ (NaN == NaN whatever the payload)."""
        bad = {}
        for k, a in self.buffers.items():
            if k == "g":
                continue
            o = other.buffers[k]
            if a.dtype == np.float32:
                diff = (a.view(np.uint32) != o.view(np.uint32)) & ~(np.isnan(a) & np.isnan(o))
            elif a.dtype == np.uint16 and k in ("m", "v", "out") or (k == "p" and self.p_dtype == DT_F24):
                fa, fo = bf16_to_f32(a), bf16_to_f32(o)
                diff = (a != o) & ~(np.isnan(fa) & np.isnan(fo))
            else:
                diff = a != o
            if diff.any():
                bad[k] = int(diff.sum())
        return bad


def default_level() -> int:
    """The SIMD level to reproduce: the reference library's active level where it is built, else AVX-512."""
    env = os.environ.get("ABX_SIMD_LEVEL")
    if env is not None:
        return int(env)
    ref = load_reference()
    return ref.simd_level if ref is not None else SIMD_AVX512
