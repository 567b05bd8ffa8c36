"""Load libabx, the sm_100a update kernels, and describe work for them.

This is the B200 counterpart of adambridge's ``native.py`` (adambridge/native.py):
the same ctypes structs (``Segment``, ``Group``, ``_HParams``; layouts of
adambridge/csrc/adambridge_kernels.c:77-88, 736-769), the same dtype and algorithm
codes, the same ``StepCoefficients`` and ``mix_seed``, and a ``NativeKernels`` class
with ``multi_step`` / ``multi_apply`` / ``fused_adamw`` / ``make_hparams``.  What
differs: segment pointers are CUDA device pointers, and the first argument of
``multi_step`` / ``multi_apply`` is the CUDA stream the update is enqueued on
(the reference's is a host thread pool).

There is no fallback: if ``adambridge_b200/_lib/libabx.so`` is missing or does not
load, ``load()`` raises.  Build it with ``python -m adambridge_b200._build``.
"""

from __future__ import annotations

import ctypes
import logging
import threading
from dataclasses import dataclass
from pathlib import Path

import torch

from . import _build

__all__ = ["NativeKernels", "Group", "Segment", "State", "StepCoefficients", "load", "build", "available", "mix_seed",
           "SIMD_NAMES", "BuildError", "LIBRARY"]

log = logging.getLogger("adambridge_b200.native")

ABI_VERSION = 1
LIBRARY = _build.LIB
SIMD_NAMES = {0: "scalar", 1: "avx2", 2: "avx512", 3: "neon"}

DT_NONE, DT_F32, DT_BF16, DT_FP8, DT_F24 = 0, 1, 2, 3, 4
_DTYPE_CODES = {torch.float32: DT_F32, torch.bfloat16: DT_BF16}
MOMENT_CODES = {"fp32": DT_F32, "bf16": DT_BF16, "fp8": DT_FP8}
MASTER_CODES = {"fp32": DT_F32, "fp24": DT_F24}
ALGORITHMS = {"adamw": 0, "lion": 1}

ERRORS = {
    -1: "invalid argument", -2: "a required buffer is NULL", -3: "unsupported gradient dtype",
    -4: "unsupported moment dtype", -5: "unsupported out dtype", -6: "out dtype set but out is NULL",
    -7: "FP8 moments without scales", -8: "segment without a group", -9: "too many work items",
    -10: "out of memory", -11: "bad element offset", -12: "unknown algorithm", -13: "unknown master dtype",
    -20: "CUDA error", -21: "misaligned buffer", -22: "unknown SIMD level",
    -23: "gradients exceed the static norm scratch",
}

_MASK64 = (1 << 64) - 1


class BuildError(RuntimeError):
    pass


class Tensor(ctypes.Structure):
    """One gradient for the norm kernels (abx_tensor): device pointer, elements, dtype code."""

    _fields_ = [("data", ctypes.c_void_p), ("n", ctypes.c_int64), ("dtype", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


class State(ctypes.Structure):
    """One optimizer-state buffer for abx_convert (abx_state): its planes, format code, FP8 role and block."""

    _fields_ = [("values", ctypes.c_void_p), ("aux", ctypes.c_void_p), ("dtype", ctypes.c_int32),
                ("role", ctypes.c_int32), ("block", ctypes.c_int64)]


class _HParams(ctypes.Structure):
    _fields_ = [
        ("beta1", ctypes.c_float),
        ("beta2", ctypes.c_float),
        ("one_minus_beta1", ctypes.c_float),
        ("one_minus_beta2", ctypes.c_float),
        ("decay", ctypes.c_float),
        ("step_size", ctypes.c_float),
        ("inv_sqrt_bc2", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("seed", ctypes.c_uint32),
        ("stochastic", ctypes.c_int32),
    ]


class Group(ctypes.Structure):
    """Hyperparameters shared by the segments of one parameter group (abx_group)."""

    _fields_ = [
        ("lr", ctypes.c_double),
        ("beta1", ctypes.c_double),
        ("beta2", ctypes.c_double),
        ("eps", ctypes.c_double),
        ("weight_decay", ctypes.c_double),
        ("seed", ctypes.c_uint64),
        ("stochastic", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class Segment(ctypes.Structure):
    """One tensor's device buffers (abx_segment).  Pointers are raw device addresses."""

    _fields_ = [
        ("p", ctypes.c_void_p),         # fp32 master, or the fp24 hi plane (bfloat16 bits) when p_dtype is DT_F24
        ("p_lo", ctypes.c_void_p),      # fp24 only: the lo plane (uint8)
        ("g", ctypes.c_void_p),
        ("m", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("m_scale", ctypes.c_void_p),
        ("v_scale", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("group", ctypes.POINTER(Group)),
        ("n", ctypes.c_int64),
        ("step", ctypes.c_int64),
        ("index", ctypes.c_uint64),
        ("offset", ctypes.c_int64),
        ("g_dtype", ctypes.c_int32),
        ("mv_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("algorithm", ctypes.c_int32),  # ALGORITHMS; Lion leaves v, v_scale NULL
        ("p_dtype", ctypes.c_int32),    # MASTER_CODES (0 means fp32)
        ("reserved", ctypes.c_int32),
    ]


def mix_seed(*values: int) -> int:
    """Combine integers into a 63-bit seed with splitmix64 rounds; the low 32 bits are the
    kernel's per-step seed (adambridge/kernels.py:29-37, csrc:773-790)."""
    h = 0x9E3779B97F4A7C15
    for v in values:
        h = ((h ^ (v & _MASK64)) * 0xBF58476D1CE4E5B9) & _MASK64
        h ^= h >> 31
        h = (h * 0x94D049BB133111EB) & _MASK64
        h ^= h >> 29
    return h & ((1 << 63) - 1)


@dataclass(frozen=True)
class StepCoefficients:
    """Per-step scalars for the fused update (adambridge/native.py:243-270), in double."""

    beta1: float
    beta2: float
    decay: float
    step_size: float
    inv_sqrt_bc2: float
    eps: float

    @classmethod
    def for_step(cls, lr: float, beta1: float, beta2: float, eps: float, weight_decay: float, step: int):
        bc1 = 1.0 - beta1**step
        bc2 = 1.0 - beta2**step
        return cls(beta1=beta1, beta2=beta2, decay=1.0 - lr * weight_decay, step_size=lr / bc1,
                   inv_sqrt_bc2=1.0 / bc2**0.5, eps=eps)

    @classmethod
    def for_lion(cls, lr: float, beta1: float, beta2: float, weight_decay: float):
        """Lion has no bias correction: the step is ``lr * sign(c)``."""
        return cls(beta1=beta1, beta2=beta2, decay=1.0 - lr * weight_decay, step_size=lr, inv_sqrt_bc2=1.0, eps=0.0)


def dtype_code_of(dtype: torch.dtype | None) -> int:
    """Kernel dtype code of a gradient / out tensor dtype (DT_NONE for None)."""
    if dtype is None:
        return DT_NONE
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise TypeError(f"the kernels read and write float32 or bfloat16 tensors, not {dtype}") from None


def _stream_handle(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class NativeKernels:
    """ctypes wrapper around libabx."""

    def __init__(self, path: Path = LIBRARY):
        self.path = Path(path)
        try:
            lib = ctypes.CDLL(str(self.path))
        except OSError as exc:
            raise BuildError(f"cannot load {self.path}: {exc}") from exc
        lib.abx_abi_version.restype = ctypes.c_int
        if lib.abx_abi_version() != ABI_VERSION:
            raise BuildError(f"{self.path} has ABI {lib.abx_abi_version()}, expected {ABI_VERSION}")
        for fn, struct in (("abx_hparams_size", _HParams), ("abx_group_size", Group), ("abx_segment_size", Segment)):
            getattr(lib, fn).restype = ctypes.c_int
            if getattr(lib, fn)() != ctypes.sizeof(struct):
                raise BuildError(f"{fn}: struct layout mismatch between C and Python")
        for fn in ("abx_simd_level", "abx_detected_simd_level", "abx_set_simd_level"):
            getattr(lib, fn).restype = ctypes.c_int
        lib.abx_set_simd_level.argtypes = [ctypes.c_int]
        seg_array = ctypes.POINTER(ctypes.POINTER(Segment))
        lib.abx_multi_step.restype = ctypes.c_int
        lib.abx_multi_step.argtypes = [ctypes.c_void_p, seg_array, ctypes.c_int32, ctypes.c_int32]
        lib.abx_multi_apply.restype = ctypes.c_int
        lib.abx_multi_apply.argtypes = [ctypes.c_void_p, seg_array, ctypes.POINTER(_HParams), ctypes.c_int32,
                                        ctypes.c_int32]
        lib.abx_multi_step_scaled.restype = ctypes.c_int
        lib.abx_multi_step_scaled.argtypes = [ctypes.c_void_p, seg_array, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]
        lib.abx_multi_step_replicated.restype = ctypes.c_int
        lib.abx_multi_step_replicated.argtypes = [ctypes.c_void_p, seg_array, ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int32]
        lib.abx_replicate_async.restype = ctypes.c_int
        lib.abx_replicate_async.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_int64,
                                            ctypes.POINTER(ctypes.c_int64), ctypes.c_int32]
        lib.abx_multi_apply_scaled.restype = ctypes.c_int
        lib.abx_multi_apply_scaled.argtypes = [ctypes.c_void_p, seg_array, ctypes.POINTER(_HParams), ctypes.c_int32,
                                               ctypes.c_int32, ctypes.c_void_p]
        lib.abx_fused_adamw.restype = ctypes.c_int
        lib.abx_fused_adamw.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                                        ctypes.c_uint64, ctypes.POINTER(_HParams), ctypes.c_void_p]
        lib.abx_hparams_for.restype = ctypes.c_int
        lib.abx_hparams_for.argtypes = [ctypes.POINTER(Segment), ctypes.POINTER(_HParams)]
        lib.abx_step_seed.restype = ctypes.c_uint32
        lib.abx_step_seed.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64]
        lib.abx_last_error.restype = ctypes.c_char_p
        lib.abx_launch_count.restype = ctypes.c_uint64
        lib.abx_pipeline_status.restype = ctypes.c_int
        lib.abx_status_word.restype = ctypes.POINTER(ctypes.c_uint)
        lib.abx_convert.restype = ctypes.c_int
        lib.abx_convert.argtypes = [ctypes.c_void_p, ctypes.POINTER(State), ctypes.POINTER(State), ctypes.c_int64]
        lib.abx_test_pipeline_fault.restype = ctypes.c_int
        lib.abx_test_pipeline_fault.argtypes = [ctypes.c_int64, ctypes.c_uint32]
        tens = ctypes.POINTER(Tensor)
        lib.abx_clip_workspace_bytes.restype = ctypes.c_size_t
        lib.abx_clip_workspace_bytes.argtypes = [tens, ctypes.c_int32]
        lib.abx_grad_sq_norms.restype = ctypes.c_int
        lib.abx_grad_sq_norms.argtypes = [ctypes.c_void_p, tens, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_size_t]
        lib.abx_clip_coef_from_sq.restype = ctypes.c_int
        lib.abx_clip_coef_from_sq.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
        lib.abx_clip_coef.restype = ctypes.c_int
        lib.abx_clip_coef.argtypes = [ctypes.c_void_p, tens, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        lib.abx_clip_coef_noalloc.restype = ctypes.c_int
        lib.abx_clip_coef_noalloc.argtypes = [ctypes.c_void_p, tens, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_void_p]
        self._lib = lib

    # -- rounding pattern ----------------------------------------------------

    @property
    def simd_level(self) -> str:
        return SIMD_NAMES[self._lib.abx_simd_level()]

    @property
    def detected_simd_level(self) -> str:
        return SIMD_NAMES[self._lib.abx_detected_simd_level()]

    def set_simd_level(self, name: str | None) -> str:
        """Reproduce the rounding of the reference built for SIMD level ``name`` (``None``: AVX-512)."""
        code = -1 if name is None else {v: k for k, v in SIMD_NAMES.items()}[name]
        return SIMD_NAMES[self._lib.abx_set_simd_level(code)]

    # -- capability queries (adambridge/native.py:327-337) ---------------------

    @staticmethod
    def supports(grad_dtype: torch.dtype, moment_precision: str, out_dtype: torch.dtype | None) -> bool:
        return (grad_dtype in _DTYPE_CODES and moment_precision in MOMENT_CODES
                and (out_dtype is None or out_dtype in _DTYPE_CODES))

    @staticmethod
    def dtype_code(dtype: torch.dtype | None) -> int:
        return DT_NONE if dtype is None else _DTYPE_CODES[dtype]

    # -- batched updates -----------------------------------------------------

    @staticmethod
    def segment_array(segments: list) -> ctypes.Array:
        """Array of pointers for multi_step/multi_apply; ``segments`` holds Segment pointers."""
        return (ctypes.POINTER(Segment) * len(segments))(*segments)

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            detail = self._lib.abx_last_error().decode() if rc in (-20, -21, -23) else ERRORS.get(rc, "")
            raise RuntimeError(f"{what} rejected the update (code {rc}: {detail})")

    def multi_step(self, stream, segments: ctypes.Array, max_ctas: int = 0, g_scale: torch.Tensor | None = None) -> None:
        """Enqueue the update of every segment on ``stream`` (a torch.cuda.Stream, a raw handle, or None for the
        current stream); coefficients come from each segment's group and step."""
        if g_scale is None:
            rc = self._lib.abx_multi_step(_stream_handle(stream), segments, len(segments), max_ctas)
        else:
            rc = self._lib.abx_multi_step_scaled(_stream_handle(stream), segments, len(segments), max_ctas,
                                                 _scale_ptr(g_scale))
        self._check(rc, "abx_multi_step")

    def multi_step_replicated(self, stream, segments: ctypes.Array, out_deltas: list[int], max_ctas: int = 0,
                              g_scale: torch.Tensor | None = None) -> None:
        """multi_step, also storing every new weight at out + delta for each of ``out_deltas`` (bytes): the
        peers' copies of a symmetric weight buffer (the all-gather of a sharded update, fused into it)."""
        deltas = (ctypes.c_int64 * max(1, len(out_deltas)))(*out_deltas)
        rc = self._lib.abx_multi_step_replicated(_stream_handle(stream), segments, len(segments), max_ctas,
                                                 None if g_scale is None else _scale_ptr(g_scale), deltas,
                                                 len(out_deltas))
        self._check(rc, "abx_multi_step_replicated")

    def replicate_async(self, streams: list, src: int, nbytes: int, deltas: list[int]) -> None:
        """Copy ``nbytes`` bytes at device address ``src`` to ``src + deltas[j]`` on ``streams[j]`` (copy
        engines): the all-gather of a sharded update into the peers' copies of a symmetric weight buffer."""
        if len(streams) != len(deltas):
            raise ValueError("one stream per replica")
        hs = (ctypes.c_void_p * max(1, len(streams)))(*[_stream_handle(s) for s in streams])
        ds = (ctypes.c_int64 * max(1, len(deltas)))(*deltas)
        rc = self._lib.abx_replicate_async(hs, src, nbytes, ds, len(deltas))
        self._check(rc, "abx_replicate_async")

    def multi_apply(self, stream, segments: ctypes.Array, hparams: list, max_ctas: int = 0,
                    g_scale: torch.Tensor | None = None) -> None:
        """Like multi_step with explicit coefficients, one ``_HParams`` per segment."""
        hps = (_HParams * len(hparams))(*hparams)
        if g_scale is None:
            rc = self._lib.abx_multi_apply(_stream_handle(stream), segments, hps, len(segments), max_ctas)
        else:
            rc = self._lib.abx_multi_apply_scaled(_stream_handle(stream), segments, hps, len(segments), max_ctas,
                                                  _scale_ptr(g_scale))
        self._check(rc, "abx_multi_apply")

    def hparams_for(self, seg: Segment) -> _HParams:
        h = _HParams()
        self._check(self._lib.abx_hparams_for(ctypes.byref(seg), ctypes.byref(h)), "abx_hparams_for")
        return h

    def step_seed(self, base: int, index: int, step: int) -> int:
        return self._lib.abx_step_seed(base & _MASK64, index & _MASK64, step)

    def launch_count(self) -> int:
        """Kernel launches made by libabx in this process so far."""
        return self._lib.abx_launch_count()

    # -- gradient norms and the clipping coefficient ---------------------------

    @staticmethod
    def tensor_array(tensors: list[torch.Tensor]) -> ctypes.Array:
        arr = (Tensor * max(1, len(tensors)))()
        for i, t in enumerate(tensors):
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError("gradients must be contiguous CUDA tensors")
            arr[i] = Tensor(t.data_ptr(), t.numel(), dtype_code_of(t.dtype), 0)
        return arr

    def clip_workspace_bytes(self, arr: ctypes.Array, n: int) -> int:
        return self._lib.abx_clip_workspace_bytes(arr, n)

    def grad_sq_norms(self, stream, arr: ctypes.Array, n: int, sq: torch.Tensor, workspace: torch.Tensor) -> None:
        """sq[i] = sum of squares of gradient i (fp32, deterministic order)."""
        rc = self._lib.abx_grad_sq_norms(_stream_handle(stream), arr, n, sq.data_ptr(), workspace.data_ptr(),
                                         workspace.numel() * workspace.element_size())
        self._check(rc, "abx_grad_sq_norms")

    def clip_coef_from_sq(self, stream, sq: torch.Tensor, dtype: torch.dtype, max_norm: float,
                          norms: torch.Tensor | None, total_coef: torch.Tensor) -> None:
        rc = self._lib.abx_clip_coef_from_sq(_stream_handle(stream), sq.data_ptr(), sq.numel(), dtype_code_of(dtype),
                                             float(max_norm), None if norms is None else norms.data_ptr(),
                                             total_coef.data_ptr())
        self._check(rc, "abx_clip_coef_from_sq")

    def clip_coef(self, stream, arr: ctypes.Array, n: int, max_norm: float, sq: torch.Tensor,
                  norms: torch.Tensor | None, total_coef: torch.Tensor, workspace: torch.Tensor) -> None:
        """abx_clip_coef: sums of squares, norms, total norm and coefficient, with a caller workspace."""
        rc = self._lib.abx_clip_coef(_stream_handle(stream), arr, n, float(max_norm), sq.data_ptr(),
                                     None if norms is None else norms.data_ptr(), total_coef.data_ptr(),
                                     workspace.data_ptr(), workspace.numel() * workspace.element_size())
        self._check(rc, "abx_clip_coef")

    def clip_coef_noalloc(self, stream, arr: ctypes.Array, n: int, max_norm: float, sq: torch.Tensor,
                          norms: torch.Tensor | None, total_coef: torch.Tensor) -> None:
        """abx_clip_coef_noalloc: the same results with the library's static device scratch (no workspace,
        nothing allocated; calls that overlap on one device race on the scratch)."""
        rc = self._lib.abx_clip_coef_noalloc(_stream_handle(stream), arr, n, float(max_norm), sq.data_ptr(),
                                             None if norms is None else norms.data_ptr(), total_coef.data_ptr())
        self._check(rc, "abx_clip_coef_noalloc")

    def pipeline_status(self) -> int:
        """The status word's bits -- nonzero if an update kernel's bounded pipeline wait gave up since the last
        call (1: a consumer's wait for a tile, 2: the producer's wait for a free stage, 4: its wait for its last
        copies) -- then cleared.  No synchronization: it covers the kernels that have finished."""
        rc = self._lib.abx_pipeline_status()
        if rc < 0:
            self._check(rc, "abx_pipeline_status")
        return rc

    def status_pending(self) -> bool:
        """Whether the status word is set, read from mapped host memory without clearing it or any CUDA call."""
        w = self._lib.abx_status_word()
        return bool(w) and w[0] != 0

    def check_status(self, where: str) -> None:
        """Raise if an update kernel that has finished gave up a pipeline wait: its tensors were left partly
        updated.  Clears the word."""
        if self.status_pending():
            bits = self.pipeline_status()
            raise RuntimeError(f"{where}: an update kernel's pipeline wait gave up (status {bits:#x}); the "
                               "optimizer state of this step is incomplete and should be restored from a checkpoint")

    def test_pipeline_fault(self, tile: int, spin_limit: int = 0) -> None:
        """Failure-path tests only: the next launch skips tile ``tile`` (no copy, no arrival), and every wait
        gives up after ``spin_limit`` polls from now on (0: the default).  See abx_test_pipeline_fault."""
        self._lib.abx_test_pipeline_fault(int(tile), int(spin_limit))

    def convert(self, stream, src: State, dst: State, n: int) -> None:
        """Enqueue the conversion of n values from state buffer ``src`` to ``dst`` (abx_convert) on ``stream``."""
        rc = self._lib.abx_convert(_stream_handle(stream), ctypes.byref(src), ctypes.byref(dst), int(n))
        self._check(rc, "abx_convert")

    @staticmethod
    def make_hparams(c: StepCoefficients, seed: int, stochastic: bool) -> _HParams:
        return _HParams(c.beta1, c.beta2, 1.0 - c.beta1, 1.0 - c.beta2, c.decay, c.step_size, c.inv_sqrt_bc2, c.eps,
                        seed & 0xFFFFFFFF, int(stochastic))

    def fused_adamw(self, master: torch.Tensor, grad: torch.Tensor, m: torch.Tensor, v: torch.Tensor,
                    out: torch.Tensor | None, hp: _HParams, lo: int, hi: int, stream=None) -> None:
        """Update elements ``[lo, hi)`` of flat contiguous CUDA tensors in place (adambridge/native.py:389-435)."""
        n = master.numel()
        tensors = {"master": master, "grad": grad, "m": m, "v": v, **({} if out is None else {"out": out})}
        for name, t in tensors.items():
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous CUDA tensor")
            if t.device != master.device:
                raise ValueError(f"{name} is on {t.device}, master on {master.device}")
            if t.numel() != n:
                raise ValueError(f"{name} has {t.numel()} elements, master has {n}")
        if master.dtype != torch.float32:
            raise TypeError("master must be float32")
        for name, t in tensors.items():
            if name != "master" and t.dtype not in _DTYPE_CODES:
                raise TypeError(f"{name} must be float32 or bfloat16, got {t.dtype}")
        if m.dtype != v.dtype:
            raise TypeError("m and v must have the same dtype")
        if not 0 <= lo <= hi <= n:
            raise IndexError(f"range [{lo}, {hi}) outside 0..{n}")
        with torch.cuda.device(master.device):
            rc = self._lib.abx_fused_adamw(
                master.data_ptr() + lo * 4, grad.data_ptr() + lo * grad.element_size(), _DTYPE_CODES[grad.dtype],
                m.data_ptr() + lo * m.element_size(), v.data_ptr() + lo * v.element_size(), _DTYPE_CODES[m.dtype],
                None if out is None else out.data_ptr() + lo * out.element_size(),
                DT_NONE if out is None else _DTYPE_CODES[out.dtype], hi - lo, lo, ctypes.byref(hp),
                _stream_handle(stream))
        self._check(rc, "abx_fused_adamw")


def _scale_ptr(g_scale: torch.Tensor) -> int:
    if not (g_scale.is_cuda and g_scale.dtype == torch.float32 and g_scale.numel() == 1):
        raise TypeError("g_scale must be a one-element float32 CUDA tensor")
    return g_scale.data_ptr()


_lock = threading.Lock()
_loaded: NativeKernels | None = None


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile libabx in-tree (nvcc, sm_100a)."""
    return _build.build(force=force, verbose=verbose)


def load() -> NativeKernels:
    """The loaded library.  Raises if it is missing: there is no other implementation of the update."""
    global _loaded
    with _lock:
        if _loaded is None:
            if not LIBRARY.exists():
                raise BuildError(f"{LIBRARY} is missing; build it with `python -m adambridge_b200._build`")
            _loaded = NativeKernels(LIBRARY)
        return _loaded


def available() -> bool:
    try:
        load()
        return True
    except BuildError:
        return False
