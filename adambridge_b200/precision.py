"""Storage formats of the master weights and the moments, resident in GPU memory.

Same formats, class names and checkpoint dicts as adambridge's ``precision.py``
(adambridge/precision.py), but every buffer lives on the parameter's CUDA device so
the fused kernels read and write it in place:

==========  =================  ====================  ===============
precision   first moment m     second moment v       bytes / param*
==========  =================  ====================  ===============
fp32        FP32               FP32                  12
bf16        BF16               BF16                  8
fp8         E4M3 + block scale E5M2 + block scale    ~6.06
==========  =================  ====================  ===============

\\* with an FP32 master weight; an FP24 master (bf16 plane + one byte) takes 3.

The hot path touches only ``native_buffers``.  ``read`` / ``write`` / ``to_fp32``
serve format conversion (``set_precision``, checkpoints) and use torch operations
on the device; their rounding follows the reference's conversions (nearest-even,
or the lowbias32 stochastic stream keyed by element index).
"""

from __future__ import annotations

import math
from abc import ABC, abstractmethod
from typing import Any

import torch

__all__ = [
    "PRECISIONS", "MASTER_PRECISIONS", "FP8_BLOCK", "canonical_precision", "canonical_master_precision",
    "MomentStore", "FP32Store", "BF16Store", "FP8Store", "FP24Store", "make_store", "make_master",
    "store_from_state_dict", "check_master_state", "load_master_", "master_to_fp32", "bytes_per_param",
    "round_to_bf16_stochastic", "round_to_fp8_stochastic", "round_to_fp24_stochastic", "round_to_fp24_nearest_",
    "moment_seed", "random_bits",
]

_ALIASES = {"fp32": "fp32", "float32": "fp32", "bf16": "bf16", "bf16_moments": "bf16", "bfloat16": "bf16",
            "fp8": "fp8", "fp8_moments": "fp8"}
PRECISIONS = ("fp32", "bf16", "fp8")
_MASTER_ALIASES = {"fp32": "fp32", "float32": "fp32", "fp24": "fp24", "float24": "fp24"}
MASTER_PRECISIONS = ("fp32", "fp24")

FP8_BLOCK = 128
_FP8_FORMATS = {
    # role -> (dtype, max finite value, mantissa bits)   (adambridge/precision.py:79-83)
    "m": (torch.float8_e4m3fn, 448.0, 3),
    "v": (torch.float8_e5m2, 57344.0, 2),
}


def canonical_precision(name: str) -> str:
    try:
        return _ALIASES[name.lower()]
    except (KeyError, AttributeError):
        raise ValueError(f"unknown precision {name!r}; expected one of {sorted(_ALIASES)}") from None


def canonical_master_precision(name: str) -> str:
    try:
        return _MASTER_ALIASES[name.lower()]
    except (KeyError, AttributeError):
        raise ValueError(f"unknown master precision {name!r}; expected one of {sorted(_MASTER_ALIASES)}") from None


def bytes_per_param(precision: str, moments: int = 2, master: str = "fp32") -> float:
    """Device bytes per parameter for the master + ``moments`` moment vectors (AdamW 2, Lion 1)."""
    moment = {"fp32": 4.0, "bf16": 2.0, "fp8": 1.0 + 4.0 / FP8_BLOCK}[canonical_precision(precision)]
    return {"fp32": 4.0, "fp24": 3.0}[canonical_master_precision(master)] + moments * moment


# ---------------------------------------------------------------- stochastic rounding (conversions)

def _hash32(x: int) -> int:
    x &= 0xFFFFFFFF
    x ^= x >> 16
    x = (x * 0x7FEB352D) & 0xFFFFFFFF
    x ^= x >> 15
    x = (x * 0x846CA68B) & 0xFFFFFFFF
    x ^= x >> 16
    return x


def moment_seed(seed: int, role: str) -> int:
    """32-bit rounding stream of ``role``: 'm', 'v' or 'p' (the fp24 master), as the kernels derive it."""
    seed &= 0xFFFFFFFF
    if role == "m":
        return seed
    return _hash32(seed ^ (0xA511E9B3 if role == "v" else 0x6C8E9CF5))


def _to_i32(value: int) -> int:
    value &= 0xFFFFFFFF
    return value - (1 << 32) if value >= 1 << 31 else value


def random_bits(offset: int, n: int, seed: int, device: torch.device | str = "cpu") -> torch.Tensor:
    """lowbias32(index ^ seed) for indices ``offset .. offset+n-1`` as int32 bit patterns."""
    x = (torch.arange(offset, offset + n, dtype=torch.int64, device=device) & 0xFFFFFFFF)
    x = x.to(torch.int32) if offset + n <= 1 << 31 else (x - ((x >= 1 << 31).long() << 32)).to(torch.int32)
    x.bitwise_xor_(_to_i32(seed))
    x.bitwise_xor_(x.bitwise_right_shift(16).bitwise_and_(0xFFFF))
    x.mul_(0x7FEB352D)
    x.bitwise_xor_(x.bitwise_right_shift(15).bitwise_and_(0x1FFFF))
    x.mul_(_to_i32(0x846CA68B))
    x.bitwise_xor_(x.bitwise_right_shift(16).bitwise_and_(0xFFFF))
    return x


def _stochastic_truncate_(x: torch.Tensor, dropped_bits: int, offset: int, seed: int) -> torch.Tensor:
    noise = random_bits(offset, x.numel(), seed, x.device).bitwise_and_((1 << dropped_bits) - 1)
    x.view(torch.int32).add_(noise).bitwise_and_(-(1 << dropped_bits))
    return x


def round_to_bf16_stochastic(x: torch.Tensor, seed: int, offset: int = 0) -> torch.Tensor:
    """FP32 ``x`` stochastically rounded to bf16 (``x`` is clobbered)."""
    return _stochastic_truncate_(x, 16, offset, seed).to(torch.bfloat16)


def round_to_fp8_stochastic(x: torch.Tensor, dtype: torch.dtype, seed: int, offset: int = 0) -> torch.Tensor:
    _, fmax, mbits = next(f for f in _FP8_FORMATS.values() if f[0] == dtype)
    _stochastic_truncate_(x, 23 - mbits, offset, seed)
    return x.clamp_(-fmax, fmax).to(dtype)


def round_to_fp24_stochastic(x: torch.Tensor, seed: int, offset: int = 0) -> torch.Tensor:
    return _stochastic_truncate_(x, 8, offset, seed)


def round_to_fp24_nearest_(x: torch.Tensor) -> torch.Tensor:
    """Round FP32 ``x`` in place to its top 24 bits, nearest even; NaN stays NaN."""
    b = x.view(torch.int32)
    nan = x.isnan()
    quiet = b.bitwise_or(0x00400000)
    b.add_(b.bitwise_right_shift(8).bitwise_and_(1).add_(0x7F)).bitwise_and_(~0xFF)
    b.copy_(torch.where(nan, quiet, b))
    return x


# ---------------------------------------------------------------- stores

class MomentStore(ABC):
    """One moment vector (or master) of one parameter, flat, on ``device``."""

    precision: str

    def __init__(self, numel: int, device: torch.device | str | None = None):
        self.numel = numel
        self.device = torch.device(device) if device is not None else torch.device("cpu")

    @abstractmethod
    def read(self, lo: int, hi: int) -> torch.Tensor: ...

    @abstractmethod
    def write(self, lo: int, hi: int, x: torch.Tensor, seed: int | None = None) -> None: ...

    @abstractmethod
    def to_fp32(self) -> torch.Tensor: ...

    @property
    @abstractmethod
    def nbytes(self) -> int: ...

    @property
    def native_buffers(self) -> tuple[torch.Tensor, torch.Tensor | None]:
        """(values or codes, per-block scales or None) in the kernels' layout."""
        raise NotImplementedError

    @property
    def chunk_alignment(self) -> int:
        return 1

    @abstractmethod
    def state_dict(self) -> dict[str, Any]: ...


class FP32Store(MomentStore):
    precision = "fp32"

    def __init__(self, numel: int, init: torch.Tensor | None = None, device=None):
        super().__init__(numel, device)
        self.data = torch.zeros(numel, dtype=torch.float32, device=self.device)
        if init is not None:
            self.data.copy_(init.reshape(-1))

    @classmethod
    def wrap(cls, data: torch.Tensor) -> "FP32Store":
        """A store over an existing flat FP32 tensor (an FP32 parameter updated in place)."""
        store = cls.__new__(cls)
        MomentStore.__init__(store, data.numel(), data.device)
        store.data = data
        return store

    def read(self, lo, hi):
        return self.data[lo:hi]

    def write(self, lo, hi, x, seed=None):
        dst = self.data[lo:hi]
        if x.data_ptr() != dst.data_ptr():
            dst.copy_(x)

    def to_fp32(self):
        return self.data.clone()

    @property
    def nbytes(self):
        return self.data.nbytes

    @property
    def native_buffers(self):
        return self.data, None

    def state_dict(self):
        return {"precision": "fp32", "data": self.data}


class BF16Store(MomentStore):
    precision = "bf16"

    def __init__(self, numel: int, init: torch.Tensor | None = None, device=None):
        super().__init__(numel, device)
        self.data = torch.zeros(numel, dtype=torch.bfloat16, device=self.device)
        if init is not None:
            self.data.copy_(init.reshape(-1))   # nearest-even

    def read(self, lo, hi):
        return self.data[lo:hi].float()

    def write(self, lo, hi, x, seed=None):
        if seed is not None:
            self.data[lo:hi].copy_(round_to_bf16_stochastic(x.to(self.device), seed, lo))
        else:
            self.data[lo:hi].copy_(x)

    def to_fp32(self):
        return self.data.float()

    @property
    def nbytes(self):
        return self.data.nbytes

    @property
    def native_buffers(self):
        return self.data, None

    def state_dict(self):
        return {"precision": "bf16", "data": self.data}


class FP8Store(MomentStore):
    """FP8 codes with one FP32 scale per ``block`` elements (absmax / format max).  The second moment is kept
    as sqrt(v), so ``m`` underflows before ``v`` does (adambridge/precision.py:341-418)."""

    precision = "fp8"

    def __init__(self, numel: int, role: str, init: torch.Tensor | None = None, block: int = FP8_BLOCK,
                 device=None):
        super().__init__(numel, device)
        if role not in _FP8_FORMATS:
            raise ValueError(f"role must be 'm' or 'v', got {role!r}")
        self.role = role
        self.block = block
        self.dtype, self.fmax, _ = _FP8_FORMATS[role]
        self.sqrt_domain = role == "v"
        nblocks = max(1, math.ceil(numel / block))
        self.q = torch.zeros(nblocks * block, dtype=self.dtype, device=self.device)
        self.scale = torch.ones(nblocks, dtype=torch.float32, device=self.device)
        if init is not None:
            self.write(0, numel, init.reshape(-1).to(self.device, torch.float32).clone())

    @property
    def chunk_alignment(self):
        return self.block

    def read(self, lo, hi):
        b0, b1 = lo // self.block, math.ceil(hi / self.block)
        x = self.q[b0 * self.block: b1 * self.block].float().view(-1, self.block)
        x.mul_(self.scale[b0:b1, None])
        if self.sqrt_domain:
            x.square_()
        off = lo - b0 * self.block
        return x.view(-1)[off: off + hi - lo]

    def write(self, lo, hi, x, seed=None):
        n = hi - lo
        b0, b1 = lo // self.block, math.ceil(hi / self.block)
        x = x.to(self.device, torch.float32)
        if self.sqrt_domain:
            x = x.clamp_(min=0).sqrt_()
        padded = (b1 - b0) * self.block
        if padded != n:
            x = torch.nn.functional.pad(x, (0, padded - n))
        xb = x.view(-1, self.block)
        amax = xb.abs().amax(dim=1)
        scale = torch.where(amax > 0, amax / self.fmax, torch.ones_like(amax))
        xb.div_(scale[:, None])
        flat = xb.view(-1)
        if seed is not None:
            q = round_to_fp8_stochastic(flat, self.dtype, seed, b0 * self.block)
        else:
            q = flat.clamp_(-self.fmax, self.fmax).to(self.dtype)
        self.q[b0 * self.block: b1 * self.block].copy_(q)
        self.scale[b0:b1].copy_(scale)

    def to_fp32(self):
        return self.read(0, self.numel).clone()

    @property
    def nbytes(self):
        return self.q.nbytes + self.scale.nbytes

    @property
    def native_buffers(self):
        if self.block != FP8_BLOCK:
            raise ValueError("the kernels implement the 128-element FP8 block only")
        return self.q, self.scale

    def state_dict(self):
        return {"precision": "fp8", "role": self.role, "block": self.block, "q": self.q, "scale": self.scale}


class FP24Store(MomentStore):
    """The FP24 master: the top 24 bits of each FP32 value as a bf16 plane ``hi`` and a byte plane ``lo``."""

    precision = "fp24"
    INIT_CHUNK = 1 << 24

    def __init__(self, numel: int, init: torch.Tensor | None = None, device=None):
        super().__init__(numel, device)
        self.hi = torch.zeros(numel, dtype=torch.bfloat16, device=self.device)
        self.lo = torch.zeros(numel, dtype=torch.uint8, device=self.device)
        if init is not None:
            self.init_from_(init)

    def init_from_(self, src: torch.Tensor) -> None:
        src = src.detach().reshape(-1)
        if src.dtype == torch.bfloat16:
            self.hi.copy_(src)
            self.lo.zero_()
            return
        for lo in range(0, self.numel, self.INIT_CHUNK):
            hi = min(lo + self.INIT_CHUNK, self.numel)
            self.write(lo, hi, src[lo:hi].to(self.device, torch.float32, copy=True))

    def read(self, lo, hi):
        bits = (self.hi[lo:hi].view(torch.int16).to(torch.int32) & 0xFFFF) << 16
        bits |= self.lo[lo:hi].to(torch.int32) << 8
        return bits.view(torch.float32)

    def write(self, lo, hi, x, seed=None):
        x = x.to(self.device, torch.float32).contiguous()
        if seed is not None:
            round_to_fp24_stochastic(x, seed, lo)
        else:
            round_to_fp24_nearest_(x)
        b = x.view(torch.int32)
        self.hi[lo:hi].view(torch.int16).copy_((b >> 16).to(torch.int16))
        self.lo[lo:hi].copy_(((b >> 8) & 0xFF).to(torch.uint8))

    def to_fp32(self):
        return self.read(0, self.numel)

    @property
    def nbytes(self):
        return self.hi.nbytes + self.lo.nbytes

    @property
    def native_buffers(self):
        return self.hi, self.lo

    def state_dict(self):
        return {"precision": "fp24", "hi": self.hi, "lo": self.lo}


def make_store(precision: str, numel: int, role: str, init: torch.Tensor | None = None, device=None) -> MomentStore:
    """Allocate a moment store on ``device``; ``role`` is 'm' or 'v' (picks the FP8 format)."""
    precision = canonical_precision(precision)
    if precision == "fp32":
        return FP32Store(numel, init, device)
    if precision == "bf16":
        return BF16Store(numel, init, device)
    return FP8Store(numel, role, init, device=device)


def make_master(precision: str, numel: int, init: torch.Tensor | None = None, device=None) -> MomentStore:
    precision = canonical_master_precision(precision)
    if precision == "fp24":
        return FP24Store(numel, init, device)
    return FP32Store(numel, init, device)


def _checked(t: Any, numel: int, what: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"checkpoint {what} is {type(t).__name__}, expected a tensor")
    if t.numel() != numel:
        raise ValueError(f"checkpoint {what} has {t.numel()} elements, expected {numel} (a different model?)")
    return t


def check_master_state(saved: Any, numel: int, what: str) -> None:
    """Validate a checkpoint's master weights: an FP32 tensor, or an fp32/fp24 store dict."""
    if isinstance(saved, torch.Tensor):
        _checked(saved, numel, what)
        return
    if not isinstance(saved, dict) or saved.get("precision") not in MASTER_PRECISIONS:
        raise ValueError(f"checkpoint {what}: expected a tensor or an fp32/fp24 store, got "
                         f"{saved.get('precision') if isinstance(saved, dict) else type(saved).__name__!r}")
    if saved["precision"] == "fp24":
        if _checked(saved.get("hi"), numel, f"{what} (hi plane)").dtype != torch.bfloat16:
            raise ValueError(f"checkpoint {what}: the hi plane must be bfloat16")
        if _checked(saved.get("lo"), numel, f"{what} (lo plane)").dtype != torch.uint8:
            raise ValueError(f"checkpoint {what}: the lo plane must be uint8")
    else:
        _checked(saved.get("data"), numel, what)


def master_to_fp32(saved: Any, numel: int, device=None) -> torch.Tensor:
    if isinstance(saved, torch.Tensor):
        return saved.detach().reshape(-1).to(device or saved.device, torch.float32)
    if saved["precision"] == "fp24":
        store = FP24Store(numel, device=device or saved["hi"].device)
        store.hi.copy_(saved["hi"].reshape(-1))
        store.lo.copy_(saved["lo"].reshape(-1))
        return store.to_fp32()
    return saved["data"].detach().reshape(-1).to(device or saved["data"].device, torch.float32)


def load_master_(store: MomentStore, saved: Any) -> None:
    """Load validated checkpoint master weights into ``store`` (converting fp32 <-> fp24)."""
    if isinstance(store, FP24Store) and isinstance(saved, dict) and saved.get("precision") == "fp24":
        store.hi.copy_(saved["hi"].reshape(-1))
        store.lo.copy_(saved["lo"].reshape(-1))
        return
    x = master_to_fp32(saved, store.numel, store.device)
    if isinstance(store, FP32Store):
        store.data.copy_(x)
        return
    store.write(0, store.numel, x.clone())


def store_from_state_dict(state: dict[str, Any], numel: int, role: str, device=None) -> MomentStore:
    """Rebuild a moment store from a checkpoint, validating every field first."""
    if not isinstance(state, dict) or state.get("precision") not in PRECISIONS:
        raise ValueError("checkpoint moment store has unknown precision "
                         f"{state.get('precision') if isinstance(state, dict) else state!r}")
    precision = state["precision"]
    if precision == "fp8":
        saved_role, block = state.get("role", role), state.get("block")
        if saved_role not in _FP8_FORMATS:
            raise ValueError(f"checkpoint FP8 store has unknown role {saved_role!r}")
        if not isinstance(block, int) or isinstance(block, bool) or not 0 < block <= 1 << 20:
            raise ValueError(f"checkpoint FP8 store has invalid block size {block!r}")
        store = FP8Store(numel, saved_role, block=block, device=device)
        store.q.copy_(_checked(state.get("q"), store.q.numel(), "FP8 codes"))
        store.scale.copy_(_checked(state.get("scale"), store.scale.numel(), "FP8 scales"))
        if saved_role != role or block != FP8_BLOCK:
            store = FP8Store(numel, role, init=store.to_fp32(), device=device)
        return store
    store = make_store(precision, numel, role, device=device)
    store.data.copy_(_checked(state.get("data"), numel, f"{precision} moments"))
    return store
