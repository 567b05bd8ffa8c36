"""The optimizer state's storage formats in GPU memory, their checkpoint form, and conversion between them.

Each parameter (or ZeRO shard) owns a master-weight buffer and one moment buffer per moment (AdamW two, Lion
one).  A :class:`StateBuffer` holds ``numel`` values in one *format*, stored as the planes the update kernels
address directly::

    format  planes                                                  bytes / value   holds
    fp32    data   float32[numel]                                   4               master, moments
    bf16    data   bfloat16[numel]                                  2               moments
    fp8     q      codes[ceil(numel / 128) * 128]: E4M3 of m,       1 + 4/128       moments
                   E5M2 of sqrt(v) (the role decides)
            scale  float32 per 128-value block
    fp24    hi     bfloat16[numel] (the top 16 bits of the fp32)    3               master
            lo     uint8[numel]    (the next 8 bits)

The formats and their checkpoint dicts are the reference's (adambridge/precision.py:1-27, 286-480), so a
checkpoint written by either side loads in the other.  What differs is where the work happens: the buffers live
in HBM, and a change of format -- ``set_precision``, a checkpoint saved in another precision or by
``torch.optim.AdamW``, an fp24 master made from the weights, a decoded master for ``master_params()`` -- is one
launch of libabx's conversion kernel (``abx_convert``) on the buffer's GPU, with the reference's roundings
(nearest-even; an FP8 block scaled by its absmax).  Only plane copies ever cross PCIe.

A checkpoint is validated in full (:meth:`StateBuffer.from_checkpoint`, :func:`check_master`) before anything
is loaded, so a mismatched one changes nothing.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from . import native

__all__ = ["BLOCK", "MOMENT_FORMATS", "MASTER_FORMATS", "StateBuffer", "moment_format", "master_format",
           "bytes_per_param", "check_master", "check_moment"]

BLOCK = 128                      # FP8 values per block scale (the kernels' block)
MAX_CHECKPOINT_BLOCK = 1 << 20   # the largest FP8 block a checkpoint may declare
ROLES = ("m", "v", "p")          # first moment, second moment, master weights


@dataclass(frozen=True)
class _Format:
    code: int                     # libabx dtype code
    planes: tuple[str, ...]       # plane names, kernel operand order
    value_bytes: float            # bytes per stored value


_FORMATS = {
    "fp32": _Format(native.DT_F32, ("data",), 4.0),
    "bf16": _Format(native.DT_BF16, ("data",), 2.0),
    "fp8": _Format(native.DT_FP8, ("q", "scale"), 1.0 + 4.0 / BLOCK),
    "fp24": _Format(native.DT_F24, ("hi", "lo"), 3.0),
}
MOMENT_FORMATS = ("fp32", "bf16", "fp8")
MASTER_FORMATS = ("fp32", "fp24")
_MOMENT_SPELLINGS = {"fp32": ("fp32", "float32"), "bf16": ("bf16", "bf16_moments", "bfloat16"),
                     "fp8": ("fp8", "fp8_moments")}
_MASTER_SPELLINGS = {"fp32": ("fp32", "float32"), "fp24": ("fp24", "float24")}
_FP8_CODE_DTYPE = {"m": torch.float8_e4m3fn, "v": torch.float8_e5m2}
_VALUE_DTYPE = {"fp32": torch.float32, "bf16": torch.bfloat16}


def _lookup(name: Any, spellings: dict[str, tuple[str, ...]], what: str) -> str:
    key = name.lower() if isinstance(name, str) else None
    for fmt, names in spellings.items():
        if key in names:
            return fmt
    accepted = sorted(n for names in spellings.values() for n in names)
    raise ValueError(f"unknown {what} precision {name!r}; expected one of {accepted}")


def moment_format(name: str) -> str:
    """The moment format a precision name means ('fp32', 'bf16' / 'bf16_moments', 'fp8' / 'fp8_moments', ...)."""
    return _lookup(name, _MOMENT_SPELLINGS, "moment")


def master_format(name: str) -> str:
    """The master format a precision name means ('fp32' / 'float32' or 'fp24' / 'float24')."""
    return _lookup(name, _MASTER_SPELLINGS, "master")


def bytes_per_param(precision: str, moments: int = 2, master: str = "fp32") -> float:
    """Device bytes per parameter of the master plus ``moments`` moment buffers (AdamW 2, Lion 1)."""
    return _FORMATS[master_format(master)].value_bytes + moments * _FORMATS[moment_format(precision)].value_bytes


def _blocks(numel: int, block: int = BLOCK) -> int:
    return max(1, -(-numel // block))


class StateBuffer:
    """``numel`` optimizer-state values of one role ('m', 'v' or 'p') in one format, as device planes."""

    __slots__ = ("fmt", "role", "numel", "block", "planes")

    def __init__(self, fmt: str, role: str, numel: int, planes: dict[str, torch.Tensor], block: int = BLOCK):
        if fmt not in _FORMATS or role not in ROLES:
            raise ValueError(f"no state buffer of format {fmt!r} and role {role!r}")
        self.fmt, self.role, self.numel, self.block = fmt, role, int(numel), int(block)
        self.planes = planes

    # ------------------------------------------------------------------ construction

    @classmethod
    def allocate(cls, fmt: str, role: str, numel: int, device) -> "StateBuffer":
        """Zero values (FP8: zero codes, unit scales) on ``device``."""
        dev = torch.device(device)
        if fmt == "fp8":
            nb = _blocks(numel)
            planes = {"q": torch.zeros(nb * BLOCK, dtype=_FP8_CODE_DTYPE["v" if role == "v" else "m"], device=dev),
                      "scale": torch.ones(nb, dtype=torch.float32, device=dev)}
        elif fmt == "fp24":
            planes = {"hi": torch.zeros(numel, dtype=torch.bfloat16, device=dev),
                      "lo": torch.zeros(numel, dtype=torch.uint8, device=dev)}
        else:
            planes = {"data": torch.zeros(numel, dtype=_VALUE_DTYPE[fmt], device=dev)}
        return cls(fmt, role, numel, planes)

    @classmethod
    def viewing(cls, values: torch.Tensor, role: str = "p") -> "StateBuffer":
        """A buffer over an existing tensor of fp32 or bf16 values (flattened, not copied): an FP32 parameter
        that is its own master, or values to convert from."""
        if values.dtype not in (torch.float32, torch.bfloat16):
            values = values.float()
        flat = values.detach().reshape(-1)
        return cls("fp32" if flat.dtype == torch.float32 else "bf16", role, flat.numel(), {"data": flat})

    @classmethod
    def converted(cls, src: "StateBuffer | torch.Tensor", fmt: str, role: str, device) -> "StateBuffer":
        """A new buffer on ``device`` holding ``src``'s values in ``fmt``."""
        n = src.numel if isinstance(src, StateBuffer) else src.numel()
        out = cls.allocate(fmt, role, n, device)
        out.assign(src)
        return out

    # ------------------------------------------------------------------ inspection

    @property
    def device(self) -> torch.device:
        return next(iter(self.planes.values())).device

    @property
    def precision(self) -> str:
        return self.fmt

    @property
    def nbytes(self) -> int:
        return sum(t.nbytes for t in self.planes.values())

    @property
    def operands(self) -> tuple[torch.Tensor, torch.Tensor | None]:
        """(values / codes / hi plane, scales / lo plane or None): what a kernel segment points at."""
        names = _FORMATS[self.fmt].planes
        return self.planes[names[0]], (self.planes[names[1]] if len(names) > 1 else None)

    @property
    def kernel_code(self) -> int:
        return _FORMATS[self.fmt].code

    def plane_runs(self) -> list[tuple[torch.Tensor, int, bool]]:
        """(plane, values per entry, padded to whole blocks) of each plane: how a ZeRO shard's planes map onto the
        per-parameter planes of a checkpoint."""
        if self.fmt == "fp8":
            return [(self.planes["q"], 1, True), (self.planes["scale"], BLOCK, True)]
        return [(self.planes[name], 1, False) for name in _FORMATS[self.fmt].planes]

    def _abi(self) -> native.State:
        first, second = self.operands
        return native.State(first.data_ptr(), second.data_ptr() if second is not None else None, self.kernel_code,
                            1 if (self.fmt == "fp8" and self.role == "v") else 0, self.block)

    def _same_layout(self, other: "StateBuffer") -> bool:
        if self.fmt != other.fmt:
            return False
        return self.fmt != "fp8" or (self.role == other.role and self.block == other.block)

    # ------------------------------------------------------------------ conversion

    def assign(self, src: "StateBuffer | torch.Tensor", stream=None) -> None:
        """Make this buffer hold ``src``'s values (another buffer, or a tensor of values) in this buffer's format.

        Planes on another device are copied here first; a different format (or FP8 role or block) is converted by
        libabx's conversion kernel on ``stream`` (default: the device's current stream)."""
        if isinstance(src, torch.Tensor):
            src = StateBuffer.viewing(src, self.role)
        if src.numel != self.numel:
            raise ValueError(f"state of {src.numel} elements assigned to a buffer of {self.numel} elements")
        dev = self.device
        if not dev.type == "cuda":
            raise ValueError("state buffers are converted on their GPU; this one is on the host")
        if src.device != dev:
            src = src.to_device(dev)
        if self._same_layout(src):
            for name in _FORMATS[self.fmt].planes:
                _raw(self.planes[name]).copy_(_raw(src.planes[name]))
            return
        with torch.cuda.device(dev):
            native.load().convert(stream, src._abi(), self._abi(), self.numel)

    def to_device(self, device) -> "StateBuffer":
        """The same planes, copied as bytes to ``device``."""
        planes = {k: v.to(device, copy=False).contiguous() for k, v in self.planes.items()}
        return StateBuffer(self.fmt, self.role, self.numel, planes, self.block)

    def to_fp32(self) -> torch.Tensor:
        """The values as a new flat fp32 tensor on the buffer's GPU (an fp32 buffer: a copy)."""
        if self.fmt == "fp32":
            return self.planes["data"].clone()
        return StateBuffer.converted(self, "fp32", self.role, self.device).planes["data"]

    # ------------------------------------------------------------------ checkpoints

    def checkpoint(self) -> dict[str, Any]:
        """The reference's dict for this buffer: ``{"precision", <planes>}``, FP8 with its role and block."""
        d: dict[str, Any] = {"precision": self.fmt}
        if self.fmt == "fp8":
            d.update(role=self.role, block=self.block)
        d.update(self.planes)
        return d

    @classmethod
    def from_checkpoint(cls, saved: Any, numel: int, role: str, what: str) -> "StateBuffer":
        """A checkpoint moment (a store dict, or a plain tensor of values as torch.optim.AdamW saves it) as a
        buffer over the checkpoint's own tensors, after checking every field; nothing is copied."""
        check_moment(saved, numel, what)
        if isinstance(saved, torch.Tensor):
            return cls.viewing(saved, role)
        fmt = saved["precision"]
        if fmt == "fp8":
            saved_role = saved.get("role", role)
            planes = {"q": saved["q"].reshape(-1), "scale": saved["scale"].reshape(-1).float()}
            return cls("fp8", saved_role, numel, planes, block=saved["block"])
        data = saved["data"].reshape(-1)
        if data.dtype != _VALUE_DTYPE[fmt]:
            data = data.to(_VALUE_DTYPE[fmt])
        return cls(fmt, role, numel, {"data": data})

    @classmethod
    def master_from_checkpoint(cls, saved: Any, numel: int, what: str) -> "StateBuffer":
        """A checkpoint's master weights (a tensor, or an fp32 / fp24 store dict) as a buffer over its tensors."""
        check_master(saved, numel, what)
        if isinstance(saved, torch.Tensor):
            return cls.viewing(saved, "p")
        if saved["precision"] == "fp24":
            return cls("fp24", "p", numel, {"hi": saved["hi"].reshape(-1), "lo": saved["lo"].reshape(-1)})
        return cls.viewing(saved["data"], "p")


def _raw(t: torch.Tensor) -> torch.Tensor:
    """The same bytes as an integer tensor, so copies move bits and never convert values."""
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])


# ---------------------------------------------------------------------- checkpoint validation

def _tensor_of(t: Any, numel: int, what: str) -> torch.Tensor:
    """``t`` when it is a tensor of exactly ``numel`` elements; a smaller one would silently broadcast."""
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"checkpoint {what}: expected a tensor, found {type(t).__name__}")
    if t.numel() != numel:
        raise ValueError(f"checkpoint {what}: {t.numel()} elements where this optimizer has {numel} "
                         "(a checkpoint of another model?)")
    return t


def check_moment(saved: Any, numel: int, what: str) -> None:
    """Raise ValueError unless ``saved`` is a loadable moment of ``numel`` values: a tensor of values, or an
    fp32 / bf16 / fp8 store dict whose planes have the sizes its format implies."""
    if isinstance(saved, torch.Tensor):
        _tensor_of(saved, numel, what)
        return
    fmt = saved.get("precision") if isinstance(saved, dict) else None
    if fmt not in MOMENT_FORMATS:
        raise ValueError(f"checkpoint {what}: unknown moment precision {fmt if isinstance(saved, dict) else saved!r}")
    if fmt != "fp8":
        _tensor_of(saved.get("data"), numel, what)
        return
    if saved.get("role", "m") not in ("m", "v"):
        raise ValueError(f"checkpoint {what}: unknown FP8 role {saved.get('role')!r}")
    block = saved.get("block")
    if isinstance(block, bool) or not isinstance(block, int) or not 0 < block <= MAX_CHECKPOINT_BLOCK:
        raise ValueError(f"checkpoint {what}: invalid FP8 block size {block!r}")
    nb = _blocks(numel, block)
    _tensor_of(saved.get("q"), nb * block, f"{what} (FP8 codes)")
    _tensor_of(saved.get("scale"), nb, f"{what} (FP8 scales)")


def check_master(saved: Any, numel: int, what: str) -> None:
    """Raise ValueError unless ``saved`` is loadable master weights: a tensor of ``numel`` values, or an fp32 /
    fp24 store dict (fp24: a bfloat16 hi plane and a uint8 lo plane)."""
    if isinstance(saved, torch.Tensor):
        _tensor_of(saved, numel, what)
        return
    fmt = saved.get("precision") if isinstance(saved, dict) else None
    if fmt not in MASTER_FORMATS:
        found = fmt if isinstance(saved, dict) else type(saved).__name__
        raise ValueError(f"checkpoint {what}: expected a tensor or an fp32 / fp24 master, found precision {found!r}")
    if fmt == "fp32":
        _tensor_of(saved.get("data"), numel, what)
        return
    if _tensor_of(saved.get("hi"), numel, f"{what} (hi plane)").dtype != torch.bfloat16:
        raise ValueError(f"checkpoint {what}: the fp24 hi plane must be bfloat16")
    if _tensor_of(saved.get("lo"), numel, f"{what} (lo plane)").dtype != torch.uint8:
        raise ValueError(f"checkpoint {what}: the fp24 lo plane must be uint8")
