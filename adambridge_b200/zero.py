"""ZeRO-1: the optimizer state sharded over the ranks of a process group.

The reference has no multi-process code (README.md:633-634); this is the B200 build's
data-parallel form of the same update.  Parameters (optimizer order) are packed into one
flat index space, each tensor starting on a 128-element boundary (the FP8 block, and a
multiple of every SIMD width, so a piece of a tensor rounds exactly like the whole
tensor: adambridge/csrc/adambridge_kernels.c:1566-1577, tests/native/selftest.c:304-336).
The space is cut into ``rounds x world`` equal chunks; rank ``r`` owns chunk ``r`` of
every round::

    flat:   | round 0: rank0 rank1 ... rankW-1 | round 1: rank0 rank1 ... | ...
    rank r state (master, moments, FP8 scales, gradient shard): its chunks, round-major

One step, per round: the rank's update kernel (libabx, writing the new bf16 weights
straight into its chunk of the flat weight buffer that the parameters view) on the update
stream, then an in-place NCCL ``all_gather_into_tensor`` of that round on the comm stream.
The all-gather of round k overlaps the update of round k+1.  ``step()`` first
reduce-scatters (mean) the gradients round by round; ``step_shard(grad_shard)`` takes a
gradient shard the caller already holds.

Results are bit-identical to the unsharded update whatever the world size: each piece is
a segment with the tensor-local ``offset`` and the parameter's optimizer ``index``.
"""

from __future__ import annotations

import bisect
import ctypes
import math
from dataclasses import dataclass
from typing import Any, Iterable

import torch
import torch.distributed as dist

from . import native
from .precision import canonical_master_precision, canonical_precision, make_master, make_store

__all__ = ["FlatLayout", "Piece", "ZeroAdamBridge", "ZeroLionBridge"]

ALIGN = 128
_MASK64 = (1 << 64) - 1


@dataclass(frozen=True)
class Piece:
    """Elements [t_lo, t_hi) of parameter ``index`` at flat position ``flat_lo`` and rank-local ``local_lo``."""

    index: int
    t_lo: int
    t_hi: int
    flat_lo: int
    local_lo: int

    @property
    def n(self) -> int:
        return self.t_hi - self.t_lo


class FlatLayout:
    """Where every parameter element lives in the flat space and in each rank's shard."""

    def __init__(self, numels: Iterable[int], world: int, rounds: int | None = None,
                 target_chunk: int = 1 << 26):
        self.numels = [int(n) for n in numels]
        if world < 1:
            raise ValueError("world must be >= 1")
        self.world = world
        self.offsets = []
        off = 0
        for n in self.numels:
            self.offsets.append(off)
            off += -(-n // ALIGN) * ALIGN
        self.used = off
        per_rank = -(-max(self.used, 1) // world)
        if rounds is None:   # one round without peers (nothing to overlap); else ~target_chunk per round
            rounds = 1 if world == 1 else max(1, min(64, -(-per_rank // target_chunk)))
        self.rounds = int(rounds)
        self.chunk = max(ALIGN, -(-per_rank // (self.rounds * ALIGN)) * ALIGN)
        self.total = self.rounds * self.world * self.chunk
        self.shard_numel = self.rounds * self.chunk

    def round_range(self, r: int) -> tuple[int, int]:
        lo = r * self.world * self.chunk
        return lo, lo + self.world * self.chunk

    def rank_range(self, r: int, rank: int) -> tuple[int, int]:
        lo = r * self.world * self.chunk + rank * self.chunk
        return lo, lo + self.chunk

    def pieces(self, rank: int) -> list[list[Piece]]:
        """For each round, the pieces of parameters in ``rank``'s chunk, in flat order."""
        out = []
        for r in range(self.rounds):
            lo, hi = self.rank_range(r, rank)
            items = []
            i = max(0, bisect.bisect_right(self.offsets, lo) - 1)
            while i < len(self.numels) and self.offsets[i] < hi:
                t0, t1 = self.offsets[i], self.offsets[i] + self.numels[i]
                a, b = max(lo, t0), min(hi, t1)
                if a < b:
                    items.append(Piece(i, a - t0, b - t0, a, r * self.chunk + (a - lo)))
                i += 1
            out.append(items)
        return out

    def flat_slice(self, index: int) -> tuple[int, int]:
        return self.offsets[index], self.offsets[index] + self.numels[index]


class ZeroAdamBridge(torch.optim.Optimizer):
    r"""AdamW with ZeRO-1-sharded GPU state; the arithmetic of :class:`adambridge_b200.AdamBridge`.

    All parameters must be contiguous CUDA tensors of one device and one dtype (bf16 or fp32).  At
    construction their storage moves into one flat buffer (``self.flat_weights``) that the parameters keep
    viewing; every rank holds all weights and 1/world of the optimizer state.

    ``step()``: the gradients in ``p.grad`` (every rank's full local gradients, as after backward) are averaged
    and scattered to their owners (NCCL reduce-scatter), each rank updates its shard, and the new weights are
    all-gathered.  ``gather='p2p'`` (the default where the GPUs can map each other's memory) fuses the
    all-gather into the update: the weight buffer lives in symmetric memory and the kernel stores each new
    weight into every peer's copy over NVLink; ``'nccl'`` runs NCCL's all-gather round by round instead.

    ``step_shard(grad_shard)``: the caller supplies this rank's already reduced gradient shard
    (``shard_numel`` elements, round-major; see :class:`FlatLayout`).  Every parameter is updated every step.
    """

    _algorithm = "adamw"

    def __init__(self, params, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, *, precision: str = "fp32", master_precision: str = "fp32",
                 stochastic_rounding: bool = True, seed: int = 0, process_group=None, rounds: int | None = None,
                 max_ctas: int = 0, grad_dtype: torch.dtype | None = None, gather: str = "auto"):
        if not 0.0 <= lr or not 0.0 <= eps or not 0.0 <= weight_decay:
            raise ValueError("lr, eps and weight_decay must be >= 0")
        if not 0.0 <= betas[0] < 1.0 or not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"invalid betas: {betas}")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.precision = canonical_precision(precision)
        self.master_precision = canonical_master_precision(master_precision)
        self.stochastic = stochastic_rounding
        self.seed = seed
        self.max_ctas = max_ctas
        self.kernels = native.load()
        self.pg = process_group if process_group is not None else (dist.group.WORLD if dist.is_initialized() else None)
        self.world = dist.get_world_size(self.pg) if self.pg is not None else 1
        self.rank = dist.get_rank(self.pg) if self.pg is not None else 0

        self._params = [p for g in self.param_groups for p in g["params"]]
        self._group_of = [gi for gi, g in enumerate(self.param_groups) for _ in g["params"]]
        if not self._params:
            raise ValueError("no parameters")
        dev, dtype = self._params[0].device, self._params[0].dtype
        for p in self._params:
            if not p.is_cuda or p.device != dev or p.dtype != dtype or not p.is_contiguous():
                raise ValueError("ZeroAdamBridge needs contiguous CUDA parameters of one device and one dtype")
        if dtype not in (torch.bfloat16, torch.float32):
            raise TypeError(f"parameters must be bfloat16 or float32, got {dtype}")
        self.device, self.dtype = dev, dtype
        self.grad_dtype = grad_dtype or dtype
        if gather not in ("auto", "p2p", "nccl"):
            raise ValueError("gather must be 'auto', 'p2p' or 'nccl'")
        self._peer_deltas: list[int] | None = None
        numels = [p.numel() for p in self._params]
        flat = None
        if self.world > 1 and gather != "nccl":
            # fused all-gather: nothing to overlap round by round, so one round unless asked otherwise
            self.layout = FlatLayout(numels, self.world, rounds or 1)
            flat = self._symmetric_buffer(self.layout.total, dtype, dev, required=gather == "p2p")
        if flat is None:
            self.layout = FlatLayout(numels, self.world, rounds)
        L = self.layout
        with torch.no_grad(), torch.cuda.device(dev):
            if flat is None:
                self.flat_weights = torch.zeros(L.total, dtype=dtype, device=dev)
            else:
                self.flat_weights = flat
                self.flat_weights.zero_()
                self._map_peers(flat)
            for i, p in enumerate(self._params):
                a, b = L.flat_slice(i)
                self.flat_weights[a:b].copy_(p.detach().view(-1))
                p.data = self.flat_weights[a:b].view(p.shape)
            self._pieces = L.pieces(self.rank)
            master_init = torch.cat([self.flat_weights[slice(*L.rank_range(r, self.rank))] for r in range(L.rounds)])
            self.master = make_master(self.master_precision, L.shard_numel, init=master_init, device=dev)
            del master_init
            self.m = make_store(self.precision, L.shard_numel, "m", device=dev)
            self.v = None if self._algorithm == "lion" else make_store(self.precision, L.shard_numel, "v", device=dev)
            self.grad_shard = torch.zeros(L.shard_numel, dtype=self.grad_dtype, device=dev)
        self._flat_grads: torch.Tensor | None = None
        self.step_count = 0
        self._update_stream = torch.cuda.Stream(dev)
        self._comm_stream = torch.cuda.Stream(dev) if self.world > 1 else None
        self._groups = [native.Group() for _ in self.param_groups]
        self._segs = self._build_segments()
        self.trace: list | None = None   # (start, end) CUDA events of every update launch, when a list

    # ------------------------------------------------------------------ fused all-gather

    @staticmethod
    def _symmetric_buffer(numel: int, dtype, dev, required: bool):
        """A buffer in symmetric memory (mapped into every peer), or None where the GPUs cannot map each
        other's memory (then NCCL does the all-gather)."""
        try:
            import torch.distributed._symmetric_memory as symm
            return symm.empty(numel, dtype=dtype, device=dev)
        except Exception as exc:  # noqa: BLE001
            if required:
                raise RuntimeError(f"gather='p2p' needs symmetric memory: {exc}") from exc
            return None

    def _map_peers(self, flat: torch.Tensor) -> None:
        import torch.distributed._symmetric_memory as symm
        self._symm = symm.rendezvous(flat, group=self.pg)
        ptrs = [int(x) for x in self._symm.buffer_ptrs]
        base = ptrs[self.rank]
        self._peer_deltas = [ptrs[r] - base for r in range(self.world) if r != self.rank]
        self._barrier_flag = torch.zeros(1, dtype=torch.float32, device=flat.device)

    def _barrier(self, stream) -> None:
        """All ranks reach this point of their update streams (a one-element NCCL all-reduce: bounded by
        the process group's timeout, no device-side spin)."""
        with torch.cuda.stream(stream):
            dist.all_reduce(self._barrier_flag, group=self.pg)

    # ------------------------------------------------------------------ segments

    def _build_segments(self) -> list[ctypes.Array]:
        """One segment array per round, pointing into this rank's state and the flat weights."""
        p_hi, p_lo = self.master.native_buffers
        m_buf, m_scale = self.m.native_buffers
        v_buf, v_scale = (None, None) if self.v is None else self.v.native_buffers
        p_es = p_hi.element_size()
        m_es = m_buf.element_size()
        out_es = self.flat_weights.element_size()
        g_es = self.grad_shard.element_size()
        rounds = []
        self._seg_objs = []
        for pieces in self._pieces:
            ptrs = []
            for pc in pieces:
                s = native.Segment()
                s.p = p_hi.data_ptr() + pc.local_lo * p_es
                s.p_lo = p_lo.data_ptr() + pc.local_lo if p_lo is not None else None
                s.p_dtype = native.MASTER_CODES[self.master.precision]
                s.g = self.grad_shard.data_ptr() + pc.local_lo * g_es
                s.g_dtype = native.dtype_code_of(self.grad_dtype)
                s.m = m_buf.data_ptr() + pc.local_lo * m_es
                s.m_scale = m_scale.data_ptr() + 4 * (pc.local_lo // ALIGN) if m_scale is not None else None
                if v_buf is not None:
                    s.v = v_buf.data_ptr() + pc.local_lo * m_es
                    s.v_scale = v_scale.data_ptr() + 4 * (pc.local_lo // ALIGN) if v_scale is not None else None
                s.out = self.flat_weights.data_ptr() + pc.flat_lo * out_es
                s.out_dtype = native.dtype_code_of(self.dtype)
                s.n = pc.n
                s.offset = pc.t_lo
                s.index = pc.index
                s.mv_dtype = native.MOMENT_CODES[self.m.precision]
                s.algorithm = native.ALGORITHMS[self._algorithm]
                s.group = ctypes.pointer(self._groups[self._group_of[pc.index]])
                self._seg_objs.append(s)
                ptrs.append(ctypes.pointer(s))
            rounds.append(self.kernels.segment_array(ptrs))
        return rounds

    def _refresh(self) -> None:
        """Step number and group hyperparameters (re-read every step, so LR schedulers work)."""
        self.step_count += 1
        for g, grp in zip(self._groups, self.param_groups):
            b1, b2 = grp["betas"]
            g.lr, g.beta1, g.beta2 = float(grp["lr"]), float(b1), float(b2)
            g.eps = float(grp.get("eps", 0.0))
            g.weight_decay = float(grp["weight_decay"])
            g.seed = self.seed & _MASK64
            g.stochastic = int(self.stochastic)
        for s in self._seg_objs:
            s.step = self.step_count

    # ------------------------------------------------------------------ steps

    def _flat_grad_buffer(self) -> torch.Tensor:
        if self._flat_grads is None:
            self._flat_grads = torch.zeros(self.layout.total, dtype=self.grad_dtype, device=self.device)
        return self._flat_grads

    @torch.no_grad()
    def step(self, closure=None):
        """Reduce-scatter (mean) the local gradients, update this rank's shard, all-gather the weights."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        L = self.layout
        flat = self._flat_grad_buffer()
        for i, p in enumerate(self._params):
            if p.grad is None:
                raise RuntimeError(f"parameter {i} has no gradient: ZeRO steps update every parameter")
            a, b = L.flat_slice(i)
            if p.grad.data_ptr() != flat[a:b].data_ptr():
                flat[a:b].copy_(p.grad.reshape(-1))
        self._run(flat)
        return loss

    @torch.no_grad()
    def step_shard(self, grad_shard: torch.Tensor | None = None) -> None:
        """Update from this rank's reduced gradient shard (default: ``self.grad_shard``) and all-gather."""
        if grad_shard is not None and grad_shard.data_ptr() != self.grad_shard.data_ptr():
            self.grad_shard.copy_(grad_shard)
        self._run(None)

    def _run(self, flat_grads: torch.Tensor | None) -> None:
        L = self.layout
        self._refresh()
        cur = torch.cuda.current_stream(self.device)
        upd, comm = self._update_stream, self._comm_stream
        p2p = self._peer_deltas is not None
        upd.wait_stream(cur)
        if comm is not None:
            comm.wait_stream(cur)
        with torch.cuda.device(self.device):
            if p2p and flat_grads is None:
                self._barrier(upd)   # no peer still reads the weights this update overwrites
            for r in range(L.rounds):
                if flat_grads is not None:
                    shard = self.grad_shard[r * L.chunk:(r + 1) * L.chunk]
                    src = flat_grads[slice(*L.round_range(r))]
                    if comm is None:
                        shard.copy_(src)
                    else:
                        with torch.cuda.stream(comm):
                            dist.reduce_scatter_tensor(shard, src, op=dist.ReduceOp.AVG, group=self.pg)
                        upd.wait_stream(comm)
                start = end = None
                if self.trace is not None:
                    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    start.record(upd)
                if len(self._segs[r]):
                    if p2p:
                        self.kernels.multi_step_replicated(upd, self._segs[r], self._peer_deltas, self.max_ctas)
                    else:
                        self.kernels.multi_step(upd, self._segs[r], self.max_ctas)
                if end is not None:
                    end.record(upd)
                    self.trace.append((start, end))
                if comm is not None and not p2p:
                    comm.wait_stream(upd)
                    with torch.cuda.stream(comm):
                        out = self.flat_weights[slice(*L.round_range(r))]
                        mine = self.flat_weights[slice(*L.rank_range(r, self.rank))]
                        dist.all_gather_into_tensor(out, mine, group=self.pg)
        if p2p:
            self._barrier(upd)       # every peer's stores into this rank's weights have landed
        cur.wait_stream(upd)
        if comm is not None:
            cur.wait_stream(comm)

    # ------------------------------------------------------------------ inspection

    def launches_per_step(self) -> int:
        """Kernel launches of one step (64 segments of one kind per launch)."""
        return sum(math.ceil(len(s) / 64) for s in self._segs)

    def memory_report(self) -> dict[str, int]:
        rep = {"master": self.master.nbytes, "moments": self.m.nbytes + (self.v.nbytes if self.v is not None else 0),
               "grad_shard": self.grad_shard.nbytes, "weights": self.flat_weights.nbytes}
        rep["total"] = sum(rep.values())
        return rep

    def state_dict(self) -> dict[str, Any]:
        raise NotImplementedError("ZeroAdamBridge checkpoints: gather with AdamBridge-format shards is not built yet")


class ZeroLionBridge(ZeroAdamBridge):
    """Lion with ZeRO-1-sharded GPU state (see :class:`ZeroAdamBridge`)."""

    _algorithm = "lion"

    def __init__(self, params, lr: float = 1e-4, betas: tuple[float, float] = (0.9, 0.99), weight_decay: float = 0.0,
                 **kwargs):
        if "eps" in kwargs:
            raise TypeError("ZeroLionBridge has no eps")
        super().__init__(params, lr=lr, betas=betas, eps=0.0, weight_decay=weight_decay, **kwargs)
