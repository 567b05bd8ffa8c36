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
stream, then the all-gather of that round: an in-place NCCL ``all_gather_into_tensor`` on
the comm stream, or -- with the weight buffer in symmetric memory -- copy-engine copies into
the peers' buffers (``gather='ce'``) or the update kernel's own stores into them
(``gather='p2p'``).  The all-gather of round k overlaps the update of round k+1.  ``step()`` first
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
from .precision import StateBuffer, check_master, check_moment, master_format, moment_format

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

    def rounds_of(self, index: int) -> list[int]:
        """The rounds whose flat range holds elements of parameter ``index`` (an empty parameter: the round of
        its offset), in order -- the reduce-scatters its gradient takes part in."""
        a, b = self.flat_slice(index)
        span = self.world * self.chunk
        return list(range(a // span, (max(b, a + 1) - 1) // span + 1))

    def shard_runs(self, rank: int, unit: int = 1, padded: bool = False) -> list[tuple[int, int, int, int]]:
        """``(index, param_lo, shard_lo, length)`` for every piece of ``rank``'s shard, in entries of an array
        holding one entry per ``unit`` elements (1: weights, master, moments; 128: FP8 block scales).
        ``padded`` extends each tensor's last piece to its last whole 128-element block (FP8 codes and scales,
        which a per-tensor store keeps padded).  Pieces start on 128-element boundaries of their tensor, so
        the runs are exact in either unit."""
        if unit not in (1, ALIGN):
            raise ValueError(f"unit must be 1 or {ALIGN}")
        runs = []
        for rnd in self.pieces(rank):
            for pc in rnd:
                hi = pc.t_hi
                if (padded or unit > 1) and hi == self.numels[pc.index]:
                    hi = -(-hi // ALIGN) * ALIGN
                runs.append((pc.index, pc.t_lo // unit, pc.local_lo // unit, (hi - pc.t_lo) // unit))
        return runs


class ZeroAdamBridge(torch.optim.Optimizer):
    r"""AdamW with ZeRO-1-sharded GPU state; the arithmetic of :class:`adambridge_b200.AdamBridge`.

    All parameters must be contiguous CUDA tensors of one device and one dtype (bf16 or fp32).  At
    construction their storage moves into one flat buffer (``self.flat_weights``) that the parameters keep
    viewing; every rank holds all weights and 1/world of the optimizer state.

    ``step()``: the gradients in ``p.grad`` (every rank's full local gradients, as after backward) are averaged
    and scattered to their owners (NCCL reduce-scatter), each rank updates its shard, and the new weights are
    all-gathered.  ``gather='p2p'`` (the default where the GPUs can map each other's memory) fuses the
    all-gather into the update: the weight buffer lives in symmetric memory and the kernel stores each new
    weight into every peer's copy over NVLink; ``'ce'`` keeps the symmetric buffer but has the copy engines
    carry each round's new weights to the peers (one asynchronous copy per peer, overlapping the next round's
    update); ``'nccl'`` runs NCCL's all-gather round by round instead.

    ``delay_updates`` (after ``delay_warmup_steps`` ordinary steps), as the reference's delayed mode: a step's
    update writes a second weight buffer and runs while the caller goes on (the next forward), and it becomes
    the weights at the next step -- the model trains with weights one step stale.  ``flush()`` applies it.  The
    parameters' storage then alternates between the two buffers (applying an update re-points them, copying
    nothing), so code should not keep views of a parameter's storage from one step to the next.

    ``step_shard(grad_shard)``: the caller supplies this rank's already reduced gradient shard
    (``shard_numel`` elements, round-major; see :class:`FlatLayout`).  Every parameter is updated every step.
    """

    _algorithm = "adamw"

    def __init__(self, params, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, *, precision: str = "fp32", master_precision: str = "fp32",
                 stochastic_rounding: bool = True, seed: int = 0, process_group=None, rounds: int | None = None,
                 max_ctas: int = 0, grad_dtype: torch.dtype | None = None, gather: str = "auto",
                 delay_updates: bool = False, delay_warmup_steps: int = 0):
        if not 0.0 <= lr or not 0.0 <= eps or not 0.0 <= weight_decay:
            raise ValueError("lr, eps and weight_decay must be >= 0")
        if not 0.0 <= betas[0] < 1.0 or not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"invalid betas: {betas}")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.precision = moment_format(precision)
        self.master_precision = master_format(master_precision)
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
        if gather not in ("auto", "p2p", "ce", "nccl"):
            raise ValueError("gather must be 'auto', 'p2p', 'ce' or 'nccl'")
        if delay_warmup_steps < 0:
            raise ValueError("delay_warmup_steps must be >= 0")
        self.delay_updates, self.delay_warmup_steps = bool(delay_updates), int(delay_warmup_steps)
        self._peer_deltas: list[int] | None = None
        numels = [p.numel() for p in self._params]
        flat = None
        if self.world > 1 and gather != "nccl":
            # fused all-gather: nothing to overlap round by round, so one round unless asked otherwise; the
            # copy-engine gather overlaps each round's copies with the next round's update
            self.layout = FlatLayout(numels, self.world, rounds if gather == "ce" else (rounds or 1))
            flat = self._symmetric_buffer(self.layout.total, dtype, dev, required=gather in ("p2p", "ce"))
        if flat is None:
            self.layout = FlatLayout(numels, self.world, rounds)
        # the all-gather this optimizer runs (None on one GPU)
        self.gather = None if self.world == 1 else ("nccl" if flat is None else ("ce" if gather == "ce" else "p2p"))
        self._replica_streams: list | None = None
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
            self.master = StateBuffer.converted(master_init, self.master_precision, "p", dev)
            del master_init
            self.m = StateBuffer.allocate(self.precision, "m", L.shard_numel, dev)
            self.v = None if self._algorithm == "lion" else StateBuffer.allocate(self.precision, "v", L.shard_numel, dev)
            self.grad_shard = torch.zeros(L.shard_numel, dtype=self.grad_dtype, device=dev)
        self._flat_grads: torch.Tensor | None = None
        self.step_count = 0
        self._update_stream = torch.cuda.Stream(dev)
        self._comm_stream = torch.cuda.Stream(dev) if self.world > 1 else None
        self._groups = [native.Group() for _ in self.param_groups]
        self._seg_objs: list = []
        self._segs = self._build_segments(self.flat_weights)
        # delayed updates: the new weights go to a second weight buffer (and, fused, into the peers' second
        # buffers), which becomes the weights at the next step; allocated at the first delayed step
        self._shadow: torch.Tensor | None = None
        self._shadow_segs: list | None = None
        self._shadow_deltas: list[int] | None = None
        self._delay_owed = False
        self._steps_done = 0
        # reduce-scatter reads of the flat gradients: the last of this step, and the last of the previous step
        # (which the next writes of the flat gradients wait for)
        self._grads_read_now: torch.cuda.Event | None = None
        self._grads_read: torch.cuda.Event | None = None
        self.trace: list | None = None   # (start, end) CUDA events of every update launch, when a list
        self.norm_trace: list = []       # (start, end) events of the norm kernels, while ``trace`` is a list
        self.release_grads = True
        self._copy_streams: tuple | None = None
        self._hooked = False
        self._hook_handles: list = []
        self._clip_coef: torch.Tensor | None = None
        self._norm_state = None
        self._update_in_backward = False
        self._backward_ctas = max_ctas
        self._rounds_updated: set[int] = set()   # hook mode: rounds this step already updated during backward

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
                raise RuntimeError(f"gather='p2p' and 'ce' need symmetric memory: {exc}") from exc
            return None

    def _rotated_deltas(self, ptrs: list[int]) -> list[int]:
        """Distances from this rank's buffer to the peers', starting at the next rank: every rank sends to a
        different peer first, so the NVLink traffic into each GPU is spread over its senders."""
        return [ptrs[(self.rank + j) % self.world] - ptrs[self.rank] for j in range(1, self.world)]

    def _map_peers(self, flat: torch.Tensor) -> None:
        import torch.distributed._symmetric_memory as symm
        self._symm = symm.rendezvous(flat, group=self.pg)
        self._peer_deltas = self._rotated_deltas([int(x) for x in self._symm.buffer_ptrs])
        self._barrier_flag = torch.zeros(1, dtype=torch.float32, device=flat.device)

    def _barrier(self, stream) -> None:
        """All ranks reach this point of their update streams (a one-element NCCL all-reduce: bounded by
        the process group's timeout, no device-side spin)."""
        with torch.cuda.stream(stream):
            dist.all_reduce(self._barrier_flag, group=self.pg)

    # ------------------------------------------------------------------ segments

    def _build_segments(self, weights: torch.Tensor) -> list[ctypes.Array]:
        """One segment array per round, pointing into this rank's state and the flat weight buffer ``weights``."""
        p_hi, p_lo = self.master.operands
        m_buf, m_scale = self.m.operands
        v_buf, v_scale = (None, None) if self.v is None else self.v.operands
        p_es = p_hi.element_size()
        m_es = m_buf.element_size()
        out_es = weights.element_size()
        g_es = self.grad_shard.element_size()
        rounds = []
        for pieces in self._pieces:
            ptrs = []
            for pc in pieces:
                s = native.Segment()
                s.p = p_hi.data_ptr() + pc.local_lo * p_es
                s.p_lo = p_lo.data_ptr() + pc.local_lo if p_lo is not None else None
                s.p_dtype = self.master.kernel_code
                s.g = self.grad_shard.data_ptr() + pc.local_lo * g_es
                s.g_dtype = native.dtype_code_of(self.grad_dtype)
                s.m = m_buf.data_ptr() + pc.local_lo * m_es
                s.m_scale = m_scale.data_ptr() + 4 * (pc.local_lo // ALIGN) if m_scale is not None else None
                if v_buf is not None:
                    s.v = v_buf.data_ptr() + pc.local_lo * m_es
                    s.v_scale = v_scale.data_ptr() + 4 * (pc.local_lo // ALIGN) if v_scale is not None else None
                s.out = weights.data_ptr() + pc.flat_lo * out_es
                s.out_dtype = native.dtype_code_of(self.dtype)
                s.n = pc.n
                s.offset = pc.t_lo
                s.index = pc.index
                s.mv_dtype = self.m.kernel_code
                s.algorithm = native.ALGORITHMS[self._algorithm]
                s.group = ctypes.pointer(self._groups[self._group_of[pc.index]])
                self._seg_objs.append(s)
                ptrs.append(ctypes.pointer(s))
            rounds.append(self.kernels.segment_array(ptrs))
        return rounds

    # ------------------------------------------------------------------ delayed updates

    def _delayed(self) -> bool:
        return self.delay_updates and self._steps_done >= self.delay_warmup_steps

    def _ensure_shadow(self) -> None:
        """The second weight buffer (symmetric like the first when the all-gather is fused); collective on first
        use, which every rank reaches at the same step."""
        if self._shadow is not None:
            return
        L = self.layout
        with torch.no_grad(), torch.cuda.device(self.device):
            if self._peer_deltas is not None:
                import torch.distributed._symmetric_memory as symm
                self._shadow = symm.empty(L.total, dtype=self.dtype, device=self.device)
                self._shadow.zero_()
                self._symm_shadow = symm.rendezvous(self._shadow, group=self.pg)
                self._shadow_deltas = self._rotated_deltas([int(x) for x in self._symm_shadow.buffer_ptrs])
            else:
                self._shadow = torch.zeros(L.total, dtype=self.dtype, device=self.device)
        self._shadow_segs = self._build_segments(self._shadow)

    def _apply_pending(self, cur) -> None:
        """The previous step's delayed update becomes the weights (on ``cur``, after that update and its gather).

        The two weight buffers trade places instead of copying 2 bytes per parameter twice: the parameters now
        view the buffer that update wrote, and the next delayed update writes the other one, after the work
        already enqueued on ``cur`` (which still reads it) and, with peers writing it, after the step's opening
        barrier.  Every rank trades at the same step, so the peers' buffers trade alike."""
        if not self._delay_owed:
            return
        cur.wait_stream(self._update_stream)
        if self._comm_stream is not None:
            cur.wait_stream(self._comm_stream)
        self.flat_weights, self._shadow = self._shadow, self.flat_weights
        self._segs, self._shadow_segs = self._shadow_segs, self._segs
        self._peer_deltas, self._shadow_deltas = self._shadow_deltas, self._peer_deltas
        L = self.layout
        with torch.no_grad():
            for i, p in enumerate(self._params):
                a, b = L.flat_slice(i)
                p.data = self.flat_weights[a:b].view(p.shape)
        self._delay_owed = False

    def _after_grad_reads(self, stream) -> None:
        """``stream`` waits until the previous step's last reduce-scatter has read the flat gradients (a delayed
        step returns before it ran, and the next backward writes the flat gradients again)."""
        if self._grads_read is not None:
            stream.wait_event(self._grads_read)
            self._grads_read = None

    @torch.no_grad()
    def flush(self) -> None:
        """Apply a pending delayed update to the parameters (before evaluating or saving).  Raises if an update
        kernel that has finished gave up a pipeline wait."""
        self.kernels.check_status("flush")
        self._apply_pending(torch.cuda.current_stream(self.device))

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

    def _local_grads(self) -> torch.Tensor:
        """Every parameter's local gradient in the flat gradient buffer (no copy where p.grad views it)."""
        L = self.layout
        flat = self._flat_grad_buffer()
        self._after_grad_reads(torch.cuda.current_stream(self.device))
        for i, p in enumerate(self._params):
            if p.grad is None:
                raise RuntimeError(f"parameter {i} has no gradient: ZeRO steps update every parameter")
            a, b = L.flat_slice(i)
            if p.grad.data_ptr() != flat[a:b].data_ptr():
                flat[a:b].copy_(p.grad.reshape(-1))
        return flat

    @torch.no_grad()
    def step(self, closure=None):
        """Reduce-scatter (mean) the local gradients, update this rank's shard, all-gather the weights.
        After :meth:`clip_grad_norm_` the gradients are already reduced and the update applies the clip;
        with :meth:`attach_hooks` the reduce-scatters ran during backward."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if self._hooked:
            self._finish_hooked_reduce()
        if self._rounds_updated:
            # hook mode, updated during backward: whatever round is left, then the end of the step
            cur = torch.cuda.current_stream(self.device)
            for r in range(self.layout.rounds):
                if r not in self._rounds_updated:
                    self._backward_update_round(r)
            self._finish_update(cur, delayed=False)
        elif self._clip_coef is not None:
            coef, self._clip_coef = self._clip_coef, None
            self._run(None, g_scale=coef, synced=True)
        elif self._hooked:
            self._run(None)
        else:
            self._run(self._local_grads())
        self._reset_hook_state()
        return loss

    # ------------------------------------------------------------------ gradients reduced during backward

    def attach_hooks(self, model: torch.nn.Module | None = None, update_in_backward: bool = True,
                     backward_max_ctas: int | None = None) -> "ZeroAdamBridge":
        """Reduce-scatter the gradients during backward (the data-parallel gradient path) and, with
        ``update_in_backward``, update the weights during backward too.

        A post-accumulate-grad hook copies each parameter's finished gradient into the flat gradient buffer
        (and, with ``release_grads``, frees ``p.grad``); when every parameter overlapping a round of the flat
        layout has arrived, that round's reduce-scatter (mean) starts on the comm stream, so it overlaps the
        rest of backward -- backward runs roughly in reverse parameter order, so the last rounds go first.  With
        ``update_in_backward`` (the reference's hook mode: each update as soon as its gradient is ready) the
        round's update kernel -- with its fused all-gather -- follows its reduce-scatter right away on the
        update stream, and ``step()`` only ends the step; otherwise ``step()`` updates every round.  Delayed
        updates and :meth:`clip_grad_norm_` (which needs every gradient before any update) update at ``step()``:
        pass ``update_in_backward=False`` to clip.  The overlap is per round: construct the optimizer with
        ``rounds`` > 1 for it.  What the step still waits for after backward is the last round to complete --
        round 0, holding the first parameters, whose gradients arrive last -- so small rounds pay: Llama-7B on
        8 B200 leaves 3.4 ms of the update after backward with 32 rounds, 6.7 ms with 8.  Every parameter must
        receive exactly one gradient per step.

        ``backward_max_ctas`` caps the CTAs of the updates run during backward (0: every SM).  By default it is
        one CTA per SM where the all-gather is fused and the update waits on NVLink (4 or more ranks): leaving SMs
        to the backward pass shortens the step (Llama-7B on 8 B200: 288.4 ms per step against 292.4 ms
        uncapped, 8 rounds).  With fewer ranks the update is HBM-bound and a cap only stretches it (2 B200: the
        capped update kernels took 37.2 ms of a 293.1 ms step, 14.5 ms uncapped), so the constructor's
        ``max_ctas`` applies."""
        self._update_in_backward = bool(update_in_backward)
        if backward_max_ctas is not None:
            if backward_max_ctas < 0:
                raise ValueError("backward_max_ctas must be >= 0")
            self._backward_ctas = int(backward_max_ctas)
        elif self.gather == "p2p" and self.world >= 4:
            self._backward_ctas = torch.cuda.get_device_properties(self.device).multi_processor_count
        else:
            self._backward_ctas = self.max_ctas
        if self._hooked:
            return self
        wanted = None if model is None else {id(p) for p in model.parameters()}
        L = self.layout
        self._rounds_of = [L.rounds_of(i) for i in range(len(self._params))]
        hook = torch.compiler.disable(self._on_grad_ready)
        self._index_of = {id(p): i for i, p in enumerate(self._params)}
        for p in self._params:
            if p.requires_grad and (wanted is None or id(p) in wanted):
                self._hook_handles.append(p.register_post_accumulate_grad_hook(hook))
        self._hooked = True
        self._reset_hook_state()
        return self

    def detach_hooks(self) -> None:
        for h in self._hook_handles:
            h.remove()
        self._hook_handles.clear()
        self._hooked = False

    def _reset_hook_state(self) -> None:
        if not self._hooked:
            return
        L = self.layout
        self._round_waiting = [0] * L.rounds
        for rounds in self._rounds_of:
            for r in rounds:
                self._round_waiting[r] += 1
        self._arrived = [False] * len(self._params)
        self._reduced = [False] * L.rounds
        self._rounds_updated = set()

    def _on_grad_ready(self, p: torch.Tensor) -> None:
        i = self._index_of[id(p)]
        if self._arrived[i]:
            raise RuntimeError("ZeroAdamBridge: parameter received a second gradient before step()")
        self._arrived[i] = True
        a, b = self.layout.flat_slice(i)
        self._after_grad_reads(torch.cuda.current_stream(self.device))
        with torch.no_grad():
            self._flat_grad_buffer()[a:b].copy_(p.grad.reshape(-1))
        if self.release_grads:
            p.grad = None
        for r in self._rounds_of[i]:
            self._round_waiting[r] -= 1
            if self._round_waiting[r] == 0:
                self._reduce_round(r)
                if self._updates_in_backward():
                    self._backward_update_round(r)

    def _reduce_round(self, r: int) -> None:
        """Reduce-scatter round ``r`` of the flat gradients into this rank's shard (comm stream, ordered after
        the work the current stream has enqueued so far)."""
        L = self.layout
        flat = self._flat_grad_buffer()
        shard = self.grad_shard[r * L.chunk:(r + 1) * L.chunk]
        src = flat[slice(*L.round_range(r))]
        cur = torch.cuda.current_stream(self.device)
        with torch.no_grad(), torch.cuda.device(self.device):
            if self._comm_stream is None:
                self._update_stream.wait_stream(cur)
                with torch.cuda.stream(self._update_stream):
                    shard.copy_(src)
                    self._record_grad_reads(self._update_stream)
            else:
                self._comm_stream.wait_stream(cur)
                self._comm_stream.wait_stream(self._update_stream)   # a delayed update may still read the shard
                with torch.cuda.stream(self._comm_stream):
                    dist.reduce_scatter_tensor(shard, src, op=dist.ReduceOp.AVG, group=self.pg)
                    self._record_grad_reads(self._comm_stream)
        self._reduced[r] = True

    def _record_grad_reads(self, stream) -> None:
        ev = torch.cuda.Event()
        ev.record(stream)
        self._grads_read_now = ev

    def _finish_hooked_reduce(self) -> None:
        """Before the update of a hooked step: every parameter's gradient arrived; the update stream waits for
        the reduce-scatters."""
        missing = [i for i, done in enumerate(self._arrived) if not done]
        if missing:
            raise RuntimeError(f"parameters {missing[:8]} have no gradient this step: ZeRO steps update every "
                               "parameter (with hooks attached, each needs exactly one gradient per step)")
        if self._comm_stream is not None:
            self._update_stream.wait_stream(self._comm_stream)

    @torch.no_grad()
    def step_shard(self, grad_shard: torch.Tensor | None = None, weights_out: torch.Tensor | None = None) -> None:
        """Update from this rank's reduced gradient shard (default: ``self.grad_shard``) and all-gather.

        ``grad_shard`` may be a pinned host tensor (``shard_numel`` gradients, round-major): it is copied in
        round by round on a copy stream, each round's copy overlapping the update of the round before.
        ``weights_out``, a pinned host tensor of ``shard_numel`` weights, receives this rank's updated weight
        shard round by round, each copy overlapping the next round's update.  Together they run the step as
        a host pipeline with both PCIe directions busy at once; the overlap is per round (``rounds`` > 1)."""
        L = self.layout
        host_in = grad_shard if grad_shard is not None and not grad_shard.is_cuda else None
        if host_in is not None and (host_in.numel() != L.shard_numel or host_in.dtype != self.grad_dtype):
            raise ValueError(f"a host gradient shard must hold {L.shard_numel} {self.grad_dtype} elements")
        if weights_out is not None and (weights_out.is_cuda or weights_out.numel() != L.shard_numel
                                        or weights_out.dtype != self.dtype):
            raise ValueError(f"weights_out must be a host tensor of {L.shard_numel} {self.dtype} elements")
        if grad_shard is not None and host_in is None and grad_shard.data_ptr() != self.grad_shard.data_ptr():
            self._apply_pending(torch.cuda.current_stream(self.device))   # a delayed update may still read it
            self.grad_shard.copy_(grad_shard)
        if self._clip_coef is not None:
            if host_in is not None:
                raise ValueError("clip_shard_grad_norm_ needs the gradient shard on the device before the step")
            coef, self._clip_coef = self._clip_coef, None
            self._run(None, g_scale=coef, synced=True, host_out=weights_out)
        else:
            self._run(None, host_in=host_in, host_out=weights_out)

    # ------------------------------------------------------------------ clipping

    def _norm_inputs(self):
        """Built once: this rank's pieces as norm-kernel tensors over ``grad_shard``, the kernel workspace, the
        per-piece sums (plus a zero slot) and, per parameter, the indices of its pieces here (padded with the
        zero slot) -- so the per-parameter partial sums are a fixed-order gather and sum."""
        if self._norm_state is None:
            pieces = [pc for rnd in self._pieces for pc in rnd]
            es = self.grad_shard.element_size()
            code = native.dtype_code_of(self.grad_dtype)
            arr = (native.Tensor * max(1, len(pieces)))()
            for j, pc in enumerate(pieces):
                arr[j] = native.Tensor(self.grad_shard.data_ptr() + pc.local_lo * es, pc.n, code, 0)
            owned: list[list[int]] = [[] for _ in self._params]
            for j, pc in enumerate(pieces):
                owned[pc.index].append(j)
            width = max(1, max(len(o) for o in owned))
            idx = [o + [len(pieces)] * (width - len(o)) for o in owned]
            dev = self.device
            ws = torch.empty(self.kernels.clip_workspace_bytes(arr, len(pieces)), dtype=torch.uint8, device=dev)
            sq_ext = torch.zeros(len(pieces) + 1, dtype=torch.float32, device=dev)
            self._norm_state = (arr, len(pieces), ws, sq_ext, torch.tensor(idx, dtype=torch.long, device=dev))
        return self._norm_state

    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float, norm_type: float = 2.0) -> torch.Tensor:
        """``torch.nn.utils.clip_grad_norm_`` of the averaged gradient, fused into the next :meth:`step`.

        Reduce-scatters (mean) the local gradients now, sums the squares of this rank's pieces of every
        parameter (libabx norm kernels), all-reduces the per-parameter sums (one small NCCL all-reduce) and
        computes the per-parameter norms, the total norm and the coefficient as torch does in the gradients'
        dtype.  Returns the total norm as a device tensor; the next ``step()`` updates from the reduced shard
        with every gradient scaled by the coefficient inside the update kernel."""
        if float(norm_type) != 2.0:
            raise ValueError("clip_grad_norm_ computes the L2 norm (norm_type=2) only")
        cur = torch.cuda.current_stream(self.device)
        if self._rounds_updated:
            raise RuntimeError("clip_grad_norm_ after the hooks already updated rounds during backward: attach the "
                               "hooks with update_in_backward=False to clip")
        if self._hooked:   # reduced during backward
            self._finish_hooked_reduce()
            self._update_stream.wait_stream(cur)
            return self._clip_shard(max_norm, cur)
        flat = self._local_grads()
        L = self.layout
        upd, comm = self._update_stream, self._comm_stream
        upd.wait_stream(cur)
        with torch.cuda.device(self.device):
            if comm is None:
                with torch.cuda.stream(upd):
                    for r in range(L.rounds):
                        self.grad_shard[r * L.chunk:(r + 1) * L.chunk].copy_(flat[slice(*L.round_range(r))])
                    self._record_grad_reads(upd)
            else:
                comm.wait_stream(cur)
                comm.wait_stream(upd)   # a delayed update may still read the shard
                with torch.cuda.stream(comm):
                    for r in range(L.rounds):
                        dist.reduce_scatter_tensor(self.grad_shard[r * L.chunk:(r + 1) * L.chunk],
                                                   flat[slice(*L.round_range(r))], op=dist.ReduceOp.AVG,
                                                   group=self.pg)
                    self._record_grad_reads(comm)
                upd.wait_stream(comm)
        return self._clip_shard(max_norm, cur)

    @torch.no_grad()
    def clip_shard_grad_norm_(self, max_norm: float, grad_shard: torch.Tensor | None = None) -> torch.Tensor:
        """:meth:`clip_grad_norm_` for the :meth:`step_shard` path: the norm of the reduced gradient whose shards
        the ranks hold (``grad_shard``, default ``self.grad_shard``); the next ``step_shard()`` applies the clip."""
        cur = torch.cuda.current_stream(self.device)
        if grad_shard is not None and grad_shard.data_ptr() != self.grad_shard.data_ptr():
            self._apply_pending(cur)   # a delayed update may still read the shard
            self.grad_shard.copy_(grad_shard)
        self._update_stream.wait_stream(cur)
        return self._clip_shard(max_norm, cur)

    def _clip_shard(self, max_norm: float, cur) -> torch.Tensor:
        """Norms of ``grad_shard`` on the update stream; keeps the coefficient for the next update."""
        upd = self._update_stream
        with torch.cuda.device(self.device):
            arr, npieces, ws, sq_ext, idx = self._norm_inputs()
            start = end = None
            if self.trace is not None:
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record(upd)
            self.kernels.grad_sq_norms(upd, arr, npieces, sq_ext, ws)
            if end is not None:
                end.record(upd)
                self.norm_trace.append((start, end))
            with torch.cuda.stream(upd):
                sq = sq_ext[idx].sum(dim=1)
                if self._comm_stream is not None:
                    dist.all_reduce(sq, group=self.pg)   # also orders every rank's update after all backward passes
                total_coef = torch.empty(2, dtype=torch.float32, device=self.device)
            self.kernels.clip_coef_from_sq(upd, sq, self.grad_dtype, max_norm, None, total_coef)
        cur.wait_stream(upd)
        self._clip_coef = total_coef[1:2]
        return total_coef[0].to(self.grad_dtype)

    def _run(self, flat_grads: torch.Tensor | None, g_scale: torch.Tensor | None = None,
             synced: bool = False, host_in: torch.Tensor | None = None, host_out: torch.Tensor | None = None) -> None:
        # an update kernel of an earlier step that gave up a pipeline wait left its shard partly updated
        # (a status word in mapped host memory, read without synchronizing)
        self.kernels.check_status("ZeroAdamBridge.step")
        L = self.layout
        cur = torch.cuda.current_stream(self.device)
        had_pending = self._delay_owed
        self._apply_pending(cur)        # delayed: the previous step's update becomes the weights now
        delayed = self._delayed()
        if delayed:
            self._ensure_shadow()
        target = self._target(delayed)
        self._refresh()
        upd, comm = self._update_stream, self._comm_stream
        mapped = self._peer_deltas is not None   # the peers write this rank's weight buffer
        upd.wait_stream(cur)
        if comm is not None:
            comm.wait_stream(cur)
        h2d = d2h = None
        if host_in is not None or host_out is not None:
            if self._copy_streams is None:
                self._copy_streams = (torch.cuda.Stream(self.device), torch.cuda.Stream(self.device))
            h2d, d2h = self._copy_streams
            h2d.wait_stream(cur)
            d2h.wait_stream(cur)
        with torch.cuda.device(self.device):
            if mapped and (delayed or had_pending or (flat_grads is None and not synced)):
                self._barrier(upd)   # no peer still reads the weights this update overwrites
            for r in range(L.rounds):
                if host_in is not None:
                    with torch.cuda.stream(h2d):
                        self.grad_shard[r * L.chunk:(r + 1) * L.chunk].copy_(
                            host_in[r * L.chunk:(r + 1) * L.chunk], non_blocking=True)
                    upd.wait_stream(h2d)
                if flat_grads is not None:
                    shard = self.grad_shard[r * L.chunk:(r + 1) * L.chunk]
                    src = flat_grads[slice(*L.round_range(r))]
                    if comm is None:
                        with torch.cuda.stream(upd):   # in order with the update that reads it
                            shard.copy_(src)
                            self._record_grad_reads(upd)
                    else:
                        with torch.cuda.stream(comm):
                            dist.reduce_scatter_tensor(shard, src, op=dist.ReduceOp.AVG, group=self.pg)
                            self._record_grad_reads(comm)
                        upd.wait_stream(comm)
                self._launch_round(r, target, g_scale)
                if host_out is not None:
                    d2h.wait_stream(upd)
                    with torch.cuda.stream(d2h):
                        host_out[r * L.chunk:(r + 1) * L.chunk].copy_(
                            target[0][slice(*L.rank_range(r, self.rank))], non_blocking=True)
        self._finish_update(cur, delayed)
        if h2d is not None:
            cur.wait_stream(h2d)
            cur.wait_stream(d2h)

    def _target(self, delayed: bool):
        """(weight buffer, per-round segments, peer deltas) this step's update writes: the weights, or with
        delayed updates the second buffer."""
        if delayed:
            return self._shadow, self._shadow_segs, self._shadow_deltas
        return self.flat_weights, self._segs, self._peer_deltas

    def _launch_round(self, r: int, target, g_scale: torch.Tensor | None, max_ctas: int | None = None) -> None:
        """Round ``r``'s update kernel on the update stream (with the fused all-gather, its peer stores), then
        that round's all-gather: the copies of this rank's new weights into the peers' buffers on the replica
        streams (copy engines), or NCCL's all-gather on the comm stream."""
        weights, segs, deltas = target
        ctas = self.max_ctas if max_ctas is None else max_ctas
        upd, comm = self._update_stream, self._comm_stream
        start = end = None
        if self.trace is not None:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(upd)
        if len(segs[r]):
            if self.gather == "p2p":
                self.kernels.multi_step_replicated(upd, segs[r], deltas, ctas, g_scale)
            else:
                self.kernels.multi_step(upd, segs[r], ctas, g_scale)
        if end is not None:
            end.record(upd)
            self.trace.append((start, end))
        if self.gather == "ce":
            self._replicate_round(r, weights, deltas)
        elif self.gather == "nccl":
            L = self.layout
            comm.wait_stream(upd)
            with torch.cuda.stream(comm):
                dist.all_gather_into_tensor(weights[slice(*L.round_range(r))],
                                            weights[slice(*L.rank_range(r, self.rank))], group=self.pg)

    def _replicate_round(self, r: int, weights: torch.Tensor, deltas: list[int]) -> None:
        """The copy-engine all-gather of round ``r``: this rank's new weights of the round, once the update
        stream has written them, copied into each peer's buffer, one replica stream (and copy) per peer."""
        a, b = self.layout.rank_range(r, self.rank)
        if b <= a:
            return
        if self._replica_streams is None:
            self._replica_streams = [torch.cuda.Stream(self.device) for _ in range(self.world - 1)]
        written = torch.cuda.Event()
        written.record(self._update_stream)
        for s in self._replica_streams:
            s.wait_event(written)
        es = weights.element_size()
        self.kernels.replicate_async(self._replica_streams, weights.data_ptr() + a * es, (b - a) * es, deltas)

    def _finish_update(self, cur, delayed: bool) -> None:
        """After the last round: every peer's stores or copies have landed (fused all-gather), the step is
        counted, and -- unless the update is delayed -- the caller's stream is ordered after the update and
        gathers."""
        if self._peer_deltas is not None:
            for s in self._replica_streams or ():
                self._update_stream.wait_stream(s)   # this rank's copies to the peers are done
            self._barrier(self._update_stream)   # every peer's stores into this rank's weights have landed
        self._steps_done += 1
        self._grads_read, self._grads_read_now = self._grads_read_now, None
        if delayed:
            # the update overlaps whatever the caller runs next; the next step (or flush) makes it the weights
            self._delay_owed = True
        else:
            cur.wait_stream(self._update_stream)
            if self._comm_stream is not None:
                cur.wait_stream(self._comm_stream)

    # ------------------------------------------------------------------ updates during backward

    def _backward_update_round(self, r: int) -> None:
        """Hook mode: update round ``r`` (and all-gather it) as soon as its reduce-scatter is enqueued, while
        backward goes on.  No barrier is needed first: a rank's reduce-scatter of round ``r`` completes only after
        every rank has issued its own, which each issues after its backward has finished with round ``r``'s
        weights -- so no peer still reads the weights these stores overwrite.  The first round of a step also
        starts the step (step count, group hyperparameters)."""
        if not self._rounds_updated:
            self.kernels.check_status("ZeroAdamBridge backward update")
            self._refresh()
        upd, comm = self._update_stream, self._comm_stream
        upd.wait_stream(comm if comm is not None else torch.cuda.current_stream(self.device))
        with torch.cuda.device(self.device):
            self._launch_round(r, self._target(False), None, self._backward_ctas)
        self._rounds_updated.add(r)

    def _updates_in_backward(self) -> bool:
        return self._hooked and self._update_in_backward and not self._delayed() and not self._delay_owed

    # ------------------------------------------------------------------ inspection

    def launches_per_step(self) -> int:
        """Kernel launches of one step (64 segments of one kind per launch)."""
        return sum(math.ceil(len(s) / 64) for s in self._segs)

    def memory_report(self) -> dict[str, int]:
        rep = {"master": self.master.nbytes, "moments": self.m.nbytes + (self.v.nbytes if self.v is not None else 0),
               "grad_shard": self.grad_shard.nbytes, "weights": self.flat_weights.nbytes,
               "delayed_weights": 0 if self._shadow is None else self._shadow.nbytes,
               "flat_grads": 0 if self._flat_grads is None else self._flat_grads.nbytes}
        rep["total"] = sum(rep.values())
        return rep

    # ------------------------------------------------------------------ checkpoints

    CKPT_ENTRIES = 1 << 25   # shard entries gathered per collective: bounds the temporary buffers

    @staticmethod
    def _raw(t: torch.Tensor) -> torch.Tensor:
        """Same bytes as an integer tensor (collectives and copies move bits, never convert values)."""
        return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])

    def _gather_plane(self, shard: torch.Tensor, dests: list[torch.Tensor], unit: int, padded: bool,
                      keep: bool) -> None:
        """Every rank's ``shard`` array, gathered ``CKPT_ENTRIES`` entries at a time, copied into the
        per-parameter host arrays ``dests`` (when ``keep``)."""
        L = self.layout
        runs = [L.shard_runs(k, unit, padded) for k in range(self.world)]
        raw = self._raw(shard)
        dst = [self._raw(d) for d in dests]
        n = raw.numel()
        for s0 in range(0, n, self.CKPT_ENTRIES):
            s1 = min(n, s0 + self.CKPT_ENTRIES)
            if self.world == 1:
                out = raw[s0:s1].unsqueeze(0)
            else:
                out = torch.empty((self.world, s1 - s0), dtype=raw.dtype, device=self.device)
                dist.all_gather_into_tensor(out, raw[s0:s1].contiguous(), group=self.pg)
            if not keep:
                continue
            host = out.cpu()
            for k in range(self.world):
                for index, p_lo, s_lo, length in runs[k]:
                    a, b = max(s_lo, s0), min(s_lo + length, s1)
                    if a < b:
                        dst[index][p_lo + a - s_lo:p_lo + b - s_lo].copy_(host[k, a - s0:b - s0])

    @torch.no_grad()
    def state_dict(self, rank0_only: bool = False) -> dict[str, Any]:
        """The AdamBridge checkpoint format (adambridge/optimizer.py:525-544): per-parameter master weights and
        moments, assembled from every rank's shard into host tensors -- loadable by ``AdamBridge`` and by a
        ZeRO optimizer of any world size.  Collective: every rank of the group must call it.  With
        ``rank0_only`` the other ranks take part in the gathers and return an empty ``state``."""
        self.flush()
        torch.cuda.current_stream(self.device).wait_stream(self._update_stream)
        sd = super().state_dict()
        sd["state"] = {}
        keep = not rank0_only or self.rank == 0
        L = self.layout
        masters = [StateBuffer.allocate(self.master_precision, "p", n, "cpu") for n in L.numels]
        stores = [("exp_avg", self.m, [StateBuffer.allocate(self.precision, "m", n, "cpu") for n in L.numels])]
        if self.v is not None:
            stores.append(("exp_avg_sq", self.v,
                           [StateBuffer.allocate(self.precision, "v", n, "cpu") for n in L.numels]))
        for shard_store, per_param in [(self.master, masters)] + [(st, pp) for _, st, pp in stores]:
            for j, (plane, unit, padded) in enumerate(shard_store.plane_runs()):
                self._gather_plane(plane, [p.plane_runs()[j][0] for p in per_param], unit, padded, keep)
        if keep and self.step_count > 0:
            for i in range(len(self._params)):
                m = masters[i]
                st = sd["state"][i] = {"step": self.step_count,
                                       "master": m.planes["data"] if m.fmt == "fp32" else m.checkpoint()}
                for key, _, per_param in stores:
                    st[key] = per_param[i].checkpoint()
        sd["adambridge"] = {"precision": self.precision, "master_precision": self.master_precision, "format": 1,
                            "algorithm": self._algorithm}
        return sd

    @torch.no_grad()
    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        """Load an AdamBridge / ZeRO checkpoint (the reference's dict format, any world size) or a
        ``torch.optim.AdamW`` one: every rank reads the whole checkpoint and keeps its own pieces; moments and
        master are converted to this optimizer's precisions.  The weights are the model's to load."""
        saved = {int(k) if isinstance(k, str) and k.isdigit() else k: v for k, v in state_dict["state"].items()}
        L = self.layout
        lion = self._algorithm == "lion"
        for index, st in saved.items():
            if isinstance(index, bool) or not isinstance(index, int) or not 0 <= index < len(self._params):
                raise ValueError(f"checkpoint state for parameter {index!r}: this optimizer has parameters "
                                 f"0..{len(self._params) - 1}")
            numel = L.numels[index]
            if st.get("master") is not None:
                check_master(st["master"], numel, f"master weights of parameter {index}")
            for key in ("exp_avg", "exp_avg_sq"):
                if key in st:
                    check_moment(st[key], numel, f"{key} of parameter {index}")
            if "exp_avg" not in st or (not lion and "exp_avg_sq" not in st):
                raise ValueError("checkpoint has no exp_avg / exp_avg_sq (saved by LionBridge?); AdamW needs both")
        if saved and len(saved) != len(self._params):
            raise ValueError(f"checkpoint holds state for {len(saved)} of {len(self._params)} parameters; a ZeRO "
                             "optimizer updates every parameter every step and needs all of them")
        steps = {int(st["step"].item() if isinstance(st["step"], torch.Tensor) else st["step"]) for st in saved.values()}
        if len(steps) > 1:
            raise ValueError(f"checkpoint parameters are at different steps {sorted(steps)}; ZeRO needs one")
        super().load_state_dict({"state": {}, "param_groups": state_dict["param_groups"]})
        dev = self.device
        torch.cuda.synchronize(dev)
        self._delay_owed = False          # a delayed update in flight is superseded by the loaded state
        runs = {}
        for unit, padded in ((1, False), (1, True), (ALIGN, True)):
            for index, p_lo, s_lo, length in L.shard_runs(self.rank, unit, padded):
                runs.setdefault((unit, padded, index), []).append((p_lo, s_lo, length))

        def scatter(shard_store, param_store, index):
            for (plane, unit, padded), (src, _, _) in zip(shard_store.plane_runs(), param_store.plane_runs()):
                raw, rsrc = self._raw(plane), self._raw(src)
                for p_lo, s_lo, length in runs.get((unit, padded, index), []):
                    raw[s_lo:s_lo + length].copy_(rsrc[p_lo:p_lo + length])

        with torch.cuda.device(dev):
            for index, st in saved.items():
                numel = L.numels[index]
                if st.get("master") is not None:
                    saved_master = StateBuffer.master_from_checkpoint(st["master"], numel, "master weights")
                    master = StateBuffer.converted(saved_master, self.master_precision, "p", dev)
                    scatter(self.master, master, index)
                for key, shard_store, role in (("exp_avg", self.m, "m"), ("exp_avg_sq", self.v, "v")):
                    if shard_store is None:
                        continue
                    scatter(shard_store, self._load_store(st[key], numel, role, dev), index)
        if saved:
            self.step_count = steps.pop()
        torch.cuda.synchronize(dev)

    def _load_store(self, saved, numel: int, role: str, device) -> StateBuffer:
        """A checkpoint moment (store dict or AdamW tensor) converted to this optimizer's precision on ``device``."""
        return StateBuffer.converted(StateBuffer.from_checkpoint(saved, numel, role, "moment"), self.precision, role,
                                     device)


class ZeroLionBridge(ZeroAdamBridge):
    """Lion with ZeRO-1-sharded GPU state (see :class:`ZeroAdamBridge`)."""

    _algorithm = "lion"

    def __init__(self, params, lr: float = 1e-4, betas: tuple[float, float] = (0.9, 0.99), weight_decay: float = 0.0,
                 **kwargs):
        if "eps" in kwargs:
            raise TypeError("ZeroLionBridge has no eps")
        super().__init__(params, lr=lr, betas=betas, eps=0.0, weight_decay=weight_decay, **kwargs)
