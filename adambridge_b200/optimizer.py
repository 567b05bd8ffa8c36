"""AdamBridge / OptiComputeAdamW / LionBridge: adambridge's optimizer API over optimizer state held in HBM.

The public surface is the reference's (adambridge/optimizer.py:24-659): the constructor and its arguments, the
two ways of driving it (``step()`` after backward, or ``attach_hooks()`` + ``step_sync()``), ``no_sync`` and
``accumulation_steps``, delayed updates, ``set_precision``, ``flush``, ``state_dict`` / ``load_state_dict``
in the reference's checkpoint format, ``memory_report``, ``master_params`` and ``close``.

Underneath there is no host state and no worker: a parameter's update is one entry of a batched launch of the
fused kernel on the device's update stream (``engine.UpdateEngine``).  So the optimizer only decides *when* a
parameter is enqueued and keeps a ledger of what this step has enqueued:

* hook mode: a parameter is enqueued the moment autograd finishes its gradient (the last micro-batch's, when
  accumulating); parameters smaller than ``small_param_threshold`` are not hooked and go in one launch at
  ``step_sync``;
* ``step()``: everything with a gradient that the ledger does not hold goes in one batched launch.
"""

from __future__ import annotations

import contextlib
import logging
import weakref
from typing import Any, Callable, Iterable

import torch

from .clip import clip_coefficient
from .engine import ParamSlot, StepStats, UpdateEngine
from .precision import StateBuffer, bytes_per_param, master_format, moment_format

__all__ = ["AdamBridge", "LionBridge", "OptiComputeAdamW"]

log = logging.getLogger("adambridge_b200")


def _validate(lr, betas, eps, weight_decay, delay_warmup_steps, accumulation_steps, chunk_size, transfer_buffer_mb,
              gpu_state_budget, algorithm, max_ctas) -> None:
    """The constructor's argument checks (the reference's, adambridge/optimizer.py:152-170, plus max_ctas)."""
    budget_ok = (gpu_state_budget is None or gpu_state_budget == "auto"
                 or (isinstance(gpu_state_budget, int) and not isinstance(gpu_state_budget, bool)
                     and gpu_state_budget >= 0))
    rules = [
        (lr >= 0.0, f"invalid learning rate: {lr}"),
        (delay_warmup_steps >= 0 and accumulation_steps >= 1,
         "delay_warmup_steps must be >= 0 and accumulation_steps >= 1"),
        (eps >= 0.0, f"invalid epsilon: {eps}"),
        (0.0 <= betas[0] < 1.0 and 0.0 <= betas[1] < 1.0, f"invalid betas: {betas}"),
        (weight_decay >= 0.0, f"invalid weight_decay: {weight_decay}"),
        (chunk_size is None or (chunk_size > 0 and chunk_size % 128 == 0),
         "chunk_size must be a positive multiple of 128"),
        (transfer_buffer_mb is None or transfer_buffer_mb >= 0, "transfer_buffer_mb must be >= 0"),
        (budget_ok, "gpu_state_budget must be None, 'auto' or a number of bytes >= 0"),
        (not gpu_state_budget or algorithm == "adamw", "gpu_state_budget is only available for AdamW"),
        (max_ctas >= 0, "max_ctas must be >= 0"),
    ]
    for ok, message in rules:
        if not ok:
            raise ValueError(message)


class _MicroBatches:
    """Counts backward passes for ``accumulation_steps``: the first gradient of a pass queues a callback that
    autograd runs when the pass ends; gradients of every pass but the last of a window are left to accumulate."""

    def __init__(self, window: int):
        self.window = window
        self.finished = 0          # passes completed since the last step_sync
        self._armed = False        # this pass's end-of-pass callback is queued

    def gradient_seen(self) -> bool:
        """Called for a finished gradient; True if it belongs to the window's last pass (update it now)."""
        if self.window == 1:
            return True
        if not self._armed:
            self._armed = True
            torch.autograd.Variable._execution_engine.queue_callback(self._pass_ended)
        return self.finished + 1 >= self.window

    def _pass_ended(self) -> None:
        self.finished += 1
        self._armed = False

    def reset(self) -> None:
        self.finished = 0


class AdamBridge(torch.optim.Optimizer):
    r"""AdamW with FP32 master weights and moments resident in HBM, updated by one fused kernel pass.

    The arithmetic is the reference ``adambridge.AdamBridge``'s with its native backend -- torch.optim.AdamW's
    update (decoupled weight decay, bias correction, the same operation order) and the same stochastic rounding
    of low-precision state -- bit for bit at the reference's SIMD level (``native.set_simd_level``)::

        loss.backward(); opt.step(); opt.zero_grad()          # after backward

        opt.attach_hooks(model)                               # each parameter updated as soon as its gradient
        loss.backward(); opt.step_sync()                      # is complete, while backward goes on

    Clipping: ``opt.clip_grad_norm_(max_norm)`` before ``step()`` (torch's clip_grad_norm_, applied inside the
    next update instead of rewriting the gradients), or ``torch.nn.utils.clip_grad_norm_`` as usual, or any
    factor as a device scalar, ``step(grad_scale=...)``.

    Arguments are the reference's (adambridge/optimizer.py:126-151): ``precision`` stores the moments as
    ``'fp32'``, ``'bf16'`` (``'bf16_moments'``) or ``'fp8'`` (``'fp8_moments'``); ``master_precision`` is
    ``'fp32'`` or ``'fp24'``; ``stochastic_rounding``, ``seed``, ``release_grads``, ``overlap_writeback``,
    ``small_param_threshold``, ``delay_updates``, ``delay_warmup_steps`` and ``accumulation_steps`` mean what
    they mean there.  The host-offload arguments (``backend``, ``numa_aware``, ``num_threads``, ``chunk_size``,
    ``autotune``, ``transfer_buffer_mb``, ``gpu_state_budget``) are checked as the reference checks them and
    change nothing: the state is on the GPU already.  ``max_ctas`` (not in the reference) caps the CTAs of each
    update launch, leaving SMs to the backward pass a hook-mode update overlaps (0: every SM).
    """

    _algorithm = "adamw"

    def __init__(
        self,
        params: Iterable[torch.Tensor] | Iterable[dict[str, Any]],
        lr: float = 1e-3,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 1e-2,
        *,
        precision: str = "fp32",
        stochastic_rounding: bool = True,
        backend: str = "auto",
        numa_aware: bool = True,
        num_threads: int | None = None,
        chunk_size: int | None = None,
        release_grads: bool = True,
        overlap_writeback: bool = True,
        autotune: bool | Any = False,
        seed: int = 0,
        small_param_threshold: int = 65536,
        delay_updates: bool = False,
        delay_warmup_steps: int = 0,
        accumulation_steps: int = 1,
        transfer_buffer_mb: int | None = None,
        gpu_state_budget: int | str | None = None,
        master_precision: str = "fp32",
        max_ctas: int = 0,
    ):
        _validate(lr, betas, eps, weight_decay, delay_warmup_steps, accumulation_steps, chunk_size,
                  transfer_buffer_mb, gpu_state_budget, self._algorithm, max_ctas)
        self.precision = moment_format(precision)
        self.master_precision = master_format(master_precision)
        self.gpu_state_budget = gpu_state_budget or None
        self.release_grads = release_grads
        self.small_param_threshold = small_param_threshold
        self.accumulation_steps = accumulation_steps
        self.delay_updates = delay_updates
        self.delay_warmup_steps = delay_warmup_steps
        self.last_step_stats: StepStats | None = None
        self.slots: list[ParamSlot] = []               # one per parameter, in optimizer order
        self._slot_of: dict[int, ParamSlot] = {}       # id(parameter) -> slot
        self._enqueued: set[int] = set()               # slot indices updated since the last step_sync
        self._hook_handles: list = []
        self._hooks_on = False
        self._no_sync_depth = 0
        self._passes = _MicroBatches(accumulation_steps)
        self._syncs = 0
        self._clip_coef: torch.Tensor | None = None
        self._engine: UpdateEngine | None = None

        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))

        self._engine = UpdateEngine(
            precision=self.precision, backend=backend, numa_aware=numa_aware, num_threads=num_threads,
            chunk_size=chunk_size, stochastic_rounding=stochastic_rounding, seed=seed,
            overlap_writeback=overlap_writeback, timing=False, algorithm=self._algorithm,
            transfer_buffer_bytes=None if transfer_buffer_mb is None else transfer_buffer_mb << 20,
            master_precision=self.master_precision, max_ctas=max_ctas)
        self._engine.may_delay = delay_updates
        self._engine.delay = delay_updates and delay_warmup_steps == 0
        self._finalizer = weakref.finalize(self, UpdateEngine.close, self._engine)

    # ------------------------------------------------------------------ parameters

    def add_param_group(self, param_group: dict[str, Any]) -> None:
        super().add_param_group(param_group)
        group = self.param_groups[-1]
        for p in group["params"]:
            if p.is_sparse:
                raise ValueError("AdamBridge does not support sparse parameters")
            slot = ParamSlot(len(self.slots), p, group)
            slot.small = p.numel() < self.small_param_threshold
            self.slots.append(slot)
            self._slot_of[id(p)] = slot
            if self._hooks_on:
                self._hook_one(slot)

    def _regroup(self) -> None:
        """Point every slot at its group dict again (Optimizer.load_state_dict replaces the dicts)."""
        for group in self.param_groups:
            for p in group["params"]:
                self._slot_of[id(p)].group = group

    # ------------------------------------------------------------------ hook mode

    def attach_hooks(self, model: torch.nn.Module | None = None) -> "AdamBridge":
        """Update each parameter (only ``model``'s, if given) as soon as autograd has finished its gradient."""
        if not self._hooks_on:
            wanted = None if model is None else {id(p) for p in model.parameters()}
            for slot in self.slots:
                if wanted is None or id(slot.param) in wanted:
                    self._hook_one(slot)
            self._hooks_on = True
        return self

    def _hook_one(self, slot: ParamSlot) -> None:
        if slot.param.requires_grad and not slot.small:
            # opaque to TorchDynamo: compiled autograd calls the hook instead of tracing the enqueue
            hook = torch.compiler.disable(self._gradient_ready)
            self._hook_handles.append(slot.param.register_post_accumulate_grad_hook(hook))

    def detach_hooks(self) -> None:
        while self._hook_handles:
            self._hook_handles.pop().remove()
        self._hooks_on = False

    @contextlib.contextmanager
    def no_sync(self):
        """Let gradients accumulate without any update (every micro-batch but the last)."""
        self._no_sync_depth += 1
        try:
            yield
        finally:
            self._no_sync_depth -= 1

    def _gradient_ready(self, p: torch.Tensor) -> None:
        if self._no_sync_depth or p.grad is None or not self._passes.gradient_seen():
            return
        self._enqueue([self._slot_of[id(p)]])
        if self.release_grads:
            p.grad = None

    # ------------------------------------------------------------------ enqueueing updates

    def _claim(self, slot: ParamSlot) -> torch.Tensor:
        """The slot's gradient, recording in the ledger that this step updates it."""
        if slot.index in self._enqueued:
            raise RuntimeError(f"parameter {slot.index} got a second gradient before step_sync(); run all but the "
                               "last backward pass of an accumulation window inside optimizer.no_sync()")
        grad = slot.param.grad
        if grad.is_sparse:
            raise RuntimeError("AdamBridge does not support sparse gradients")
        self._enqueued.add(slot.index)
        return grad

    def _enqueue(self, slots: list[ParamSlot], g_scale: torch.Tensor | None = None) -> None:
        """One batched launch per device for ``slots`` (each with a gradient, none in the ledger yet)."""
        if slots:
            self._engine.submit_many([(s, self._claim(s)) for s in slots], g_scale=g_scale)

    def _outstanding(self, small: bool | None) -> list[ParamSlot]:
        """Slots with a gradient that this step has not updated (only small / only large ones, or all)."""
        return [s for s in self.slots if s.index not in self._enqueued and s.param.grad is not None
                and (small is None or s.small == small)]

    def step_sync(self) -> StepStats:
        """Update what hooks left (small parameters, or a window the hooks never completed) and order every update
        of this step before later work on the current stream.  With delayed updates: enqueue and return."""
        try:
            if not self._no_sync_depth:
                leftovers = self._outstanding(small=None if self.accumulation_steps > 1 else True)
                self._enqueue(leftovers)
                if self.release_grads and self._hooks_on:
                    for s in leftovers:
                        if s.small:   # as a hook releases a large parameter's gradient
                            s.param.grad = None
            stats = self._engine.finish_step()
        finally:
            self._enqueued.clear()
            self._passes.reset()
        self.last_step_stats = stats
        self._syncs += 1
        if self.delay_updates and self._syncs >= self.delay_warmup_steps:
            self._engine.delay = True
        return stats

    @torch.no_grad()
    def step(self, closure: Callable[[], torch.Tensor] | None = None, grad_scale: torch.Tensor | None = None):
        """Update every parameter that has a gradient and that no hook updated this step -- all in one batched
        launch per device -- then :meth:`step_sync`.  ``grad_scale`` (a one-element float32 CUDA tensor)
        multiplies every gradient inside the kernel, rounded as an in-place multiply of the gradient would be."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        coef, self._clip_coef = self._clip_coef, None
        if coef is not None:
            if grad_scale is not None:
                raise ValueError("step(grad_scale=...) after clip_grad_norm_(): the clip coefficient is the scale")
            grad_scale = coef
        self._enqueue(self._outstanding(small=None), g_scale=grad_scale)
        self.step_sync()
        return loss

    def flush(self) -> None:
        """Write every pending update into the parameters (delayed mode: before evaluating or saving)."""
        self._engine.flush()

    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float, norm_type: float = 2.0, error_if_nonfinite: bool = False,
                        foreach: bool | None = None) -> torch.Tensor:
        """``torch.nn.utils.clip_grad_norm_`` over this optimizer's gradients, applied by the next :meth:`step`.

        Returns the total L2 norm (a device tensor in the gradients' dtype, as torch returns it) without a host
        synchronization, from libabx's norm kernels (one read of the gradients).  The gradients stay as they
        are: the next ``step()`` multiplies each by the coefficient inside the update kernel, rounded to the
        gradient's dtype as torch's in-place multiply rounds it, so ``opt.clip_grad_norm_(c); opt.step()``
        equals ``clip_grad_norm_(params, c); opt.step()``.  L2 only; bf16 and fp32 gradients may be mixed.
        ``error_if_nonfinite`` synchronizes to look at the norm."""
        del foreach
        if float(norm_type) != 2.0:
            raise ValueError("AdamBridge.clip_grad_norm_ computes the L2 norm (norm_type=2) only")
        if self._enqueued:
            raise RuntimeError("clip_grad_norm_ after a hook already updated parameters: clip before any update")
        grads = [s.param.grad for s in self.slots if s.param.grad is not None]
        if not grads:
            return torch.tensor(0.0)
        total, coef, _ = clip_coefficient(grads, max_norm, kernels=self._engine.native)
        if error_if_nonfinite and not bool(torch.isfinite(total)):
            raise RuntimeError("The total norm of order 2.0 for gradients from `parameters` is non-finite, so it "
                               "cannot be clipped.")
        self._clip_coef = coef
        return total

    # ------------------------------------------------------------------ precision

    def set_precision(self, precision: str) -> None:
        """Re-encode every moment in another precision (between steps), on the device."""
        target = moment_format(precision)
        self._engine.wait()
        if target != self.precision:
            for slot in self.slots:
                if slot.initialized:
                    self._engine.convert_moments(slot, target)
            self.precision = self._engine.precision = target

    @property
    def autotune_log(self) -> list[str]:
        """The reference's autotuner picks host thread counts and precisions; nothing is tuned here."""
        return []

    def tune_threads(self, numel: int = 1 << 22) -> dict[str, dict[int, float]]:
        """No host threads to tune (the reference benchmarks its thread pool here)."""
        return {}

    # ------------------------------------------------------------------ inspection

    @property
    def backend(self) -> str:
        return f"cuda/sm_100a ({self._engine.native.simd_level} rounding)"

    def memory_report(self) -> dict[str, int]:
        """Device bytes the optimizer holds, by category (the reference reports host bytes)."""
        live = [s for s in self.slots if s.initialized]
        report = {"master": sum(s.master.nbytes for s in live if not s.in_place),
                  "moments": sum(s.m.nbytes + (s.v.nbytes if s.v is not None else 0) for s in live),
                  "staging": sum(s.out.nbytes for s in live if s.out is not None)}
        report["total"] = sum(report.values())
        report["gpu_state"] = report["total"]
        return report

    def expected_bytes_per_param(self) -> float:
        return bytes_per_param(self.precision, 1 if self._algorithm == "lion" else 2, master=self.master_precision)

    def master_params(self) -> list[torch.Tensor | None]:
        """FP32 master weights per parameter: the live tensor for an fp32 master, a decoded copy for an fp24 one,
        None before the parameter's first update."""
        self._engine.wait()
        return [None if not s.initialized else
                (s.master.planes["data"] if s.master.fmt == "fp32" else s.master.to_fp32()) for s in self.slots]

    # ------------------------------------------------------------------ checkpoints

    def state_dict(self) -> dict[str, Any]:
        """The reference's checkpoint format (adambridge/optimizer.py:525-544), tensors left on the GPU.  Pending
        delayed updates are applied first, so the weights match the saved master."""
        self._engine.flush()
        self._engine.wait()
        sd = super().state_dict()
        per_param = {}
        for s in self.slots:
            if not s.initialized:
                continue
            entry = {"step": s.step,
                     "master": s.master.planes["data"] if s.master.fmt == "fp32" else s.master.checkpoint(),
                     "exp_avg": s.m.checkpoint()}
            if s.v is not None:
                entry["exp_avg_sq"] = s.v.checkpoint()
            per_param[s.index] = entry
        sd["state"] = per_param
        sd["adambridge"] = {"precision": self.precision, "master_precision": self.master_precision, "format": 1,
                            "algorithm": self._algorithm}
        return sd

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        """Load an AdamBridge / LionBridge checkpoint (from this package or the reference) or a
        ``torch.optim.AdamW`` one.  Everything is checked before anything changes; moments and master weights
        are converted on the GPU to this optimizer's precisions."""
        self._engine.discard_pending()
        parsed = self._parse_checkpoint(state_dict)
        super().load_state_dict({"state": {}, "param_groups": state_dict["param_groups"]})
        self._regroup()
        for index, (step, master, moments) in parsed.items():
            slot = self.slots[index]
            if not slot.initialized:
                self._engine.initialize(slot)
            slot.step = step
            dev = slot.param.device
            with torch.no_grad(), torch.cuda.device(dev):
                if master is not None:
                    slot.master.assign(master)
                fresh = [StateBuffer.converted(src, self.precision, role, dev) for role, src in moments]
            self._engine.replace_moments(slot, fresh[0], fresh[1] if len(fresh) > 1 else None)

    def _parse_checkpoint(self, state_dict: dict[str, Any]) -> dict[int, tuple]:
        """{parameter index: (step, master buffer or None, [(role, moment buffer)])}, every field checked; the
        buffers view the checkpoint's tensors where they are."""
        roles = [("exp_avg", "m")] if self._algorithm == "lion" else [("exp_avg", "m"), ("exp_avg_sq", "v")]
        out = {}
        for key, entry in state_dict["state"].items():
            index = int(key) if isinstance(key, str) and key.isdigit() else key
            if isinstance(index, bool) or not isinstance(index, int) or not 0 <= index < len(self.slots):
                raise ValueError(f"checkpoint state for parameter {key!r}: this optimizer has parameters "
                                 f"0..{len(self.slots) - 1}")
            numel = self.slots[index].numel
            missing = [name for name, _ in roles if name not in entry]
            if missing:
                raise ValueError(f"checkpoint parameter {index} has no {' or '.join(missing)} (saved by LionBridge?): "
                                 f"{type(self).__name__} needs {len(roles)} moment(s)")
            master = None
            if entry.get("master") is not None:
                master = StateBuffer.master_from_checkpoint(entry["master"], numel, f"master weights of parameter {index}")
            moments = [(role, StateBuffer.from_checkpoint(entry[name], numel, role, f"{name} of parameter {index}"))
                       for name, role in roles]
            step = entry["step"]
            out[index] = (int(step.item() if isinstance(step, torch.Tensor) else step), master, moments)
        return out

    def close(self) -> None:
        """Apply pending delayed updates and release the engine (collection releases it without applying)."""
        self.detach_hooks()
        if self._finalizer.alive:
            try:
                self._engine.flush()
            finally:
                self._finalizer()


OptiComputeAdamW = AdamBridge


class LionBridge(AdamBridge):
    r"""Lion (Chen et al., 2023) on the same HBM-resident state and fused kernels as :class:`AdamBridge`::

        c = beta1 * m + (1 - beta1) * g
        p = p * (1 - lr * weight_decay) - lr * sign(c)
        m = beta2 * m + (1 - beta2) * g

    It keeps one moment (saved as ``exp_avg``); every keyword of :class:`AdamBridge` but ``eps`` applies.
    """

    _algorithm = "lion"

    def __init__(self, params, lr: float = 1e-4, betas: tuple[float, float] = (0.9, 0.99),
                 weight_decay: float = 0.0, **kwargs):
        if "eps" in kwargs:
            raise TypeError("LionBridge takes no eps")
        super().__init__(params, lr=lr, betas=betas, eps=0.0, weight_decay=weight_decay, **kwargs)
