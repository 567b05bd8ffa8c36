"""AdamBridge / LionBridge on B200: the reference's optimizer API (adambridge/optimizer.py) with the FP32
master weights and moments resident in GPU memory and updated by the fused sm_100a kernels."""

from __future__ import annotations

import contextlib
import logging
import weakref
from typing import Any, Callable, Iterable

import torch

from .clip import clip_coefficient
from .engine import ParamSlot, SmallGroup, StepStats, UpdateEngine
from .precision import (FP32Store, _checked, bytes_per_param, canonical_master_precision, canonical_precision,
                        check_master_state, load_master_, make_store, master_to_fp32, store_from_state_dict)

__all__ = ["AdamBridge", "LionBridge", "OptiComputeAdamW"]

log = logging.getLogger("adambridge_b200")


class AdamBridge(torch.optim.Optimizer):
    r"""AdamW whose FP32 master weights and moments live in HBM, updated by one fused kernel pass.

    Numerically this is the reference ``adambridge.AdamBridge`` with its native backend: the same
    arithmetic as ``torch.optim.AdamW`` (decoupled weight decay, bias correction, same operation order), the
    same stochastic rounding of low-precision moments, bit for bit (see ``native.set_simd_level``).

    Two ways to drive it, as in the reference::

        loss.backward(); opt.step(); opt.zero_grad()          # synchronous drop-in

        opt.attach_hooks(model)                               # layer-wise: each parameter is updated on the
        loss.backward(); opt.step_sync()                      # GPU as soon as its gradient is complete

    In hook mode gradients are released as soon as the update kernel has been enqueued
    (``release_grads=True``).  Global gradient clipping needs every gradient first: in ``step()`` mode call
    ``opt.clip_grad_norm_(max_norm)`` (torch's ``clip_grad_norm_``, with the gradients scaled inside the next
    update instead of in place), or ``torch.nn.utils.clip_grad_norm_`` as usual, or pass any factor as a
    device scalar (``step(grad_scale=...)``).

    Args mirror the reference (adambridge/optimizer.py:126-151).  ``precision``: moment storage, ``'fp32'``,
    ``'bf16'`` (``'bf16_moments'``) or ``'fp8'`` (``'fp8_moments'``).  ``master_precision``: ``'fp32'`` or
    ``'fp24'``.  ``stochastic_rounding``, ``seed``, ``release_grads``, ``overlap_writeback``,
    ``small_param_threshold``, ``delay_updates``, ``delay_warmup_steps``, ``accumulation_steps`` have the
    reference's meaning.  Host-offload knobs (``backend``, ``numa_aware``, ``num_threads``, ``chunk_size``,
    ``autotune``, ``transfer_buffer_mb``, ``gpu_state_budget``) are validated as in the reference and have no
    effect: the state is on the GPU already.  ``max_ctas`` (new) caps the CTAs of each update launch, leaving
    SMs to the backward pass that hook-mode updates overlap (0: every SM).
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
        if not 0.0 <= lr:
            raise ValueError(f"invalid learning rate: {lr}")
        if delay_warmup_steps < 0 or accumulation_steps < 1:
            raise ValueError("delay_warmup_steps must be >= 0 and accumulation_steps >= 1")
        if not 0.0 <= eps:
            raise ValueError(f"invalid epsilon: {eps}")
        if not 0.0 <= betas[0] < 1.0 or not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"invalid betas: {betas}")
        if not 0.0 <= weight_decay:
            raise ValueError(f"invalid weight_decay: {weight_decay}")
        if chunk_size is not None and (chunk_size <= 0 or chunk_size % 128):
            raise ValueError("chunk_size must be a positive multiple of 128")
        if transfer_buffer_mb is not None and transfer_buffer_mb < 0:
            raise ValueError("transfer_buffer_mb must be >= 0")
        if not (gpu_state_budget is None or gpu_state_budget == "auto"
                or (isinstance(gpu_state_budget, int) and gpu_state_budget >= 0)):
            raise ValueError("gpu_state_budget must be None, 'auto' or a number of bytes >= 0")
        if gpu_state_budget and self._algorithm != "adamw":
            raise ValueError("gpu_state_budget is only available for AdamW")
        if max_ctas < 0:
            raise ValueError("max_ctas must be >= 0")
        self.gpu_state_budget = gpu_state_budget or None

        self.precision = canonical_precision(precision)
        self.master_precision = canonical_master_precision(master_precision)
        self.release_grads = release_grads
        self.small_param_threshold = small_param_threshold
        self._slots: dict[torch.Tensor, ParamSlot] = {}
        self._ordered: list[ParamSlot] = []
        self._hooks: list = []
        self._hooked = False
        self._accumulating = 0
        self.accumulation_steps = accumulation_steps
        self._micro = 0
        self._backward_counted = False
        self.delay_updates = delay_updates
        self.delay_warmup_steps = delay_warmup_steps
        self._steps_synced = 0
        self.last_step_stats: StepStats | None = None
        self._autotune_requested = bool(autotune)
        self._clip_coef: torch.Tensor | None = None

        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))

        self._engine = UpdateEngine(
            precision=self.precision, backend=backend, numa_aware=numa_aware, num_threads=num_threads,
            chunk_size=chunk_size, stochastic_rounding=stochastic_rounding, seed=seed,
            overlap_writeback=overlap_writeback, timing=False, algorithm=self._algorithm,
            transfer_buffer_bytes=None if transfer_buffer_mb is None else transfer_buffer_mb << 20,
            master_precision=self.master_precision, max_ctas=max_ctas)
        self._engine.delay = delay_updates and delay_warmup_steps == 0
        self._engine.may_delay = delay_updates
        self._finalizer = weakref.finalize(self, UpdateEngine.close, self._engine)
        self._small_groups = self._build_small_groups()

    # ---------------------------------------------------------------- groups

    def add_param_group(self, param_group: dict[str, Any]) -> None:
        super().add_param_group(param_group)
        group = self.param_groups[-1]
        for p in group["params"]:
            if p.is_sparse:
                raise ValueError("AdamBridge does not support sparse parameters")
            slot = ParamSlot(len(self._ordered), p, group)
            self._slots[p] = slot
            self._ordered.append(slot)
            if self._hooked and p.requires_grad:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._hook()))

    def _build_small_groups(self) -> list[SmallGroup]:
        by_key: dict[tuple, list[ParamSlot]] = {}
        for slot in self._ordered:
            p = slot.param
            if p.is_cuda and p.requires_grad and slot.numel < self.small_param_threshold:
                by_key.setdefault((p.device, p.dtype), []).append(slot)
        return [SmallGroup(slots) for slots in by_key.values()]

    def _rebind_groups(self) -> None:
        for group in self.param_groups:
            for p in group["params"]:
                self._slots[p].group = group

    # ------------------------------------------------------------ async mode

    def attach_hooks(self, model: torch.nn.Module | None = None) -> "AdamBridge":
        """Start updating each parameter as soon as its gradient is ready (only ``model``'s, if given)."""
        if self._hooked:
            return self
        wanted = None if model is None else {id(p) for p in model.parameters()}
        hook = self._hook()
        for slot in self._ordered:
            p = slot.param
            if p.requires_grad and slot.small is None and (wanted is None or id(p) in wanted):
                self._hooks.append(p.register_post_accumulate_grad_hook(hook))
        self._hooked = True
        return self

    def _hook(self):
        """The gradient hook, opaque to TorchDynamo (compiled autograd calls it instead of tracing it)."""
        return torch.compiler.disable(self._on_grad_ready)

    def detach_hooks(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks.clear()
        self._hooked = False

    @contextlib.contextmanager
    def no_sync(self):
        """Accumulate gradients without triggering updates (all but the last micro-batch)."""
        self._accumulating += 1
        try:
            yield
        finally:
            self._accumulating -= 1

    def _on_grad_ready(self, p: torch.Tensor) -> None:
        if self._accumulating or p.grad is None:
            return
        if self.accumulation_steps > 1:
            if not self._backward_counted:
                self._backward_counted = True
                torch.autograd.Variable._execution_engine.queue_callback(self._end_of_backward)
            if self._micro + 1 < self.accumulation_steps:
                return
        self._submit(self._slots[p], p.grad)
        if self.release_grads:
            p.grad = None

    def _end_of_backward(self) -> None:
        self._micro += 1
        self._backward_counted = False

    def _check_submit(self, slot: ParamSlot, grad: torch.Tensor) -> None:
        if slot.submitted:
            raise RuntimeError(
                "AdamBridge: parameter received a second gradient before step_sync(); "
                "run extra backward passes inside optimizer.no_sync() to accumulate gradients")
        if grad.is_sparse:
            raise RuntimeError("AdamBridge does not support sparse gradients")
        slot.submitted = True

    def _submit(self, slot: ParamSlot, grad: torch.Tensor) -> None:
        self._check_submit(slot, grad)
        self._engine.submit(slot, grad)

    def _flush_small(self, release: bool, g_scale: torch.Tensor | None = None) -> None:
        """Enqueue the small parameters' updates: one launch per group."""
        for group in self._small_groups:
            items = [(s, s.param.grad) for s in group.slots if not s.submitted and s.param.grad is not None]
            for slot, grad in items:
                self._check_submit(slot, grad)
            self._engine.submit_many(items, g_scale=g_scale)
            if release:
                for slot, _ in items:
                    slot.param.grad = None

    def step_sync(self) -> StepStats:
        """Update the small parameters and order every update before later work on the current stream.
        With delayed updates, enqueue and return."""
        try:
            if not self._accumulating:
                if self.accumulation_steps > 1:
                    self._submit_remaining()
                self._flush_small(release=self.release_grads and self._hooked)
            stats = self._engine.finish_step()
        finally:
            for slot in self._ordered:
                slot.submitted = False
            self._micro = 0
        self.last_step_stats = stats
        self._steps_synced += 1
        if self.delay_updates and self._steps_synced >= self.delay_warmup_steps:
            self._engine.delay = True
        return stats

    def _submit_remaining(self, g_scale: torch.Tensor | None = None) -> None:
        """Every large parameter with a gradient not yet updated, in one batched launch."""
        items = []
        for slot in self._ordered:
            if not slot.submitted and slot.small is None and slot.param.grad is not None:
                self._check_submit(slot, slot.param.grad)
                items.append((slot, slot.param.grad))
        self._engine.submit_many(items, g_scale=g_scale)

    def flush(self) -> None:
        """Apply every pending update to the parameters (delayed mode: call before evaluating or saving)."""
        self._engine.flush()

    # ------------------------------------------------------------- sync mode

    @torch.no_grad()
    def step(self, closure: Callable[[], torch.Tensor] | None = None, grad_scale: torch.Tensor | None = None):
        """Update every parameter that has a gradient and was not already updated by a hook, then
        :meth:`step_sync`.  ``grad_scale`` (a one-element float32 CUDA tensor) multiplies every gradient
        inside the kernel -- e.g. the clip coefficient -- with the rounding of an in-place multiply."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if self._clip_coef is not None:
            if grad_scale is not None:
                raise ValueError("step(grad_scale=...) after clip_grad_norm_(): the clip coefficient is the scale")
            grad_scale, self._clip_coef = self._clip_coef, None
        self._submit_remaining(grad_scale)
        self._flush_small(release=False, g_scale=grad_scale)
        self.step_sync()
        return loss

    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float, norm_type: float = 2.0, error_if_nonfinite: bool = False,
                        foreach: bool | None = None) -> torch.Tensor:
        """``torch.nn.utils.clip_grad_norm_`` over this optimizer's gradients, fused into the next :meth:`step`.

        Returns the total L2 norm (a device tensor in the gradients' dtype, as torch returns it) without a host
        synchronization.  The gradients are not modified: the next ``step()`` multiplies each one by the clipping
        coefficient inside the update kernel, rounding to the gradient's dtype exactly as torch's in-place
        multiply does, so ``opt.clip_grad_norm_(c); opt.step()`` equals ``clip_grad_norm_(params, c); opt.step()``.
        The norms come from libabx's multi-tensor norm kernels (one read of the gradients).  Only the L2 norm is
        fused; bf16 and fp32 gradients may be mixed (norms rounded per dtype, the total in fp32, as torch does).
        ``error_if_nonfinite`` synchronizes to check the norm."""
        del foreach
        if float(norm_type) != 2.0:
            raise ValueError("AdamBridge.clip_grad_norm_ computes the L2 norm (norm_type=2) only")
        if any(slot.submitted for slot in self._ordered):
            raise RuntimeError("clip_grad_norm_ after a hook already updated parameters: clip before any update")
        grads = [slot.param.grad for slot in self._ordered if slot.param.grad is not None]
        if not grads:
            return torch.tensor(0.0)
        total, coef, _ = clip_coefficient(grads, max_norm, kernels=self._engine.native)
        if error_if_nonfinite and not torch.isfinite(total).item():
            raise RuntimeError(f"The total norm of order 2.0 for gradients from `parameters` is non-finite, "
                               "so it cannot be clipped.")
        self._clip_coef = coef
        return total

    # ------------------------------------------------------------- precision

    def set_precision(self, precision: str) -> None:
        """Re-encode all moments in another precision (between steps)."""
        precision = canonical_precision(precision)
        self._engine.wait()
        if precision == self.precision:
            return
        for slot in self._ordered:
            if slot.initialized:
                self._engine.convert_moments(slot, precision)
        self.precision = self._engine.precision = precision

    @property
    def autotune_log(self) -> list[str]:
        return []

    def tune_threads(self, numel: int = 1 << 22) -> dict[str, dict[int, float]]:
        return {}

    # ------------------------------------------------------------ inspection

    @property
    def backend(self) -> str:
        return f"cuda/sm_100a ({self._engine.native.simd_level} rounding)"

    def memory_report(self) -> dict[str, int]:
        """Bytes held by the optimizer on the GPU, by category (the reference reports host bytes)."""
        report = {"master": 0, "moments": 0, "staging": 0}
        for slot in self._ordered:
            if not slot.initialized:
                continue
            if not slot.in_place:
                report["master"] += slot.master.nbytes
            report["moments"] += slot.m.nbytes + (slot.v.nbytes if slot.v is not None else 0)
            if slot.out is not None:
                report["staging"] += slot.out.nbytes
        report["total"] = sum(report.values())
        report["gpu_state"] = report["total"]
        return report

    def expected_bytes_per_param(self) -> float:
        return bytes_per_param(self.precision, 1 if self._algorithm == "lion" else 2, master=self.master_precision)

    def master_params(self) -> list[torch.Tensor | None]:
        """FP32 master copies (``None`` before a parameter's first update; a decoded copy for an FP24 master)."""
        self._engine.wait()
        return [_master_fp32(slot) if slot.initialized else None for slot in self._ordered]

    # ------------------------------------------------------------ checkpoint

    def state_dict(self) -> dict[str, Any]:
        """The reference's checkpoint format (adambridge/optimizer.py:525-544); tensors stay on the GPU.
        Also applies pending delayed updates."""
        self._engine.flush()
        self._engine.wait()
        sd = super().state_dict()
        sd["state"] = {}
        for slot in self._ordered:
            if slot.initialized:
                master = slot.master.data if isinstance(slot.master, FP32Store) else slot.master.state_dict()
                st = sd["state"][slot.index] = {"step": slot.step, "master": master, "exp_avg": slot.m.state_dict()}
                if slot.v is not None:
                    st["exp_avg_sq"] = slot.v.state_dict()
        sd["adambridge"] = {"precision": self.precision, "master_precision": self.master_precision, "format": 1,
                            "algorithm": self._algorithm}
        return sd

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        """Load an AdamBridge/LionBridge checkpoint (from this package or the reference), or a
        ``torch.optim.AdamW`` one; moments are converted to this optimizer's precision."""
        self._engine.discard_pending()
        saved = {int(k) if isinstance(k, str) and k.isdigit() else k: v for k, v in state_dict["state"].items()}
        lion = self._algorithm == "lion"
        for index, st in saved.items():
            if isinstance(index, bool) or not isinstance(index, int) or not 0 <= index < len(self._ordered):
                raise ValueError(f"checkpoint state for parameter {index!r}: this optimizer has parameters "
                                 f"0..{len(self._ordered) - 1}")
            numel = self._ordered[index].numel
            if st.get("master") is not None:
                check_master_state(st["master"], numel, f"master weights of parameter {index}")
            for key in ("exp_avg", "exp_avg_sq"):
                if isinstance(st.get(key), torch.Tensor):
                    _checked(st[key], numel, f"{key} of parameter {index}")
        super().load_state_dict({"state": {}, "param_groups": state_dict["param_groups"]})
        self._rebind_groups()
        for index, st in saved.items():
            slot = self._ordered[index]
            if not lion and "exp_avg_sq" not in st:
                raise ValueError("checkpoint has no exp_avg_sq (saved by LionBridge?); AdamW needs both moments")
            if not slot.initialized:
                self._engine.initialize(slot)
            slot.step = int(st["step"])
            dev = slot.param.device
            with torch.no_grad(), torch.cuda.device(dev):
                if st.get("master") is not None:
                    load_master_(slot.master, st["master"])
                self._engine.replace_moments(
                    slot, self._load_store(st["exp_avg"], slot.numel, "m", dev),
                    None if lion else self._load_store(st["exp_avg_sq"], slot.numel, "v", dev))

    def _load_store(self, saved, numel: int, role: str, device):
        if isinstance(saved, torch.Tensor):  # torch.optim.AdamW layout
            return make_store(self.precision, numel, role, init=saved.to(device, torch.float32), device=device)
        store = store_from_state_dict(saved, numel, role, device=device)
        if store.precision != self.precision:
            store = make_store(self.precision, numel, role, init=store.to_fp32(), device=device)
        return store

    def close(self) -> None:
        """Apply pending delayed updates and release the engine."""
        self.detach_hooks()
        if self._finalizer.alive:
            try:
                self._engine.flush()
            finally:
                self._finalizer()


def _master_fp32(slot: ParamSlot) -> torch.Tensor:
    return slot.master.data if isinstance(slot.master, FP32Store) else slot.master.to_fp32()


OptiComputeAdamW = AdamBridge


class LionBridge(AdamBridge):
    r"""Lion (Chen et al., 2023) with the same GPU-resident state and kernels as :class:`AdamBridge`::

        c = beta1 * m + (1 - beta1) * g
        p = p * (1 - lr * weight_decay) - lr * sign(c)
        m = beta2 * m + (1 - beta2) * g

    Every keyword argument of :class:`AdamBridge` except ``eps`` applies.  The moment is saved as ``exp_avg``.
    """

    _algorithm = "lion"

    def __init__(self, params, lr: float = 1e-4, betas: tuple[float, float] = (0.9, 0.99),
                 weight_decay: float = 0.0, **kwargs):
        if "eps" in kwargs:
            raise TypeError("LionBridge has no eps")
        super().__init__(params, lr=lr, betas=betas, eps=0.0, weight_decay=weight_decay, **kwargs)
