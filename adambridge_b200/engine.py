"""Update engine: the fused kernels on a side CUDA stream, ordered by stream dependencies.

The reference engine (adambridge/engine.py:1-73) moves each gradient to pinned host
memory, updates host-resident state on a native thread pool and copies the new weights
back.  Here the optimizer state lives in HBM next to the parameters, so one update is::

    autograd thread (hook)          update stream (per device)
    ----------------------          --------------------------
    grad ready
    update stream waits on the
    current (compute) stream  --->  fused kernel: reads grad, master, moments;
                                    writes master, moments and the new weights
                                    straight into param.data
    ...backward continues on the compute stream for earlier layers...

``finish_step`` makes the caller's current stream wait on the update stream, so the
next forward pass sees the new weights.  A batch of updates (``step()``, the small
parameters at ``step_sync``) is one ``abx_multi_step`` call: one kernel launch per
(algorithm, moment, master) combination for up to 64 tensors.

**Delayed updates** (``delay = True``, adambridge/engine.py:46-69): the kernel writes
the new weights to the slot's ``out`` buffer instead of the parameter.  At the next
step's gradient of that parameter the update stream first copies ``out`` into the
parameter, then runs the new update; ``finish_step`` waits only for those copies (an
event recorded after them), so this step's updates overlap the next forward pass.  The
model trains with weights one step stale, exactly as the reference's delayed mode.

``overlap_writeback=False``: updates write ``out``, and every copy to the parameters is
issued in ``finish_step`` (for code that reads a parameter during backward after its
gradient is complete).
"""

from __future__ import annotations

import ctypes
import logging
import threading
import time
from dataclasses import dataclass, field

import torch

from . import native
from .native import StepCoefficients, mix_seed
from .precision import StateBuffer

__all__ = ["UpdateEngine", "ParamSlot", "StepStats"]

log = logging.getLogger("adambridge_b200")

_MASK64 = (1 << 64) - 1
_OUT_DTYPES = (torch.float32, torch.bfloat16)
_GRAD_DTYPES = (torch.float32, torch.bfloat16)


class ParamSlot:
    """Device-side optimizer state for one parameter."""

    __slots__ = ("index", "param", "group", "numel", "step", "master", "out", "m", "v", "seg", "seg_group", "small",
                 "in_place")

    def __init__(self, index: int, param: torch.Tensor, group: dict):
        self.index = index
        self.param = param
        self.group = group
        self.numel = param.numel()
        self.step = 0
        self.master: StateBuffer | None = None  # fp32 (maybe viewing the FP32 parameter itself) or fp24
        self.out: torch.Tensor | None = None     # new weights when not written to the parameter directly
        self.m: StateBuffer | None = None
        self.v: StateBuffer | None = None        # None for Lion
        self.seg: native.Segment | None = None   # kernel description of the buffers above
        self.seg_group = None
        self.small = False                       # updated at step_sync with the other small parameters, not hooked
        self.in_place = False                    # the master is the parameter itself (FP32 + fp32 master)

    @property
    def initialized(self) -> bool:
        return self.master is not None

    @property
    def gpu(self):
        """Kept for API parity with the reference (its GPU-resident subset); all state is on the GPU here."""
        return None


@dataclass
class StepStats:
    """Timing of one optimizer step (seconds)."""

    num_updates: int = 0
    gpu_backward: float | None = None  # first to last gradient-ready event, on the GPU (timing=True)
    gpu_update: float | None = None    # first update start to last update end on the update streams (timing=True)
    cpu_update: float = 0.0            # host time spent describing and launching updates
    stall: float = 0.0                 # time finish_step blocked the caller
    per_device_cpu: dict[str, float] = field(default_factory=dict)


class UpdateEngine:
    def __init__(
        self,
        *,
        precision: str,
        backend: str = "auto",
        numa_aware: bool = True,
        num_threads: int | None = None,
        chunk_size: int | None = None,
        stochastic_rounding: bool = True,
        seed: int = 0,
        overlap_writeback: bool = True,
        timing: bool = False,
        algorithm: str = "adamw",
        transfer_buffer_bytes: int | None = None,
        master_precision: str = "fp32",
        max_ctas: int = 0,
    ):
        if backend not in ("auto", "native", "torch"):
            raise ValueError("backend must be 'auto', 'native' or 'torch'")
        if backend == "torch":
            raise ValueError("backend='torch' is not available: the update runs only as the sm_100a kernels")
        if algorithm not in native.ALGORITHMS:
            raise ValueError(f"algorithm must be one of {sorted(native.ALGORITHMS)}")
        if master_precision not in native.MASTER_CODES:
            raise ValueError(f"master_precision must be one of {sorted(native.MASTER_CODES)}")
        self.native = native.load()
        self.algorithm = algorithm
        self.lion = algorithm == "lion"
        self.delay = False
        self.may_delay = False   # delayed updates will be switched on (the optimizer sets this before any update)
        self.precision = precision
        self.master_precision = master_precision
        self.stochastic = stochastic_rounding
        self.seed = seed
        self.overlap_writeback = overlap_writeback
        self.timing = timing
        self.max_ctas = max_ctas
        # Host-offload knobs of the reference, accepted for compatibility and unused here.
        self.numa_aware, self.num_threads, self.chunk_size = numa_aware, num_threads, chunk_size
        self.transfer_buffer_bytes = transfer_buffer_bytes

        self._lock = threading.RLock()
        self._streams: dict[torch.device, torch.cuda.Stream] = {}
        self._groups: dict[int, tuple[dict, native.Group]] = {}
        self._owed: dict[ParamSlot, None] = {}      # delayed: `out` holds an update not yet in the parameter
        self._fresh: dict[ParamSlot, None] = {}
        self._unwritten: dict[ParamSlot, None] = {}  # overlap_writeback=False: copy at finish_step
        self._copied: dict[torch.device, torch.cuda.Event] = {}  # delayed: last write-back copy per device
        self._first_ready: torch.cuda.Event | None = None
        self._last_ready: torch.cuda.Event | None = None
        self._update_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []
        self._num_updates = 0
        self._busy = 0.0
        self._closed = False

    # ------------------------------------------------------------------ streams

    def stream_for(self, device: torch.device) -> torch.cuda.Stream:
        s = self._streams.get(device)
        if s is None:
            with self._lock:
                s = self._streams.get(device)
                if s is None:
                    if self._closed:
                        raise RuntimeError("UpdateEngine is closed")
                    s = self._streams[device] = torch.cuda.Stream(device)
        return s

    # ------------------------------------------------------------------ state

    def initialize_many(self, slots: list[ParamSlot], pool=None) -> None:
        """Allocate master weights and moments on each parameter's device."""
        for slot in slots:
            p = slot.param
            if not p.is_cuda:
                raise ValueError("adambridge_b200 updates CUDA parameters only (the state lives in GPU memory)")
            if not p.is_contiguous():
                raise ValueError("non-contiguous parameters are not supported")
            if p.dtype not in _OUT_DTYPES:
                raise TypeError(f"parameters must be float32 or bfloat16, got {p.dtype}")
            with torch.cuda.device(p.device):
                # An FP32 parameter is its own FP32 master -- unless its update must land somewhere else first
                # (delayed updates, deferred write-back), which needs a master separate from the parameter.
                if (p.dtype == torch.float32 and self.master_precision == "fp32" and not self.may_delay
                        and self.overlap_writeback):
                    slot.master, slot.in_place = StateBuffer.viewing(p.data.view(-1)), True
                else:
                    slot.master = StateBuffer.converted(p.detach(), self.master_precision, "p", p.device)
                    slot.in_place = False
                slot.m = StateBuffer.allocate(self.precision, "m", slot.numel, p.device)
                slot.v = None if self.lion else StateBuffer.allocate(self.precision, "v", slot.numel, p.device)
            slot.seg = None

    def initialize(self, slot: ParamSlot, pool=None) -> None:
        self.initialize_many([slot])

    def convert_moments(self, slot: ParamSlot, precision: str) -> None:
        """Re-encode an initialized slot's moments in another precision (between steps)."""
        dev = slot.param.device
        with torch.cuda.device(dev):
            torch.cuda.current_stream(dev).wait_stream(self.stream_for(dev))
            slot.m = StateBuffer.converted(slot.m, precision, "m", dev)
            if slot.v is not None:
                slot.v = StateBuffer.converted(slot.v, precision, "v", dev)
        slot.seg = None

    def replace_moments(self, slot: ParamSlot, m: StateBuffer, v: StateBuffer | None) -> None:
        slot.m, slot.v = m, v
        slot.seg = None

    def free_buffers(self, slot: ParamSlot) -> None:
        self.wait()
        slot.master = slot.out = slot.m = slot.v = None
        slot.seg = None

    # ------------------------------------------------------------------ segments

    def _group_struct(self, group: dict) -> tuple[dict, native.Group]:
        """The kernel copy of a parameter group's hyperparameters, refreshed from the dict each update (an LR
        scheduler may have changed it; adambridge/engine.py:931-946)."""
        entry = self._groups.get(id(group))
        if entry is None or entry[0] is not group:
            entry = self._groups[id(group)] = (group, native.Group())
        g = entry[1]
        beta1, beta2 = group["betas"]
        g.lr = float(group["lr"])
        g.beta1 = float(beta1)
        g.beta2 = float(beta2)
        g.eps = float(group.get("eps", 0.0))
        g.weight_decay = float(group["weight_decay"])
        g.seed = self.seed & _MASK64
        g.stochastic = int(self.stochastic)
        return entry

    def _segment(self, slot: ParamSlot) -> native.Segment:
        seg = slot.seg
        if seg is None:
            seg = native.Segment()
            p_hi, p_lo = slot.master.operands
            seg.p = p_hi.data_ptr()
            seg.p_lo = p_lo.data_ptr() if p_lo is not None else None
            seg.p_dtype = slot.master.kernel_code
            m_buf, m_scale = slot.m.operands
            seg.m = m_buf.data_ptr()
            seg.m_scale = m_scale.data_ptr() if m_scale is not None else None
            if slot.v is not None:
                v_buf, v_scale = slot.v.operands
                seg.v = v_buf.data_ptr()
                seg.v_scale = v_scale.data_ptr() if v_scale is not None else None
            seg.n = slot.numel
            seg.index = slot.index
            seg.offset = 0
            seg.mv_dtype = slot.m.kernel_code
            seg.algorithm = native.ALGORITHMS[self.algorithm]
            slot.seg, slot.seg_group = seg, None
        return seg

    def _out_target(self, slot: ParamSlot) -> torch.Tensor | None:
        """Where the kernel writes the new weights: the parameter, the slot's ``out`` buffer, or nowhere (the
        master is the parameter)."""
        if slot.in_place:
            return None
        if self.delay or not self.overlap_writeback:
            if slot.out is None:
                slot.out = torch.empty_like(slot.param.data).view(-1)
            return slot.out
        return slot.param.data

    # ------------------------------------------------------------------ submission

    def submit(self, slot: ParamSlot, grad: torch.Tensor, g_scale: torch.Tensor | None = None) -> None:
        """Enqueue the update of ``slot`` with ``grad`` (called from autograd hooks or ``step``)."""
        self.submit_many([(slot, grad)], g_scale=g_scale)

    def submit_many(self, items: list[tuple[ParamSlot, torch.Tensor]], g_scale: torch.Tensor | None = None) -> None:
        """Enqueue updates for (slot, grad) pairs: one ``abx_multi_step`` call per device."""
        if not items:
            return
        t0 = time.perf_counter()
        by_device: dict[torch.device, list[tuple[ParamSlot, torch.Tensor]]] = {}
        for slot, grad in items:
            if grad.is_sparse:
                raise RuntimeError("adambridge_b200 does not support sparse gradients")
            by_device.setdefault(slot.param.device, []).append((slot, grad))
        for device, pairs in by_device.items():
            self._launch(device, pairs, g_scale)
        self._busy += time.perf_counter() - t0

    def _launch(self, device: torch.device, pairs: list, g_scale: torch.Tensor | None) -> None:
        fresh = [slot for slot, _ in pairs if not slot.initialized]
        if fresh:
            self.initialize_many(fresh)
        stream = self.stream_for(device)
        current = torch.cuda.current_stream(device)
        ready = torch.cuda.Event(enable_timing=self.timing)
        ready.record(current)
        if self._first_ready is None:
            self._first_ready = ready
        self._last_ready = ready
        stream.wait_event(ready)
        grads = []
        for slot, grad in pairs:
            if grad.dtype not in _GRAD_DTYPES:
                raise TypeError(f"gradients must be float32 or bfloat16, got {grad.dtype}")
            if grad.numel() != slot.numel:
                raise ValueError(f"gradient has {grad.numel()} elements, parameter {slot.index} has {slot.numel}")
            if grad.device != device:
                raise ValueError(f"gradient on {grad.device}, parameter on {device}")
            grads.append(grad if grad.is_contiguous() else grad.contiguous())
        with torch.cuda.device(device), torch.cuda.stream(stream):
            if self.delay:
                owed = [slot for slot, _ in pairs if slot in self._owed]
                if owed:
                    self._copy_out(owed)
                    ev = torch.cuda.Event()
                    ev.record(stream)
                    self._copied[device] = ev
                with self._lock:
                    for slot, _ in pairs:
                        self._owed.pop(slot, None)
                        self._fresh[slot] = None
            segs = []
            for (slot, _), grad in zip(pairs, grads):
                seg = self._segment(slot)
                slot.step += 1
                seg.step = slot.step
                seg.g = grad.data_ptr()
                seg.g_dtype = native.dtype_code_of(grad.dtype)
                out = self._out_target(slot)
                seg.out = out.data_ptr() if out is not None else None
                seg.out_dtype = native.DT_NONE if out is None else native.dtype_code_of(out.dtype)
                entry = self._group_struct(slot.group)
                if slot.seg_group is not entry[1]:
                    seg.group = ctypes.pointer(entry[1])
                    slot.seg_group = entry[1]
                segs.append(ctypes.pointer(seg))
                if not self.delay and not self.overlap_writeback and out is not None:
                    self._unwritten[slot] = None
            start = end = None
            if self.timing:
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record(stream)
            self.native.multi_step(stream, self.native.segment_array(segs), self.max_ctas, g_scale)
            if end is not None:
                end.record(stream)
                self._update_events.append((start, end))
        for grad in grads:
            grad.record_stream(stream)   # keep the gradient's memory alive until the kernel has read it
        if g_scale is not None:
            g_scale.record_stream(stream)
        self._num_updates += len(pairs)

    @staticmethod
    def _copy_out(slots: list[ParamSlot]) -> None:
        """Copy the slots' pending new weights into their parameters (on the current stream)."""
        torch._foreach_copy_([s.param.data.view(-1) for s in slots], [s.out for s in slots])

    # ------------------------------------------------------------------ synchronizing

    def wait(self) -> None:
        """Block until every enqueued update has finished on the GPU; raise if one of them gave up a pipeline
        wait (its parameters were left partly updated)."""
        for stream in list(self._streams.values()):
            stream.synchronize()
        if self._streams:
            self.native.check_status("UpdateEngine.wait")

    def _order_writebacks(self) -> None:
        """The caller's current streams wait for the updates (or, delayed, for the write-back copies)."""
        for device, stream in list(self._streams.items()):
            current = torch.cuda.current_stream(device)
            if self.delay:
                ev = self._copied.get(device)
                if ev is not None:
                    current.wait_event(ev)
            else:
                current.wait_stream(stream)

    def _write_back_slots(self, slots: list[ParamSlot]) -> None:
        """Copy ``slots``' pending updates to their parameters, after the updates that produced them."""
        by_device: dict[torch.device, list[ParamSlot]] = {}
        for slot in slots:
            by_device.setdefault(slot.param.device, []).append(slot)
        for device, members in by_device.items():
            stream = self.stream_for(device)
            with torch.cuda.device(device), torch.cuda.stream(stream):
                stream.wait_stream(torch.cuda.current_stream(device))
                self._copy_out(members)
                ev = torch.cuda.Event()
                ev.record(stream)
                self._copied[device] = ev
            torch.cuda.current_stream(device).wait_event(ev)

    def flush(self) -> None:
        """Apply every pending (delayed or deferred) update to the parameters; the caller's current stream then
        sees the weights an exact, undelayed optimizer would have produced.  Raises if an update that has
        finished gave up a pipeline wait."""
        if self._streams:
            self.native.check_status("flush")
        with self._lock:
            slots = list({**self._owed, **self._fresh, **self._unwritten})
            self._owed, self._fresh, self._unwritten = {}, {}, {}
        self._write_back_slots(slots)
        for device, stream in list(self._streams.items()):
            torch.cuda.current_stream(device).wait_stream(stream)

    def discard_pending(self) -> None:
        """Wait for enqueued updates and drop any not yet written to the parameters."""
        self.wait()
        with self._lock:
            self._owed, self._fresh, self._unwritten = {}, {}, {}

    def finish_step(self) -> StepStats:
        """Order this step's updates before the caller's next GPU work.

        Delayed mode: only the write-back copies are waited for; updates from earlier steps whose parameters got
        no gradient this step are written back now, so no parameter lags by more than one step.

        Raises if an update kernel that has finished by now gave up a pipeline wait (a status word in mapped
        host memory, read without synchronizing: a failure surfaces at the first step_sync after its kernel)."""
        if self._streams:
            self.native.check_status("step_sync")
        t0 = time.perf_counter()
        if self.delay:
            with self._lock:
                left, self._owed, self._fresh = list(self._owed), self._fresh, {}
            if left:
                self._write_back_slots(left)
        with self._lock:
            unwritten, self._unwritten = list(self._unwritten), {}
        if unwritten:
            self._write_back_slots(unwritten)
        self._order_writebacks()
        stats = StepStats(stall=time.perf_counter() - t0)
        first, last = self._first_ready, self._last_ready
        self._first_ready = self._last_ready = None
        stats.num_updates, self._num_updates = self._num_updates, 0
        stats.cpu_update, self._busy = self._busy, 0.0
        events, self._update_events = self._update_events, []
        if self.timing:
            if first is not None and last is not None and first is not last:
                last.synchronize()
                stats.gpu_backward = first.elapsed_time(last) / 1e3
            if events:
                events[-1][1].synchronize()
                stats.gpu_update = events[0][0].elapsed_time(events[-1][1]) / 1e3
        for device in self._streams:
            stats.per_device_cpu[str(device)] = stats.cpu_update
        return stats

    # ------------------------------------------------------------------ standalone kernel

    def run_kernel(self, master, grad, m, v, out, c: StepCoefficients, seed: int, pool=None, stream=None) -> None:
        """One standalone update with explicit coefficients (benchmarks, tests); adambridge/engine.py:1064-1099.
        ``master`` is a flat FP32 CUDA tensor or a master store; ``v=None`` runs Lion."""
        if isinstance(master, torch.Tensor):
            n, p_hi, p_lo, p_code = master.numel(), master, None, native.DT_F32
        else:
            n, (p_hi, p_lo), p_code = master.numel, master.operands, master.kernel_code
        if n == 0:
            return
        lion = v is None
        m_data, m_scale = m.operands
        v_data, v_scale = (None, None) if lion else v.operands
        seg = native.Segment(
            p=p_hi.data_ptr(), p_lo=p_lo.data_ptr() if p_lo is not None else None, p_dtype=p_code,
            g=grad.data_ptr(), m=m_data.data_ptr(), v=v_data.data_ptr() if v_data is not None else None,
            m_scale=m_scale.data_ptr() if m_scale is not None else None,
            v_scale=v_scale.data_ptr() if v_scale is not None else None,
            out=out.data_ptr() if out is not None else None, n=n, g_dtype=native.dtype_code_of(grad.dtype),
            mv_dtype=m.kernel_code,
            out_dtype=native.DT_NONE if out is None else native.dtype_code_of(out.dtype),
            algorithm=native.ALGORITHMS["lion" if lion else "adamw"])
        hp = self.native.make_hparams(c, seed, self.stochastic)
        with torch.cuda.device(grad.device):
            self.native.multi_apply(stream, self.native.segment_array([ctypes.pointer(seg)]), [hp], self.max_ctas)

    def step_seed(self, slot: ParamSlot) -> int:
        return mix_seed(self.seed, slot.index, slot.step) & 0xFFFFFFFF

    # ------------------------------------------------------------------ misc

    def set_parallelism(self, ctas: int) -> None:
        """Cap the CTAs of each update launch (0: every SM).  The analogue of the reference's thread count."""
        self.max_ctas = max(0, int(ctas))

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            self._closed = True
        try:
            self.wait()
        except Exception:  # noqa: BLE001 -- a dead context at interpreter exit
            pass
