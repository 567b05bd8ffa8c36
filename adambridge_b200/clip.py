"""Gradient clipping on the device, fused into the update.

``torch.nn.utils.clip_grad_norm_`` reads every gradient for the norm and then reads and
writes every gradient again to scale it.  ``clip_coefficient`` computes the same total norm
and clipping coefficient on the device in one read of the gradients (libabx's deterministic
multi-tensor norm kernels) and leaves the gradients untouched; the optimizer then applies the
coefficient inside the update kernel while it reads each gradient, rounding a bf16 gradient
back to bf16 exactly as torch's in-place multiply would (``AdamBridge.clip_grad_norm_``).

The norms are accumulated in fp32 in a fixed order, then rounded to the gradients' dtype, as
torch's are; torch's own order of fp32 additions differs, so in rare cases a norm differs from
torch's by one unit in the last place of that dtype.
"""

from __future__ import annotations

import torch

from . import native

__all__ = ["clip_coefficient"]


def clip_coefficient(grads: list[torch.Tensor], max_norm: float, stream=None, kernels=None):
    """(total_norm, coefficient, norms) of ``grads`` as device tensors, without a host synchronization.

    All gradients must be CUDA tensors (bf16 or fp32) of one device.  ``total_norm`` is a 0-dim tensor in the
    gradients' dtype (what clip_grad_norm_ returns); ``coefficient`` a 1-element float32 tensor usable as the
    update's ``grad_scale``; ``norms`` the per-gradient norms.

    ``stream`` (a ``torch.cuda.Stream``, a raw ``cudaStream_t`` handle, or None for the current stream) is where
    all of the work runs: it first waits for the work already enqueued on the current stream (which produced
    the gradients), and every temporary -- contiguous copies of strided gradients, the kernels' workspace -- is
    allocated on it, so the caching allocator cannot hand that memory out again before the kernels that read
    it have run.  The results are ready on ``stream``; a caller that reads them on another stream orders
    that stream after ``stream`` first.

    Mixed bf16 and fp32 gradients are handled as torch handles them: each norm is rounded to its gradient's
    dtype and the total, taken over all norms, is in the promoted dtype (fp32); the sums of squares still come
    from the norm kernels, the few per-tensor values are combined with torch's own reduction."""
    if not grads:
        raise ValueError("no gradients")
    k = kernels or native.load()
    dev = grads[0].device
    if any(g.device != dev for g in grads):
        raise ValueError("clip_coefficient needs gradients of one device")
    dtypes = {g.dtype for g in grads}
    current = torch.cuda.current_stream(dev)
    if stream is None:
        run_on = current
    elif isinstance(stream, int):
        run_on = torch.cuda.ExternalStream(stream, device=dev)
    else:
        run_on = stream
    if run_on.cuda_stream != current.cuda_stream:
        run_on.wait_stream(current)
        for g in grads:
            g.record_stream(run_on)   # the caller may free a gradient while the kernels still read it
    n = len(grads)
    with torch.cuda.device(dev), torch.cuda.stream(run_on):
        grads = [g if g.is_contiguous() else g.contiguous() for g in grads]
        arr = k.tensor_array(grads)
        ws = torch.empty(k.clip_workspace_bytes(arr, n), dtype=torch.uint8, device=dev)
        sq = torch.empty(n, dtype=torch.float32, device=dev)
        k.grad_sq_norms(run_on, arr, n, sq, ws)
        if len(dtypes) == 1:
            dtype = dtypes.pop()
            norms = torch.empty(n, dtype=torch.float32, device=dev)
            total_coef = torch.empty(2, dtype=torch.float32, device=dev)
            k.clip_coef_from_sq(run_on, sq, dtype, max_norm, norms, total_coef)
            return total_coef[0].to(dtype), total_coef[1:2], norms
        norms = torch.sqrt(sq)
        bf16 = torch.tensor([g.dtype == torch.bfloat16 for g in grads], device=dev)
        norms = torch.where(bf16, norms.to(torch.bfloat16).float(), norms)
        total = torch.linalg.vector_norm(norms, 2.0)
        coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
        return total, coef.reshape(1), norms
