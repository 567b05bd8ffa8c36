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

import contextlib

import torch

from . import native

__all__ = ["clip_coefficient"]


def clip_coefficient(grads: list[torch.Tensor], max_norm: float, stream=None, kernels=None):
    """(total_norm, coefficient, norms) of ``grads`` as device tensors, without a host synchronization.

    All gradients must be contiguous CUDA tensors (bf16 or fp32) of one device.  ``total_norm`` is a 0-dim
    tensor in the gradients' dtype (what clip_grad_norm_ returns); ``coefficient`` a 1-element float32 tensor
    usable as the update's ``grad_scale``; ``norms`` the per-gradient norms.

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
    grads = [g if g.is_contiguous() else g.contiguous() for g in grads]
    arr = k.tensor_array(grads)
    n = len(grads)
    with torch.cuda.device(dev):
        ws = torch.empty(k.clip_workspace_bytes(arr, n), dtype=torch.uint8, device=dev)
        sq = torch.empty(n, dtype=torch.float32, device=dev)
        k.grad_sq_norms(stream, arr, n, sq, ws)
        if len(dtypes) == 1:
            dtype = dtypes.pop()
            norms = torch.empty(n, dtype=torch.float32, device=dev)
            total_coef = torch.empty(2, dtype=torch.float32, device=dev)
            k.clip_coef_from_sq(stream, sq, dtype, max_norm, norms, total_coef)
            return total_coef[0].to(dtype), total_coef[1:2], norms
        ctx = torch.cuda.stream(stream) if isinstance(stream, torch.cuda.Stream) else contextlib.nullcontext()
        with ctx:
            norms = torch.sqrt(sq)
            bf16 = torch.tensor([g.dtype == torch.bfloat16 for g in grads], device=dev)
            norms = torch.where(bf16, norms.to(torch.bfloat16).float(), norms)
            total = torch.linalg.vector_norm(norms, 2.0)
            coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
        return total, coef.reshape(1), norms
