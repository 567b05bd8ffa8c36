"""abx_clip_coef_noalloc -- the clip entry point for callers that cannot allocate device memory (a C or FFI host
without a CUDA allocator of its own, or a loop that must not allocate per step), whose scratch is a static
device array in libabx -- against abx_clip_coef (caller workspace): the same sums of squares, norms, total norm
and coefficient, bit for bit, over two calls in a row; the second call reuses the static scratch the first one
wrote.  Collected last (file name), so it also runs after every other GPU test in the same process."""

from __future__ import annotations

import pytest
import torch

from adambridge_b200 import native

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 7, 127, 16383, 16384, 16385, 100_000, (1 << 20) + 3] + [(i * 7919) % 40000 + 1 for i in range(70)]


def _grads(dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(n, generator=g) * 1e-2).to("cuda", dtype) for n in SIZES]


def _outputs(n):
    return (torch.full((n,), float("nan"), device="cuda"), torch.full((n,), float("nan"), device="cuda"),
            torch.full((2,), float("nan"), device="cuda"))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_equals_workspace_entry_two_calls_in_a_row(dtype):
    k = native.load()
    for call, (seed, max_norm) in enumerate([(1, 0.5), (2, 1e4)]):   # second call: other data, other sizes' sums
        grads = _grads(dtype, seed)
        arr = k.tensor_array(grads)
        n = len(grads)
        ws = torch.empty(k.clip_workspace_bytes(arr, n), dtype=torch.uint8, device="cuda")
        want = _outputs(n)
        k.clip_coef(None, arr, n, max_norm, want[0], want[1], want[2], ws)
        got = _outputs(n)
        k.clip_coef_noalloc(None, arr, n, max_norm, got[0], got[1], got[2])
        torch.cuda.synchronize()
        for a, b in zip(got, want):
            assert torch.equal(a, b), call
        assert not torch.isnan(got[2]).any()

