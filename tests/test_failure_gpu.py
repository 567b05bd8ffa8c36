"""Failure detection of the update pipeline, without a GPU fault.

Every mbarrier wait of the update kernels is bounded.  These tests make one wait run out on purpose by the
library's failure-path switch (abx_test_pipeline_fault): the producer leaves one tile's ring stage untouched --
no bulk copy is issued into it and nothing arrives on its barrier -- and a short poll limit makes the consumers
waiting for it give up.  The kernel returns, the status word in mapped host memory is set, and the public API
raises instead of carrying on with a partly updated tensor.  No test here faults, traps or hangs the GPU: every
wait, the drained copies included, ends after the poll limit."""

from __future__ import annotations

import pytest
import torch

import adambridge_b200 as ab

pytestmark = pytest.mark.gpu

TILE = 2048          # elements of one update tile
SHORT_LIMIT = 1 << 12


@pytest.fixture
def fault(kernels):
    """The failure-path switch, always restored (no pending skip, the default poll limit, a clear word)."""
    kernels.pipeline_status()
    yield kernels
    kernels.test_pipeline_fault(-1, 0)
    kernels.pipeline_status()


def _step_expecting_failure(run, then):
    """``run()`` enqueues the faulty update; it or ``then()`` (after a synchronize) must raise."""
    try:
        run()
    except RuntimeError as exc:
        return exc
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="pipeline wait gave up") as info:
        then()
    return info.value


def test_adambridge_raises_and_leaves_the_skipped_tile(fault):
    n = 64 * TILE                                   # 64 whole, aligned tiles: one per CTA
    p = torch.nn.Parameter(torch.randn(n, device="cuda", dtype=torch.bfloat16))
    opt = ab.AdamBridge([p], lr=1e-2, precision="bf16")
    p.grad = torch.randn_like(p)
    opt.step()
    torch.cuda.synchronize()
    assert fault.pipeline_status() == 0             # a correct step sets nothing
    before = p.detach().clone()
    p.grad = torch.randn_like(p)
    fault.test_pipeline_fault(0, SHORT_LIMIT)
    exc = _step_expecting_failure(opt.step, opt.flush)
    assert "pipeline wait gave up" in str(exc)
    torch.cuda.synchronize()
    assert torch.equal(p.detach()[:TILE], before[:TILE])          # the skipped tile was not updated
    assert not torch.equal(p.detach()[TILE:], before[TILE:])      # the other CTAs' tiles were
    assert fault.pipeline_status() == 0             # raising cleared the word
    # the library keeps working once the switch is off
    fault.test_pipeline_fault(-1, 0)
    p.grad = torch.randn_like(p)
    opt.step()
    torch.cuda.synchronize()
    opt.flush()
    assert fault.pipeline_status() == 0


def test_status_word_is_readable_without_synchronizing(fault):
    n = 8 * TILE
    p = torch.nn.Parameter(torch.randn(n, device="cuda", dtype=torch.bfloat16))
    opt = ab.AdamBridge([p], lr=1e-2, precision="fp32", small_param_threshold=0)   # updated on its own
    p.grad = torch.randn_like(p)
    opt.step()
    torch.cuda.synchronize()
    assert not fault.status_pending()
    fault.test_pipeline_fault(3, SHORT_LIMIT)
    p.grad = torch.randn_like(p)
    opt._enqueue(opt._outstanding(small=None))     # the update alone, no step_sync check
    torch.cuda.synchronize()
    assert fault.status_pending()                   # read from host memory, no CUDA call
    bits = fault.pipeline_status()
    assert bits & 1                                 # a consumer's wait for the skipped tile gave up
    assert not fault.status_pending()
    opt.step_sync()                                 # cleared: nothing to report


def test_zero_step_raises_after_a_failed_update(fault):
    from adambridge_b200.zero import ZeroAdamBridge
    params = [torch.nn.Parameter(torch.randn(16 * TILE, device="cuda", dtype=torch.bfloat16)) for _ in range(2)]
    opt = ZeroAdamBridge(params, lr=1e-2, precision="bf16")
    opt.grad_shard.normal_()
    opt.step_shard()
    torch.cuda.synchronize()
    fault.test_pipeline_fault(0, SHORT_LIMIT)
    opt.step_shard()                                # the faulty update
    torch.cuda.synchronize()
    fault.test_pipeline_fault(-1, 0)
    with pytest.raises(RuntimeError, match="pipeline wait gave up"):
        opt.step_shard()                            # the next step reports it before updating anything
    assert fault.pipeline_status() == 0
    opt.step_shard()
    torch.cuda.synchronize()
    opt.flush()
