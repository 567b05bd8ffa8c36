"""Gradient norms and clipping on the GPU (libabx's norm kernels): per-tensor sums of squares against fp64,
the total norm and coefficient against torch.nn.utils.clip_grad_norm_ (torch/nn/utils/clip_grad.py), and the
fused clip -- ``opt.clip_grad_norm_(c); opt.step()`` -- against torch's in-place clip followed by ``step()``
(the reference's tests/test_cuda.py:273-287 clips in place before its step)."""

from __future__ import annotations

import pytest
import torch

import adambridge_b200 as ab
from adambridge_b200 import native
from adambridge_b200.clip import clip_coefficient
from adambridge_b200.zero import ZeroAdamBridge

pytestmark = pytest.mark.gpu

RAGGED = [0, 1, 7, 8, 9, 127, 16383, 16384, 16385, 100_000, (1 << 20) + 3]


def _grads(sizes, dtype, seed=0, scale=1e-2, offset=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for i, n in enumerate(sizes):
        base = (torch.randn(n + offset, generator=g) * scale * (1 + i % 5)).to("cuda", dtype)
        out.append(base[offset:])          # offset 1: not 16-byte aligned, the scalar-load path
    return out


def _sq_norms(grads):
    k = native.load()
    arr = k.tensor_array(grads)
    ws = torch.empty(k.clip_workspace_bytes(arr, len(grads)), dtype=torch.uint8, device="cuda")
    sq = torch.full((len(grads),), float("nan"), device="cuda")
    k.grad_sq_norms(None, arr, len(grads), sq, ws)
    torch.cuda.synchronize()
    return sq


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("offset", [0, 1])
def test_sum_of_squares_matches_fp64(dtype, offset):
    grads = _grads(RAGGED, dtype, offset=offset)
    sq = _sq_norms(grads).double().cpu()
    want = torch.stack([g.double().square().sum() for g in grads]).cpu()
    assert sq[0] == 0.0
    # fp32 accumulation: 64 sequential FMAs per thread, then fixed trees -- well inside 2e-5 relative
    torch.testing.assert_close(sq, want, rtol=2e-5, atol=0.0)


def test_more_tensors_than_one_launch_and_deterministic():
    sizes = [(i * 7919) % 40000 + 1 for i in range(150)]      # 150 tensors: three parameter blocks
    grads = _grads(sizes, torch.bfloat16, seed=3)
    a, b = _sq_norms(grads), _sq_norms(grads)
    assert torch.equal(a, b)
    want = torch.stack([g.double().square().sum() for g in grads])
    torch.testing.assert_close(a.double(), want, rtol=2e-5, atol=0.0)


def _torch_total_and_coef(grads, max_norm):
    """torch's clip_grad_norm_ arithmetic (torch/nn/utils/clip_grad.py: _get_total_norm, _clip_grads_with_norm_)."""
    total = torch.nn.utils.get_total_norm(grads, 2.0)
    coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
    return total, coef


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("max_norm", [0.1, 1e4])            # clipping, and a coefficient clamped at 1
def test_total_norm_and_coefficient_match_torch(dtype, max_norm):
    grads = _grads([4096, 300, 65536, 5, 100_000], dtype, seed=7)
    total, coef, norms = clip_coefficient(grads, max_norm)
    want_total, want_coef = _torch_total_and_coef(grads, max_norm)
    assert total.dtype == want_total.dtype == dtype
    if dtype == torch.bfloat16:
        # per-tensor norms rounded to bf16 absorb the different fp32 summation order
        assert torch.equal(total, want_total)
        assert coef.item() == want_coef.float().item()
        assert torch.equal(norms.to(dtype), torch.stack(torch._foreach_norm(grads, 2.0)))
    else:
        torch.testing.assert_close(total, want_total, rtol=1e-6, atol=0.0)
        torch.testing.assert_close(coef, want_coef.reshape(1), rtol=2e-6, atol=0.0)
    if max_norm > 1e3:
        assert coef.item() == 1.0


def test_non_finite_gradient_gives_torch_coefficient():
    grads = _grads([1000, 1000], torch.float32)
    grads[1][17] = float("inf")
    total, coef, _ = clip_coefficient(grads, 1.0)
    want_total, want_coef = _torch_total_and_coef(grads, 1.0)
    assert total.item() == want_total.item() == float("inf")
    assert coef.item() == want_coef.item() == 0.0


def test_mixed_dtypes_follow_torch():
    """bf16 and fp32 gradients together (a bf16 model whose norms stay fp32): each norm in its gradient's dtype,
    the total in fp32 over all of them, as torch's clip_grad_norm_ groups them."""
    grads = _grads([4096, 300, 65536], torch.bfloat16, seed=3) + _grads([896, 70_000], torch.float32, seed=4)
    total, coef, norms = clip_coefficient(grads, 0.05)
    want_total, want_coef = _torch_total_and_coef(grads, 0.05)
    assert total.dtype == want_total.dtype == torch.float32
    torch.testing.assert_close(total, want_total, rtol=1e-6, atol=0.0)
    torch.testing.assert_close(coef, want_coef.reshape(1), rtol=2e-6, atol=0.0)
    want_norms = [torch.linalg.vector_norm(g, 2.0).float() for g in grads]
    torch.testing.assert_close(norms, torch.stack(want_norms), rtol=1e-6, atol=0.0)
    assert all(norms[i].item() == norms[i].to(torch.bfloat16).float().item() for i in range(3))


class _MixedNet(torch.nn.Module):
    """bf16 linear layers with an fp32 norm weight between them."""

    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(128, 256).to(torch.bfloat16)
        self.norm = torch.nn.LayerNorm(256)
        self.b = torch.nn.Linear(256, 64).to(torch.bfloat16)

    def forward(self, x):
        return self.b(self.norm(self.a(x).float()).to(torch.bfloat16))


def test_fused_clip_with_mixed_dtypes_applies_its_coefficient():
    """opt.clip_grad_norm_ + step() on a mixed bf16/fp32 model == scaling the gradients in place by the same
    coefficient (torch's _foreach_mul_, as clip_grad_norm_ scales them) then step(), bit for bit."""
    results = []
    for fused in (True, False):
        torch.manual_seed(0)
        model = _MixedNet().cuda()
        opt = ab.AdamBridge(model.parameters(), lr=3e-3, precision="bf16", small_param_threshold=100)
        for step in range(3):
            x = torch.randn(32, 128, device="cuda", generator=torch.Generator(device="cuda").manual_seed(step))
            model(x.to(torch.bfloat16)).float().square().mean().backward()
            grads = [p.grad for p in model.parameters()]
            if fused:
                opt.clip_grad_norm_(0.02)
            else:
                _, coef, _ = clip_coefficient(grads, 0.02)
                for dtype in (torch.bfloat16, torch.float32):
                    group = [g for g in grads if g.dtype == dtype]
                    torch._foreach_mul_(group, coef[0])
            opt.step()
            opt.zero_grad()
        torch.cuda.synchronize()
        results.append([p.detach().clone() for p in model.parameters()])
        opt.close()
    assert all(torch.equal(a, b) for a, b in zip(*results))


class _Net(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(128, 512)
        self.b = torch.nn.Linear(512, 384)
        self.c = torch.nn.Linear(384, 64)

    def forward(self, x):
        return self.c(torch.nn.functional.gelu(self.b(torch.nn.functional.gelu(self.a(x)))))


def _loss(model, step):
    g = torch.Generator(device="cuda").manual_seed(step)
    x = torch.randn(64, 128, device="cuda", generator=g).to(next(model.parameters()).dtype)
    return model(x).float().square().mean()


@pytest.mark.parametrize("precision", ["fp32", "bf16", "fp8"])
def test_fused_clip_equals_torch_clip_then_step(precision):
    """opt.clip_grad_norm_(c) + step() (grads untouched, scaled in the kernel) == torch's in-place
    clip_grad_norm_ + step(), bit for bit, and both return the same norm."""
    results, norms = [], []
    for fused in (False, True):
        torch.manual_seed(0)
        model = _Net().cuda().to(torch.bfloat16)
        opt = ab.AdamBridge(model.parameters(), lr=3e-3, precision=precision, small_param_threshold=1000)
        got = []
        for step in range(4):
            _loss(model, step).backward()
            if fused:
                got.append(opt.clip_grad_norm_(0.05))
            else:
                got.append(torch.nn.utils.clip_grad_norm_(model.parameters(), 0.05))
            opt.step()
            opt.zero_grad()
        torch.cuda.synchronize()
        results.append([p.detach().clone() for p in model.parameters()])
        norms.append(torch.stack(got))
        opt.close()
    assert torch.equal(norms[0], norms[1])
    assert all(torch.equal(a, b) for a, b in zip(*results))


def test_clip_after_hook_update_raises():
    model = _Net().cuda()
    opt = ab.AdamBridge(model.parameters(), lr=1e-3, small_param_threshold=0).attach_hooks(model)
    _loss(model, 0).backward()
    with pytest.raises(RuntimeError, match="clip before any update"):
        opt.clip_grad_norm_(1.0)
    opt.step_sync()
    opt.close()


def test_zero_world1_clip_equals_adambridge_clip():
    """ZeroAdamBridge.clip_grad_norm_ (per-piece sums over the shard, combined per parameter) == AdamBridge's."""
    results, norms = [], []
    for zero in (False, True):
        torch.manual_seed(0)
        model = _Net().cuda().to(torch.bfloat16)
        if zero:
            opt = ZeroAdamBridge(model.parameters(), lr=3e-3, precision="bf16", rounds=3)
        else:
            opt = ab.AdamBridge(model.parameters(), lr=3e-3, precision="bf16", small_param_threshold=0)
        got = []
        for step in range(3):
            _loss(model, step).backward()
            got.append(opt.clip_grad_norm_(0.05))
            opt.step()
            opt.zero_grad()
        torch.cuda.synchronize()
        results.append([p.detach().clone() for p in model.parameters()])
        norms.append(torch.stack(got))
        if not zero:
            opt.close()
    assert torch.equal(norms[0], norms[1])
    assert all(torch.equal(a, b) for a, b in zip(*results))
