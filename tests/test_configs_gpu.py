"""The reference benchmark's configurations as full-size parity cases on the GPU.

Each runs the real shapes through the public API (AdamBridge, with its chunking, small-parameter
grouping, LR scheduler and fused clip) and checks every buffer of chosen tensors bit for bit against the
oracle -- the reference's arithmetic (adambridge/csrc/adambridge_kernels.c) -- fed the same gradients.
The update is elementwise per tensor (the stochastic-rounding stream is indexed by parameter index and
element), so a subset of tensors checked whole is a full check of those tensors at the full model's size.

* C1: one flat fp32 tensor of 16,777,216 params, fp32 moments, 10 steps (the reference's CPU case).
* C2: Qwen2.5-0.5B shapes (494,032,768 params, tied embedding), bf16 moments, per-tensor gradient scales
  log-uniform in [1e-4, 1e-2], 50 steps of cosine LR from 2e-5 read from ``param_groups`` every step.
* C3: Llama-1.5B shapes (1,364,297,728 params), fp8 moments, 1% of gradient entries x100, clip_grad_norm_ 1.0
  fused into the step.
* C4: Llama-7B shapes (6,738,415,616 params), ZeroLionBridge (world 1) with a bf16 moment, lr 1e-5,
  betas (0.9, 0.99), weight decay 0.1: the sharded optimizer's flat, round-major state at the full size.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import adambridge_b200 as ab
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _decoder_shapes(hidden, layers, mlp, vocab, kv, tied, qkv_bias):
    """Parameter shapes in module order: embedding, per layer (q, k, v[, biases], o, gate, up, down, 2 norms),
    final norm[, lm_head]."""
    shapes = [(vocab, hidden)]
    for _ in range(layers):
        shapes += [(hidden, hidden)] + ([(hidden,)] if qkv_bias else [])
        shapes += [(kv, hidden)] + ([(kv,)] if qkv_bias else [])
        shapes += [(kv, hidden)] + ([(kv,)] if qkv_bias else [])
        shapes += [(hidden, hidden), (mlp, hidden), (mlp, hidden), (hidden, mlp), (hidden,), (hidden,)]
    shapes.append((hidden,))
    if not tied:
        shapes.append((vocab, hidden))
    return shapes


QWEN05B = _decoder_shapes(896, 24, 4864, 151936, 128, tied=True, qkv_bias=True)
LLAMA15B = _decoder_shapes(2048, 24, 5632, 32000, 2048, tied=False, qkv_bias=False)
LLAMA7B = _decoder_shapes(4096, 32, 11008, 32000, 4096, tied=False, qkv_bias=False)


def test_config_shapes_have_the_published_sizes():
    assert sum(math.prod(s) for s in QWEN05B) == 494_032_768
    assert sum(math.prod(s) for s in LLAMA15B) == 1_364_297_728
    assert sum(math.prod(s) for s in LLAMA7B) == 6_738_415_616


def _bf16_params(shapes, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    out = []
    for s in shapes:
        p = torch.empty(s, dtype=torch.bfloat16, device="cuda")
        p.normal_(0.0, 0.02, generator=gen)
        out.append(torch.nn.Parameter(p))
    return out


def _host_segment(p: torch.Tensor, index: int, mv: int, pt: int = O.DT_F32) -> O.HostSegment:
    """The oracle's copy of a fresh parameter: master = the parameter's exact upcast, zero moments."""
    n = p.numel()
    fp32_param = p.dtype == torch.float32
    hs = O.HostSegment.random(n, O.DT_F32 if fp32_param else O.DT_BF16, mv, O.DT_NONE if fp32_param else O.DT_BF16,
                              pt, O.ADAMW, index=index)
    hs.buffers["p"] = p.detach().float().cpu().numpy().reshape(-1).copy()
    return hs


def _set_grad(hs: O.HostSegment, g: torch.Tensor, step: int) -> None:
    flat = g.detach().reshape(-1)
    if flat.dtype == torch.bfloat16:
        hs.buffers["g"][:] = flat.view(torch.int16).cpu().numpy().view(np.uint16)
    else:
        hs.buffers["g"][:] = flat.cpu().numpy()
    hs.step = step


def _assert_slot_matches(hs: O.HostSegment, p: torch.Tensor, slot, mv: int) -> None:
    got = hs.clone()
    if "out" in got.buffers:
        got.buffers["out"][:] = p.detach().reshape(-1).view(torch.int16).cpu().numpy().view(np.uint16)
    got.buffers["p"][:] = (p.detach().reshape(-1) if slot.in_place else slot.master.planes["data"]).cpu().numpy()
    for name, store in (("m", slot.m), ("v", slot.v)):
        if mv == O.DT_FP8:
            got.buffers[name][:] = store.planes["q"].view(torch.uint8).cpu().numpy()
            got.buffers[f"{name}_scale"][:] = store.planes["scale"].cpu().numpy()
        elif mv == O.DT_BF16:
            got.buffers[name][:] = store.planes["data"].view(torch.int16).cpu().numpy().view(np.uint16)
        else:
            got.buffers[name][:] = store.planes["data"].cpu().numpy()
    assert got.mismatches(hs) == {}, (slot.index, got.mismatches(hs))


def _group(lr, wd, seed=0, betas=(0.9, 0.999), eps=1e-8):
    return O.Group(lr=lr, beta1=betas[0], beta2=betas[1], eps=eps, weight_decay=wd, seed=seed, stochastic=1)


def test_c1_flat_fp32_tensor_ten_steps():
    gen = torch.Generator().manual_seed(0)
    n = 16_777_216
    p = torch.nn.Parameter((torch.randn(n, generator=gen) * 0.02).cuda())
    opt = ab.AdamBridge([p], lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, precision="fp32")
    hs = _host_segment(p, 0, O.DT_F32)
    group = _group(1e-4, 0.01)
    orc = O.load_oracle()
    for step in range(1, 11):
        g = torch.randn(n, generator=gen) * 1e-3
        p.grad = g.cuda()
        _set_grad(hs, g, step)
        opt.step()
        assert orc.multi_step([hs.ctype(group)], O.SIMD_AVX512) == 0
    torch.cuda.synchronize()
    _assert_slot_matches(hs, p, opt.slots[0], O.DT_F32)
    opt.close()


def test_c2_qwen05b_bf16_moments_cosine_lr_50_steps():
    params = _bf16_params(QWEN05B, seed=5)
    opt = ab.AdamBridge(params, lr=2e-5, precision="bf16")
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=50)
    rng = np.random.default_rng(11)
    sigma = 10.0 ** rng.uniform(-4, -2, len(params))
    # checked whole: layer-0 q weight and bias, a k projection, the last down projection, the final norm
    per_layer = 12
    checked = [1, 2, 1 + 11 * per_layer + 2, 1 + 23 * per_layer + 9, len(params) - 1]
    host = {i: _host_segment(params[i], i, O.DT_BF16) for i in checked}
    orc = O.load_oracle()
    gen = torch.Generator(device="cuda").manual_seed(12)
    for step in range(1, 51):
        for i, p in enumerate(params):
            g = torch.empty(p.shape, dtype=torch.float32, device="cuda")
            g.normal_(0.0, float(sigma[i]), generator=gen)
            p.grad = g.to(torch.bfloat16)
        lr = opt.param_groups[0]["lr"]
        group = _group(lr, 0.01)
        for i, hs in host.items():
            _set_grad(hs, params[i].grad, step)
        opt.step()
        assert orc.multi_step([hs.ctype(group) for hs in host.values()], O.SIMD_AVX512) == 0
        opt.zero_grad()
        sched.step()
    torch.cuda.synchronize()
    for i, hs in host.items():
        _assert_slot_matches(hs, params[i], opt.slots[i], O.DT_BF16)
    opt.close()


def test_c3_llama15b_fp8_moments_with_fused_clip():
    params = _bf16_params(LLAMA15B, seed=6)
    opt = ab.AdamBridge(params, lr=1e-4, precision="fp8")
    # checked whole: layer-0 q, the last down projection, a norm, the final norm, the (chunked) lm_head
    per_layer = 9
    checked = [1, 1 + 23 * per_layer + 6, 1 + 5 * per_layer + 8, len(params) - 2, len(params) - 1]
    host = {i: _host_segment(params[i], i, O.DT_FP8) for i in checked}
    group = _group(1e-4, 0.01)
    orc = O.load_oracle()
    gen = torch.Generator(device="cuda").manual_seed(13)
    bf16_ulp = 2.0 ** -7
    for step in range(1, 3):
        for p in params:
            g = torch.empty(p.shape, dtype=torch.float32, device="cuda")
            g.normal_(0.0, 1e-3, generator=gen)
            hot = torch.rand(p.shape, device="cuda", generator=gen) < 0.01
            p.grad = torch.where(hot, g * 100.0, g).to(torch.bfloat16)
        grads = [p.grad for p in params]
        want_total = torch.nn.utils.get_total_norm(grads, 2.0)
        want_coef = torch.clamp(1.0 / (want_total + 1e-6), max=1.0)
        total = opt.clip_grad_norm_(1.0)
        coef = opt._clip_coef
        assert total.dtype == torch.bfloat16
        # fp32 sums in another order: the bf16 total and coefficient agree to one bf16 unit at most
        assert abs(total.float().item() - want_total.float().item()) <= bf16_ulp * want_total.float().item()
        assert abs(coef.item() - want_coef.float().item()) <= bf16_ulp * want_coef.float().item()
        assert coef.item() < 1.0
        for i, hs in host.items():   # the oracle gets the gradients as torch's in-place clip leaves them
            _set_grad(hs, params[i].grad * coef.to(torch.bfloat16), step)
        opt.step()
        assert orc.multi_step([hs.ctype(group) for hs in host.values()], O.SIMD_AVX512) == 0
        opt.zero_grad()
    torch.cuda.synchronize()
    for i, hs in host.items():
        _assert_slot_matches(hs, params[i], opt.slots[i], O.DT_FP8)
    opt.close()


def _shard_slice(opt, index: int, buf: torch.Tensor) -> torch.Tensor:
    """Parameter ``index``'s elements gathered, in order, from a world-1 ZeRO shard buffer (round-major pieces)."""
    parts = sorted((pc.t_lo, buf[pc.local_lo:pc.local_lo + pc.n]) for rnd in opt._pieces for pc in rnd
                   if pc.index == index)
    return torch.cat([t for _, t in parts])


def test_c4_llama7b_zero_lion_bf16_moment():
    from adambridge_b200.zero import ZeroLionBridge
    params = _bf16_params(LLAMA7B, seed=7)
    opt = ZeroLionBridge(params, lr=1e-5, betas=(0.9, 0.99), weight_decay=0.1, precision="bf16", rounds=4)
    # checked whole: the embedding and lm_head (131M elements each, cut across rounds), layer-0 q, the last down
    # projection, a norm
    per_layer = 9
    checked = [0, 1, 1 + 31 * per_layer + 6, 1 + 7 * per_layer + 7, len(params) - 1]
    host = {}
    for i in checked:
        p = params[i]
        hs = O.HostSegment.random(p.numel(), O.DT_BF16, O.DT_BF16, O.DT_BF16, O.DT_F32, O.LION, index=i)
        hs.buffers["p"] = p.detach().float().cpu().numpy().reshape(-1).copy()
        host[i] = hs
    group = _group(1e-5, 0.1, betas=(0.9, 0.99), eps=0.0)
    orc = O.load_oracle()
    gen = torch.Generator(device="cuda").manual_seed(14)
    for step in range(1, 4):
        for p in params:
            p.grad = torch.empty(p.shape, dtype=torch.bfloat16, device="cuda").normal_(0.0, 1e-3, generator=gen)
        for i, hs in host.items():
            _set_grad(hs, params[i].grad, step)
        opt.step()
        assert orc.multi_step([hs.ctype(group) for hs in host.values()], O.SIMD_AVX512) == 0
        opt.zero_grad(set_to_none=True)
    torch.cuda.synchronize()
    for i, hs in host.items():
        got = hs.clone()
        got.buffers["out"][:] = params[i].detach().reshape(-1).view(torch.int16).cpu().numpy().view(np.uint16)
        got.buffers["p"][:] = _shard_slice(opt, i, opt.master.planes["data"]).cpu().numpy()
        got.buffers["m"][:] = _shard_slice(opt, i, opt.m.planes["data"]).view(torch.int16).cpu().numpy().view(np.uint16)
        assert got.mismatches(hs) == {}, (i, got.mismatches(hs))
