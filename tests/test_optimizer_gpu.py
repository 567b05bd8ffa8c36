"""The drop-in optimizer API on the GPU (models: the reference's tests/test_optimizer.py, test_cuda.py,
test_lion.py): torch AdamW / Lion agreement within the reference's tolerances, hooks == step bit for bit,
bit-exact agreement with the oracle through the public API, delayed updates == one-step-stale AdamW,
checkpoints, accumulation, clipping fused into the kernel."""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

import adambridge_b200 as ab
from oracle import oracle as O

pytestmark = pytest.mark.gpu


class TinyLM(torch.nn.Module):
    """Embedding, residual MLP blocks, tied output head (small params and one tied large one)."""

    def __init__(self, vocab=97, dim=64, layers=3):
        super().__init__()
        self.emb = torch.nn.Embedding(vocab, dim)
        self.blocks = torch.nn.ModuleList(
            torch.nn.Sequential(torch.nn.LayerNorm(dim), torch.nn.Linear(dim, 4 * dim), torch.nn.GELU(),
                                torch.nn.Linear(4 * dim, dim)) for _ in range(layers))
        self.norm = torch.nn.LayerNorm(dim)

    def forward(self, tokens):
        h = self.emb(tokens)
        for blk in self.blocks:
            h = h + blk(h)
        return self.norm(h) @ self.emb.weight.t()


def lm_loss(model, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    tokens = torch.randint(0, 97, (8, 33), device="cuda", generator=g)
    logits = model(tokens[:, :-1])
    return torch.nn.functional.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), tokens[:, 1:].reshape(-1))


def max_param_diff(a, b):
    return max((x.float() - y.float()).abs().max().item() for x, y in zip(a.parameters(), b.parameters()))


class RefLion(torch.optim.Optimizer):
    """Lion as published: decoupled weight decay, the sign of the interpolated moment."""

    def __init__(self, params, lr=1e-4, betas=(0.9, 0.99), weight_decay=0.0):
        super().__init__(params, dict(lr=lr, betas=betas, weight_decay=weight_decay))

    @torch.no_grad()
    def step(self):
        for group in self.param_groups:
            b1, b2 = group["betas"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                m = self.state[p].setdefault("m", torch.zeros_like(p))
                c = m * b1 + p.grad * (1 - b1)
                p.mul_(1 - group["lr"] * group["weight_decay"]).add_(c.sign(), alpha=-group["lr"])
                m.mul_(b2).add_(p.grad, alpha=1 - b2)


def test_matches_torch_adamw_with_groups_and_scheduler():
    torch.manual_seed(0)
    ref_model = TinyLM().cuda()
    model = copy.deepcopy(ref_model)

    def groups(m):
        named = list(m.named_parameters())
        return [{"params": [p for n, p in named if n.endswith("weight") and p.dim() == 2], "weight_decay": 0.1},
                {"params": [p for n, p in named if not (n.endswith("weight") and p.dim() == 2)],
                 "weight_decay": 0.0, "lr": 3e-3}]

    ref = torch.optim.AdamW(groups(ref_model), lr=1e-2, betas=(0.8, 0.99))
    opt = ab.AdamBridge(groups(model), lr=1e-2, betas=(0.8, 0.99))
    s_ref = torch.optim.lr_scheduler.StepLR(ref, step_size=3, gamma=0.5)
    s_opt = torch.optim.lr_scheduler.StepLR(opt, step_size=3, gamma=0.5)
    for step in range(10):
        for m, o, s in ((ref_model, ref, s_ref), (model, opt, s_opt)):
            o.zero_grad()
            lm_loss(m, step).backward()
            o.step()
            s.step()
    assert max_param_diff(ref_model, model) < 1e-6
    opt.close()


@pytest.mark.parametrize("overlap", [True, False])
def test_hooks_match_torch_adamw(overlap):
    torch.manual_seed(0)
    ref_model = TinyLM().cuda()
    model = copy.deepcopy(ref_model)
    ref = torch.optim.AdamW(ref_model.parameters(), lr=3e-3)
    opt = ab.AdamBridge(model.parameters(), lr=3e-3, overlap_writeback=overlap,
                        small_param_threshold=1000).attach_hooks(model)
    for step in range(8):
        ref.zero_grad()
        lm_loss(ref_model, step).backward()
        ref.step()
        opt.zero_grad()
        lm_loss(model, step).backward()
        assert all(p.grad is None for p in model.parameters() if p.numel() >= opt.small_param_threshold)
        stats = opt.step_sync()
        assert all(p.grad is None for p in model.parameters())
        assert stats.num_updates == len(list(model.parameters()))
    assert max_param_diff(ref_model, model) < 1e-5
    opt.close()


@pytest.mark.parametrize("precision", ["fp32", "bf16", "fp8"])
def test_hooks_and_step_bit_identical(precision):
    """Layer-wise hook updates and one batched step() give the same bits (independent of launch grouping)."""
    results = []
    for hooks in (False, True):
        torch.manual_seed(0)
        model = TinyLM().cuda().to(torch.bfloat16)
        opt = ab.AdamBridge(model.parameters(), lr=3e-3, precision=precision, small_param_threshold=1000)
        if hooks:
            opt.attach_hooks(model)
        for step in range(5):
            lm_loss(model, step).backward()
            opt.step_sync() if hooks else opt.step()
            opt.zero_grad()
        results.append([p.detach().clone() for p in model.parameters()] + [m.clone() for m in opt.master_params()])
        opt.close()
    assert all(torch.equal(a, b) for a, b in zip(*results))


@pytest.mark.parametrize("algo,precision,master", [("adamw", "bf16", "fp32"), ("adamw", "fp8", "fp24"),
                                                    ("lion", "bf16", "fp32"), ("lion", "fp8", "fp24")])
def test_public_api_bit_exact_with_oracle(algo, precision, master):
    """AdamBridge / LionBridge through the public API == the oracle (the reference's arithmetic) fed the same
    gradients, every buffer bit for bit: weights, master, moments (codes and scales)."""
    torch.manual_seed(1)
    model = TinyLM().cuda().to(torch.bfloat16)
    params = list(model.parameters())
    cls = ab.LionBridge if algo == "lion" else ab.AdamBridge
    kw = dict(lr=1e-3, weight_decay=0.05, betas=(0.9, 0.99)) if algo == "lion" else dict(lr=3e-3, weight_decay=0.02)
    opt = cls(params, precision=precision, master_precision=master, seed=17, **kw)
    orc = O.load_oracle()
    lion = algo == "lion"
    mv = {"fp32": O.DT_F32, "bf16": O.DT_BF16, "fp8": O.DT_FP8}[precision]
    pt = O.DT_F24 if master == "fp24" else O.DT_F32
    host = []
    for i, p in enumerate(params):
        n = p.numel()
        hs = O.HostSegment.random(n, O.DT_BF16, mv, O.DT_BF16, pt, O.LION if lion else O.ADAMW, index=i)
        w = p.detach().float().cpu().numpy().reshape(-1)
        if pt == O.DT_F24:
            hs.buffers["p"], hs.buffers["p_lo"] = O.bf16_bits(w), np.zeros(n, np.uint8)
        else:
            hs.buffers["p"] = w.copy()
        host.append(hs)
    group = O.Group(lr=kw["lr"], beta1=kw["betas"][0] if lion else 0.9, beta2=kw["betas"][1] if lion else 0.999,
                    eps=0.0 if lion else 1e-8, weight_decay=kw["weight_decay"], seed=17, stochastic=1)
    for step in range(1, 5):
        opt.zero_grad()
        lm_loss(model, step).backward()
        for hs, p in zip(host, params):
            hs.buffers["g"][:] = p.grad.detach().reshape(-1).view(torch.int16).cpu().numpy().view(np.uint16)
            hs.step = step
        opt.step()
        assert orc.multi_step([hs.ctype(group) for hs in host], O.SIMD_AVX512) == 0
    torch.cuda.synchronize()
    for hs, p, slot in zip(host, params, opt.slots):
        got = hs.clone()
        got.buffers["out"][:] = p.detach().reshape(-1).view(torch.int16).cpu().numpy().view(np.uint16)
        if pt == O.DT_F24:
            got.buffers["p"][:] = slot.master.planes["hi"].view(torch.int16).cpu().numpy().view(np.uint16)
            got.buffers["p_lo"][:] = slot.master.planes["lo"].cpu().numpy()
        else:
            got.buffers["p"][:] = slot.master.planes["data"].cpu().numpy()
        for name, store in (("m", slot.m), ("v", slot.v)):
            if store is None:
                continue
            if mv == O.DT_FP8:
                got.buffers[name][:] = store.planes["q"].view(torch.uint8).cpu().numpy()
                got.buffers[f"{name}_scale"][:] = store.planes["scale"].cpu().numpy()
            elif mv == O.DT_BF16:
                got.buffers[name][:] = store.planes["data"].view(torch.int16).cpu().numpy().view(np.uint16)
            else:
                got.buffers[name][:] = store.planes["data"].cpu().numpy()
        assert got.mismatches(hs) == {}, (slot.index, got.mismatches(hs))
    opt.close()


def test_bf16_params_follow_the_fp32_master():
    torch.manual_seed(0)
    model = TinyLM().cuda().to(torch.bfloat16)
    opt = ab.AdamBridge(model.parameters(), lr=3e-3, precision="bf16").attach_hooks(model)
    losses = []
    for step in range(30):
        loss = lm_loss(model, step % 4)
        loss.backward()
        opt.step_sync()
        losses.append(loss.item())
    assert losses[-1] < losses[0] - 0.5
    for p, master in zip(model.parameters(), opt.master_params()):
        assert p.dtype == torch.bfloat16 and master.dtype == torch.float32
        assert torch.equal(p.reshape(-1), master.to(torch.bfloat16))
    rep = opt.memory_report()
    n = sum(p.numel() for p in model.parameters())
    assert rep["master"] == 4 * n and rep["moments"] == 4 * n
    opt.close()


def test_lion_matches_reference_lion():
    torch.manual_seed(0)
    ref_model = TinyLM().cuda()
    model = copy.deepcopy(ref_model)
    ref = RefLion(ref_model.parameters(), lr=1e-3, weight_decay=0.1)
    opt = ab.LionBridge(model.parameters(), lr=1e-3, weight_decay=0.1)
    for step in range(6):
        for m, o in ((ref_model, ref), (model, opt)):
            o.zero_grad()
            lm_loss(m, step).backward()
            o.step()
    assert max_param_diff(ref_model, model) < 1e-6
    with pytest.raises(TypeError):
        ab.LionBridge(model.parameters(), eps=1e-8)
    opt.close()


def _stale_reference(model, steps, make_opt, warmup):
    """Losses and final weights of AdamW whose updates reach the model one step late after ``warmup`` exact
    steps (forward k uses the weights after k-1 updates up to step warmup+1, after k-2 from then on)."""
    master = copy.deepcopy(model).float()
    ref = make_opt(master.parameters())
    snapshots = [[p.detach().clone() for p in master.parameters()]]
    losses = []
    for k in range(1, steps + 1):
        lag = k - 1 if k <= warmup + 1 else k - 2
        with torch.no_grad():
            for p, w in zip(model.parameters(), snapshots[lag]):
                p.copy_(w)
        model.zero_grad()
        loss = lm_loss(model, k)
        loss.backward()
        losses.append(loss.item())
        for p, q in zip(master.parameters(), model.parameters()):
            p.grad = q.grad.float()
        ref.step()
        snapshots.append([p.detach().clone() for p in master.parameters()])
    return losses, snapshots[-1]


@pytest.mark.parametrize("warmup", [0, 3])
def test_delayed_updates_match_one_step_stale_adamw(warmup):
    torch.manual_seed(0)
    model = TinyLM().cuda()
    want_losses, want = _stale_reference(copy.deepcopy(model), 10, lambda ps: torch.optim.AdamW(ps, lr=3e-3), warmup)
    opt = ab.AdamBridge(model.parameters(), lr=3e-3, delay_updates=True, delay_warmup_steps=warmup,
                        small_param_threshold=2000).attach_hooks(model)
    assert any(s.small for s in opt.slots) and any(not s.small for s in opt.slots)
    losses = []
    for k in range(1, 11):
        loss = lm_loss(model, k)
        loss.backward()
        opt.step_sync()
        losses.append(loss.item())
    opt.flush()
    assert max(abs(a - b) for a, b in zip(losses, want_losses)) < 1e-4
    assert max((p - w).abs().max().item() for p, w in zip(model.parameters(), want)) < 1e-5
    opt.close()


def test_resume_from_state_dict_is_exact():
    torch.manual_seed(0)
    model = TinyLM().cuda().to(torch.bfloat16)
    opt = ab.AdamBridge(model.parameters(), lr=3e-3, precision="fp8", master_precision="fp24")
    for step in range(3):
        lm_loss(model, step).backward()
        opt.step()
        opt.zero_grad()
    sd = copy.deepcopy(opt.state_dict())
    weights = copy.deepcopy(model.state_dict())
    assert sd["adambridge"] == {"precision": "fp8", "master_precision": "fp24", "format": 1, "algorithm": "adamw"}
    for step in range(3, 6):
        lm_loss(model, step).backward()
        opt.step()
        opt.zero_grad()
    after = [p.detach().clone() for p in model.parameters()]

    model2 = TinyLM().cuda().to(torch.bfloat16)
    model2.load_state_dict(weights)
    opt2 = ab.AdamBridge(model2.parameters(), lr=3e-3, precision="fp8", master_precision="fp24")
    opt2.load_state_dict(sd)
    for step in range(3, 6):
        lm_loss(model2, step).backward()
        opt2.step()
        opt2.zero_grad()
    assert all(torch.equal(a, b) for a, b in zip(after, model2.parameters()))
    opt.close()
    opt2.close()


def test_loads_torch_adamw_checkpoint():
    torch.manual_seed(0)
    ref_model = TinyLM().cuda()
    ref = torch.optim.AdamW(ref_model.parameters(), lr=3e-3)
    for step in range(3):
        ref.zero_grad()
        lm_loss(ref_model, step).backward()
        ref.step()
    model = copy.deepcopy(ref_model)
    opt = ab.AdamBridge(model.parameters(), lr=3e-3)
    opt.load_state_dict(ref.state_dict())
    for step in range(3, 6):
        for m, o in ((ref_model, ref), (model, opt)):
            o.zero_grad()
            lm_loss(m, step).backward()
            o.step()
    assert max_param_diff(ref_model, model) < 1e-5
    opt.close()


def test_gradient_accumulation_with_no_sync():
    torch.manual_seed(0)
    ref_model = TinyLM().cuda()
    model = copy.deepcopy(ref_model)
    ref = torch.optim.AdamW(ref_model.parameters(), lr=3e-3)
    opt = ab.AdamBridge(model.parameters(), lr=3e-3).attach_hooks(model)
    for step in range(3):
        ref.zero_grad()
        for micro in range(3):
            (lm_loss(ref_model, 10 * step + micro) / 3).backward()
        ref.step()
        for micro in range(3):
            if micro < 2:
                with opt.no_sync():
                    (lm_loss(model, 10 * step + micro) / 3).backward()
            else:
                (lm_loss(model, 10 * step + micro) / 3).backward()
        opt.step_sync()
    assert max_param_diff(ref_model, model) < 1e-5
    opt.close()


def test_second_gradient_before_step_sync_raises():
    model = TinyLM().cuda()
    opt = ab.AdamBridge(model.parameters(), lr=1e-3, small_param_threshold=0).attach_hooks(model)
    lm_loss(model, 0).backward()
    with pytest.raises(RuntimeError, match="second gradient"):
        lm_loss(model, 1).backward()
    opt.close()


def test_clip_factor_fused_equals_torch_clip():
    """clip_grad_norm_ on bf16 gradients then step(), vs step(grad_scale=coefficient): identical bits.
    The coefficient is computed exactly as torch does (in the gradients' dtype)."""
    results = []
    for fused in (False, True):
        torch.manual_seed(0)
        model = TinyLM().cuda().to(torch.bfloat16)
        opt = ab.AdamBridge(model.parameters(), lr=3e-3, precision="bf16")
        for step in range(4):
            lm_loss(model, step).backward()
            if fused:
                grads = [p.grad for p in model.parameters()]
                norms = torch._foreach_norm(grads, 2.0)
                total = torch.linalg.vector_norm(torch.stack(norms), 2.0)
                coef = torch.clamp(0.1 / (total + 1e-6), max=1.0)
                opt.step(grad_scale=coef.float().reshape(1))
            else:
                torch.nn.utils.clip_grad_norm_(model.parameters(), 0.1)
                opt.step()
            opt.zero_grad()
        results.append([p.detach().clone() for p in model.parameters()])
        opt.close()
    assert all(torch.equal(a, b) for a, b in zip(*results))


def test_set_precision_between_steps():
    torch.manual_seed(0)
    model = TinyLM().cuda()
    opt = ab.AdamBridge(model.parameters(), lr=3e-3, precision="fp32")
    for step in range(3):
        lm_loss(model, step).backward()
        opt.step()
        opt.zero_grad()
    before = [s.m.to_fp32().clone() for s in opt.slots]
    opt.set_precision("bf16")
    assert opt.precision == "bf16" and all(s.m.precision == "bf16" for s in opt.slots)
    for b, s in zip(before, opt.slots):
        assert torch.equal(s.m.to_fp32(), b.to(torch.bfloat16).float())
    lm_loss(model, 3).backward()
    opt.step()
    assert opt.expected_bytes_per_param() == 8
    opt.close()


def test_weights_visible_to_next_forward_without_host_sync():
    torch.manual_seed(0)
    model = TinyLM().cuda()
    opt = ab.AdamBridge(model.parameters(), lr=0.5).attach_hooks(model)
    lm_loss(model, 0).backward()
    opt.step_sync()
    after = [p.clone() for p in model.parameters()]   # enqueued on the current stream
    torch.cuda.synchronize()
    for p, q in zip(model.parameters(), after):
        assert torch.equal(p, q)
    opt.close()
