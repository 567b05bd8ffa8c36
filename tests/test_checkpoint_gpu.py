"""Checkpoints written by the reference load here and training continues bit for bit.

Each fixture in tests/golden/checkpoints/ was made by the reference's own AdamBridge / LionBridge on CPU
parameters (tests/golden/make_reference_states.py): three steps, its state_dict(), the gradients of a fourth
step and the weights and state_dict() after the reference took that step.  Here the checkpoint is loaded into
adambridge_b200 on the GPU (at the reference's SIMD level), the fourth step is taken with the same gradients,
and the weights, master weights and moments must equal the reference's bit for bit -- fp32, bf16 and FP8
moments, fp32 and fp24 masters, bf16 and fp32 weights, AdamW and Lion."""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

import adambridge_b200 as ab

pytestmark = pytest.mark.gpu

FIXTURES = sorted((Path(__file__).resolve().parent / "golden" / "checkpoints").glob("*.pt"))


def bits(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().cpu().contiguous()
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])


def assert_same(a, b, what):
    """Checkpoint entries (tensors or store dicts) equal bit for bit."""
    if isinstance(a, torch.Tensor):
        assert isinstance(b, torch.Tensor), what
        assert a.numel() == b.numel() and torch.equal(bits(a).reshape(-1), bits(b).reshape(-1)), what
        return
    assert isinstance(b, dict) and a.get("precision") == b.get("precision"), what
    for key, val in a.items():
        if isinstance(val, torch.Tensor):
            assert_same(val, b[key], f"{what}.{key}")
        else:
            assert val == b[key], f"{what}.{key}"


@pytest.fixture
def simd(kernels):
    yield kernels
    kernels.set_simd_level(None)


@pytest.mark.parametrize("path", FIXTURES, ids=[p.stem for p in FIXTURES])
def test_reference_checkpoint_resumes_bit_exact(path, simd):
    blob = torch.load(path, weights_only=False)
    simd.set_simd_level(blob["simd_level"])
    h = blob["hyper"]
    params = [torch.nn.Parameter(w.clone().cuda()) for w in blob["before"]["weights"]]
    kw = dict(lr=h["lr"], betas=h["betas"], weight_decay=h["weight_decay"], precision=blob["precision"],
              master_precision=blob["master_precision"], seed=h["seed"])
    opt = ab.LionBridge(params, **kw) if blob["algorithm"] == "lion" else ab.AdamBridge(params, eps=1e-8, **kw)
    opt.load_state_dict(blob["before"]["state_dict"])
    for p, g in zip(params, blob["grads"]):
        p.grad = g.clone().cuda()
    opt.step()
    torch.cuda.synchronize()
    for i, (p, w) in enumerate(zip(params, blob["after"]["weights"])):
        assert torch.equal(bits(p), bits(w)), f"weights of parameter {i}"
    ours, theirs = opt.state_dict(), blob["after"]["state_dict"]
    assert ours["adambridge"]["precision"] == theirs["adambridge"]["precision"]
    assert sorted(ours["state"]) == sorted(theirs["state"])
    for i, st in theirs["state"].items():
        mine = ours["state"][i]
        assert mine["step"] == st["step"]
        for key in ("master", "exp_avg", "exp_avg_sq"):
            if key in st:
                assert_same(mine[key], st[key], f"parameter {i} {key}")
    opt.close()


def test_torch_adamw_checkpoint_converts_on_the_device(simd):
    """A torch.optim.AdamW state_dict (fp32 moments as plain tensors) loads into every moment precision; the
    moments are the reference's conversions of those values (checked against the CPU checker)."""
    import numpy as np

    from oracle import convert as C
    torch.manual_seed(0)
    ref_params = [torch.nn.Parameter(torch.randn(300, 7, device="cuda")), torch.nn.Parameter(torch.randn(64, device="cuda"))]
    inner = torch.optim.AdamW(ref_params, lr=1e-3)
    for _ in range(2):
        for p in ref_params:
            p.grad = torch.randn_like(p)
        inner.step()
    sd = inner.state_dict()
    for prec in ("fp32", "bf16", "fp8"):
        params = [torch.nn.Parameter(p.detach().clone()) for p in ref_params]
        opt = ab.AdamBridge(params, lr=1e-3, precision=prec)
        opt.load_state_dict(sd)
        for i, slot in enumerate(opt.slots):
            for name, role, buf in (("exp_avg", "m", slot.m), ("exp_avg_sq", "v", slot.v)):
                want = C.encode(prec, sd["state"][i][name].detach().cpu().numpy().reshape(-1), role)
                for k, a in want.items():
                    got = buf.planes[k].detach().cpu()
                    got = got.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[got.element_size()]).numpy()
                    assert np.array_equal(got.view(a.dtype) if a.dtype != np.float32 else got.view(np.float32), a), \
                        (prec, name, k)
        opt.close()
