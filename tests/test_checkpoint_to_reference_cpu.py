"""Checkpoints written by adambridge_b200 load into the reference's own optimizer and continue bit for bit.

Each fixture in tests/golden/checkpoints_b200/ was written on a B200 by tests/golden/make_b200_checkpoints.py:
three steps of adambridge_b200's AdamBridge / LionBridge, its state_dict() (moved to the host), the gradients of
a fourth step and adambridge_b200's weights and state_dict() after it.  Here the reference's own AdamBridge /
LionBridge (its native backend, CPU parameters) loads the checkpoint, takes the fourth step, and must end where
adambridge_b200 ended.  The reference is imported from its checkout ($ABX_REFERENCE, else a ``reference``
directory beside this repository); without it the test is skipped."""

from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
FIXTURES = sorted((ROOT / "tests" / "golden" / "checkpoints_b200").glob("*.pt"))


def _reference():
    env = os.environ.get("ABX_REFERENCE")
    tree = Path(env) if env else ROOT.parent / "reference"
    if not (tree / "adambridge" / "optimizer.py").exists():
        pytest.skip("the reference checkout is not here")
    os.environ.setdefault("ADAMBRIDGE_CACHE_DIR", tempfile.mkdtemp(prefix="abx-ref-cache-"))
    if str(tree) not in sys.path:
        sys.path.insert(0, str(tree))
    import adambridge
    from adambridge import native
    if native.load() is None:
        pytest.skip("the reference's native backend did not build")
    return adambridge, native


def bits(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().cpu().contiguous()
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()]).reshape(-1)


def same(a, b, what):
    if isinstance(a, torch.Tensor):
        assert torch.equal(bits(a), bits(b)), what
        return
    assert a["precision"] == b["precision"], what
    for k, v in a.items():
        if isinstance(v, torch.Tensor):
            same(v, b[k], f"{what}.{k}")
        else:
            assert v == b[k], f"{what}.{k}"


@pytest.mark.skipif(not FIXTURES, reason="no adambridge_b200 checkpoints generated yet")
@pytest.mark.parametrize("path", FIXTURES, ids=[p.stem for p in FIXTURES])
def test_b200_checkpoint_resumes_in_the_reference(path):
    adambridge, native = _reference()
    blob = torch.load(path, weights_only=False)
    if native.load().simd_level != blob["simd_level"]:
        pytest.skip(f"the reference here runs {native.load().simd_level}, the checkpoint was made at "
                    f"{blob['simd_level']} rounding")
    h = dict(blob["hyper"])
    params = [torch.nn.Parameter(w.clone()) for w in blob["before"]["weights"]]
    kw = dict(precision=blob["precision"], master_precision=blob["master_precision"], **h)
    opt = adambridge.LionBridge(params, **kw) if blob["algorithm"] == "lion" else adambridge.AdamBridge(params, **kw)
    opt.load_state_dict(blob["before"]["state_dict"])
    for p, g in zip(params, blob["grads"]):
        p.grad = g.clone()
    opt.step()
    for i, (p, w) in enumerate(zip(params, blob["after"]["weights"])):
        assert torch.equal(bits(p), bits(w)), f"weights of parameter {i}"
    theirs, ours = opt.state_dict(), blob["after"]["state_dict"]
    for i, st in ours["state"].items():
        mine = theirs["state"][i]
        assert mine["step"] == st["step"]
        for key in ("master", "exp_avg", "exp_avg_sq"):
            if key in st:
                same(mine[key], st[key], f"parameter {i} {key}")
    opt.close()
