"""The optimizer API's argument and checkpoint checks without a GPU (the reference's tests/test_optimizer.py and
tests/test_hardening.py cases): they all reject before any device work, so they run on a CPU machine."""

from __future__ import annotations

import pytest
import torch

import adambridge_b200 as ab


def params():
    return [torch.nn.Parameter(torch.zeros(8, 4)), torch.nn.Parameter(torch.zeros(4))]


@pytest.mark.parametrize("kw, match", [
    (dict(lr=-1.0), "learning rate"),
    (dict(eps=-1.0), "epsilon"),
    (dict(betas=(1.0, 0.9)), "betas"),
    (dict(betas=(0.9, -0.1)), "betas"),
    (dict(weight_decay=-0.1), "weight_decay"),
    (dict(accumulation_steps=0), "accumulation_steps"),
    (dict(delay_warmup_steps=-1), "delay_warmup_steps"),
    (dict(chunk_size=100), "chunk_size"),
    (dict(transfer_buffer_mb=-1), "transfer_buffer_mb"),
    (dict(gpu_state_budget="most"), "gpu_state_budget"),
    (dict(max_ctas=-2), "max_ctas"),
    (dict(precision="int4"), "precision"),
    (dict(master_precision="bf16"), "precision"),
])
def test_bad_arguments_are_rejected(kw, match):
    with pytest.raises(ValueError, match=match):
        ab.AdamBridge(params(), **kw)


def test_lion_arguments():
    with pytest.raises(TypeError, match="eps"):
        ab.LionBridge(params(), eps=1e-8)
    with pytest.raises(ValueError, match="AdamW"):
        ab.LionBridge(params(), gpu_state_budget=1 << 20)
    opt = ab.LionBridge(params(), precision="fp8_moments", master_precision="float24")
    assert opt.precision == "fp8" and opt.master_precision == "fp24"
    assert opt.expected_bytes_per_param() == pytest.approx(3 + 1 + 4 / 128)
    assert ab.OptiComputeAdamW is ab.AdamBridge


def test_backend_rejects_a_cpu_fallback():
    with pytest.raises(ValueError, match="torch"):
        ab.AdamBridge(params(), backend="torch")


def _checkpoint(state: dict) -> dict:
    return {"state": state, "param_groups": [{"lr": 1e-3, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 0.01,
                                              "params": [0, 1]}]}


@pytest.mark.parametrize("index", [-1, 2, 99, "x", True])
def test_checkpoint_with_unknown_parameter_index(index):
    opt = ab.AdamBridge(params())
    entry = {"step": 1, "exp_avg": torch.zeros(4), "exp_avg_sq": torch.zeros(4)}
    with pytest.raises(ValueError, match="parameter"):
        opt.load_state_dict(_checkpoint({index: entry}))


def test_checkpoint_problems_are_found_before_anything_loads():
    opt = ab.AdamBridge(params())
    groups_before = [dict(g) for g in opt.param_groups]
    good = {"step": 3, "master": torch.zeros(4), "exp_avg": torch.zeros(4), "exp_avg_sq": torch.zeros(4)}
    for bad, match in ((dict(good, master=torch.zeros(1)), "elements"),
                       (dict(good, exp_avg=torch.zeros(3)), "elements"),
                       (dict(good, exp_avg_sq={"precision": "int4", "data": torch.zeros(4)}), "precision"),
                       ({"step": 3, "exp_avg": torch.zeros(4)}, "exp_avg_sq")):
        with pytest.raises(ValueError, match=match):
            opt.load_state_dict(_checkpoint({0: dict(good, master=torch.zeros(32), exp_avg=torch.zeros(32),
                                                     exp_avg_sq=torch.zeros(32)), 1: bad}))
        assert [dict(g) for g in opt.param_groups] == groups_before   # nothing changed


def test_string_indices_and_lion_ignoring_exp_avg_sq():
    """A checkpoint's indices may be strings (JSON round trips); a LionBridge reads only exp_avg -- checked on
    the CPU up to the point where loading would move the state to the parameters' GPU."""
    opt = ab.LionBridge(params())
    parsed = opt._parse_checkpoint(_checkpoint({"1": {"step": 2, "exp_avg": torch.zeros(4)}}))
    assert list(parsed) == [1] and parsed[1][0] == 2 and [r for r, _ in parsed[1][2]] == ["m"]


def test_micro_batch_counting_and_no_sync():
    opt = ab.AdamBridge(params(), accumulation_steps=3)
    passes = opt._passes
    assert passes.window == 3 and passes.finished == 0
    passes._pass_ended()
    passes._pass_ended()
    assert passes.finished == 2
    passes.reset()
    assert passes.finished == 0
    with opt.no_sync():
        with opt.no_sync():
            assert opt._no_sync_depth == 2
    assert opt._no_sync_depth == 0
