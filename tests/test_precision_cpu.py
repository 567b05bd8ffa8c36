"""Checkpoint validation and state-format bookkeeping without a GPU (the reference's tests/test_hardening.py cases
for its stores: a checkpoint of another model, an unknown precision, a bad FP8 block or role is rejected with a
clear message before anything is loaded)."""

from __future__ import annotations

import pytest
import torch

from adambridge_b200.precision import (BLOCK, StateBuffer, bytes_per_param, check_master, check_moment,
                                       master_format, moment_format)


def test_precision_spellings():
    assert [moment_format(n) for n in ("fp32", "float32", "BF16", "bf16_moments", "bfloat16", "fp8", "fp8_moments")] \
        == ["fp32", "fp32", "bf16", "bf16", "bf16", "fp8", "fp8"]
    assert [master_format(n) for n in ("fp32", "float32", "fp24", "FLOAT24")] == ["fp32", "fp32", "fp24", "fp24"]
    for bad in ("int4", "fp16", None, 3):
        with pytest.raises(ValueError, match="precision"):
            moment_format(bad)
    with pytest.raises(ValueError, match="precision"):
        master_format("bf16")


def test_bytes_per_param():
    assert bytes_per_param("fp32") == 12 and bytes_per_param("bf16") == 8
    assert bytes_per_param("fp8") == pytest.approx(4 + 2 * (1 + 4 / 128))
    assert bytes_per_param("bf16", moments=1, master="fp24") == 5


def test_host_buffers_have_the_reference_planes():
    n = 300
    fp8 = StateBuffer.allocate("fp8", "v", n, "cpu")
    ck = fp8.checkpoint()
    assert ck["precision"] == "fp8" and ck["role"] == "v" and ck["block"] == BLOCK
    assert ck["q"].dtype == torch.float8_e5m2 and ck["q"].numel() == 3 * BLOCK
    assert ck["scale"].dtype == torch.float32 and torch.equal(ck["scale"], torch.ones(3))
    assert StateBuffer.allocate("fp8", "m", n, "cpu").planes["q"].dtype == torch.float8_e4m3fn
    f24 = StateBuffer.allocate("fp24", "p", n, "cpu").checkpoint()
    assert f24["hi"].dtype == torch.bfloat16 and f24["lo"].dtype == torch.uint8
    assert StateBuffer.allocate("bf16", "m", n, "cpu").checkpoint()["data"].dtype == torch.bfloat16
    assert fp8.nbytes == 3 * BLOCK + 3 * 4
    runs = fp8.plane_runs()
    assert [(u, p) for _, u, p in runs] == [(1, True), (BLOCK, True)]


def test_moment_checkpoints_are_validated():
    n = 300
    check_moment(torch.zeros(n), n, "exp_avg")                       # a torch.optim.AdamW tensor
    with pytest.raises(ValueError, match="elements"):
        check_moment(torch.zeros(n - 1), n, "exp_avg")
    with pytest.raises(ValueError, match="precision"):
        check_moment({"precision": "int4", "data": torch.zeros(n)}, n, "exp_avg")
    with pytest.raises(ValueError, match="elements"):
        check_moment({"precision": "fp32", "data": torch.zeros(n - 1)}, n, "exp_avg")
    with pytest.raises(ValueError, match="tensor"):
        check_moment({"precision": "bf16", "data": [0.0] * n}, n, "exp_avg")
    fp8 = StateBuffer.allocate("fp8", "m", n, "cpu").checkpoint()
    check_moment(fp8, n, "exp_avg")
    for block in (0, -128, 2.5, True, 1 << 21):
        with pytest.raises(ValueError, match="block"):
            check_moment({**fp8, "block": block}, n, "exp_avg")
    with pytest.raises(ValueError, match="role"):
        check_moment({**fp8, "role": "w"}, n, "exp_avg")
    with pytest.raises(ValueError, match="elements"):
        check_moment({**fp8, "scale": torch.ones(1)}, n, "exp_avg")
    with pytest.raises(ValueError, match="elements"):
        check_moment({**fp8, "q": torch.zeros(n, dtype=torch.uint8)}, n, "exp_avg")
    # another block size is loadable: its codes and scales are sized by that block
    check_moment({**fp8, "block": 64, "q": torch.zeros(320, dtype=torch.uint8), "scale": torch.ones(5)}, n, "m")


def test_master_checkpoints_are_validated():
    n = 50
    check_master(torch.zeros(n), n, "master")
    check_master({"precision": "fp32", "data": torch.zeros(n)}, n, "master")
    check_master(StateBuffer.allocate("fp24", "p", n, "cpu").checkpoint(), n, "master")
    with pytest.raises(ValueError, match="elements"):
        check_master(torch.zeros(1), n, "master")
    with pytest.raises(ValueError, match="precision"):
        check_master({"precision": "bf16", "data": torch.zeros(n)}, n, "master")
    bad = StateBuffer.allocate("fp24", "p", n, "cpu").checkpoint()
    with pytest.raises(ValueError, match="bfloat16"):
        check_master({**bad, "hi": torch.zeros(n, dtype=torch.int16)}, n, "master")
    with pytest.raises(ValueError, match="uint8"):
        check_master({**bad, "lo": torch.zeros(n, dtype=torch.int8)}, n, "master")


def test_checkpoint_buffers_view_the_checkpoint():
    """Parsing a checkpoint copies nothing: the buffer's planes are the checkpoint's tensors (a moment saved under
    another FP8 role keeps its role, for the conversion to decode it correctly)."""
    n = 300
    ck = StateBuffer.allocate("fp8", "m", n, "cpu").checkpoint()
    buf = StateBuffer.from_checkpoint(ck, n, "v", "exp_avg_sq")
    assert buf.role == "m" and buf.planes["q"].data_ptr() == ck["q"].data_ptr()
    t = torch.arange(n, dtype=torch.float32)
    view = StateBuffer.from_checkpoint(t, n, "v", "exp_avg_sq")
    assert view.fmt == "fp32" and view.planes["data"].data_ptr() == t.data_ptr()
    m = StateBuffer.master_from_checkpoint({"precision": "fp32", "data": t}, n, "master")
    assert m.fmt == "fp32" and m.planes["data"].data_ptr() == t.data_ptr()


def test_assign_needs_a_gpu_destination():
    host = StateBuffer.allocate("bf16", "m", 10, "cpu")
    with pytest.raises(ValueError, match="GPU"):
        host.assign(torch.zeros(10))
    with pytest.raises(ValueError, match="elements"):
        host.assign(torch.zeros(11))
