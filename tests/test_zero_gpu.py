"""ZeRO-1 on the GPU: ZeroAdamBridge / ZeroLionBridge equal the unsharded AdamBridge / LionBridge bit for bit
-- in one process (world 1, no collective) and across 2 GPUs over NCCL (reduce-scatter of gradients,
sharded update, all-gather of weights).  The 2-GPU test runs as child processes and is skipped with fewer
GPUs."""

from __future__ import annotations

import datetime
import os
import pickle
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import adambridge_b200 as ab
from adambridge_b200.zero import ZeroAdamBridge, ZeroLionBridge

pytestmark = pytest.mark.gpu

SHAPES = [(97, 64), (64,), (256, 64), (64, 256), (64,), (1000, 33), (5,), (4096, 3)]


def _params(device, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.nn.Parameter((torch.randn(s, generator=g) * 0.02).to(device, torch.bfloat16)) for s in SHAPES]


def _grads(step, device):
    g = torch.Generator().manual_seed(1000 + step)
    return [(torch.randn(s, generator=g) * 1e-3).to(device, torch.bfloat16) for s in SHAPES]


def _reference(algo, precision, steps, device):
    params = _params(device)
    cls = ab.LionBridge if algo == "lion" else ab.AdamBridge
    opt = cls(params, lr=1e-3, precision=precision, small_param_threshold=0, seed=3)
    for step in range(1, steps + 1):
        for p, g in zip(params, _grads(step, device)):
            p.grad = g
        opt.step()
    torch.cuda.synchronize()
    out = [p.detach().clone() for p in params], [m.clone() for m in opt.master_params()]
    opt.close()
    return out


@pytest.mark.parametrize("algo,precision", [("adamw", "bf16"), ("adamw", "fp8"), ("lion", "fp32")])
def test_zero_world1_equals_adambridge(algo, precision):
    want_w, want_m = _reference(algo, precision, 4, "cuda")
    params = _params("cuda")
    cls = ZeroLionBridge if algo == "lion" else ZeroAdamBridge
    opt = cls(params, lr=1e-3, precision=precision, seed=3, rounds=3)
    for step in range(1, 5):
        for p, g in zip(params, _grads(step, "cuda")):
            p.grad = g
        opt.step()
    torch.cuda.synchronize()
    for p, w in zip(params, want_w):
        assert torch.equal(p, w)
    assert opt.kernels.pipeline_status() == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, algo, precision, steps, out_dir, gather):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        params = _params(f"cuda:{rank}")
        cls = ZeroLionBridge if algo == "lion" else ZeroAdamBridge
        opt = cls(params, lr=1e-3, precision=precision, seed=3, rounds=2, gather=gather)
        assert (opt._peer_deltas is not None) == (gather == "p2p")
        for step in range(1, steps + 1):
            for p, g in zip(params, _grads(step, f"cuda:{rank}")):
                p.grad = g
            opt.step()
        torch.cuda.synchronize()
        with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
            pickle.dump([p.detach().cpu() for p in params], f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("gather", ["nccl", "p2p"])
@pytest.mark.parametrize("algo,precision", [("adamw", "bf16"), ("adamw", "fp8"), ("lion", "bf16")])
def test_zero_two_gpus_equals_unsharded(tmp_path, algo, precision, gather):
    """Reduce-scatter, sharded update and all-gather (NCCL's, or fused into the update as peer stores):
    every rank ends with the unsharded update's weights, bit for bit."""
    steps = 3
    want_w, _ = _reference(algo, precision, steps, "cuda:0")
    mp.start_processes(_rank, args=(2, _free_port(), algo, precision, steps, str(tmp_path), gather), nprocs=2,
                       start_method="spawn", join=True)
    for r in range(2):
        got = pickle.load(open(tmp_path / f"rank{r}.pkl", "rb"))
        for g, w in zip(got, want_w):
            assert torch.equal(g, w.cpu())
