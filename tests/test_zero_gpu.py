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


def _reference(algo, precision, steps, device, clip=None):
    params = _params(device)
    cls = ab.LionBridge if algo == "lion" else ab.AdamBridge
    opt = cls(params, lr=1e-3, precision=precision, small_param_threshold=0, seed=3)
    for step in range(1, steps + 1):
        for p, g in zip(params, _grads(step, device)):
            p.grad = g
        if clip is not None:
            opt.clip_grad_norm_(clip)
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


def _rank(rank, world, port, algo, precision, steps, out_dir, gather, clip=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        params = _params(f"cuda:{rank}")
        cls = ZeroLionBridge if algo == "lion" else ZeroAdamBridge
        opt = cls(params, lr=1e-3, precision=precision, seed=3, rounds=2, gather=gather)
        assert opt.gather == gather
        for step in range(1, steps + 1):
            for p, g in zip(params, _grads(step, f"cuda:{rank}")):
                p.grad = g
            if clip is not None:
                opt.clip_grad_norm_(clip)
            opt.step()
        torch.cuda.synchronize()
        with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
            pickle.dump([p.detach().cpu() for p in params], f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("gather", ["nccl", "p2p", "ce"])
@pytest.mark.parametrize("algo,precision", [("adamw", "bf16"), ("adamw", "fp8"), ("lion", "bf16")])
def test_zero_two_gpus_equals_unsharded(tmp_path, algo, precision, gather):
    """Reduce-scatter, sharded update and all-gather (NCCL's, fused into the update as peer stores, or
    copy-engine copies into the peers' buffers): every rank ends with the unsharded update's weights, bit for
    bit."""
    steps = 3
    want_w, _ = _reference(algo, precision, steps, "cuda:0")
    mp.start_processes(_rank, args=(2, _free_port(), algo, precision, steps, str(tmp_path), gather), nprocs=2,
                       start_method="spawn", join=True)
    for r in range(2):
        got = pickle.load(open(tmp_path / f"rank{r}.pkl", "rb"))
        for g, w in zip(got, want_w):
            assert torch.equal(g, w.cpu())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("gather", ["nccl", "p2p", "ce"])
def test_zero_two_gpus_clip_equals_unsharded(tmp_path, gather):
    """clip_grad_norm_ on the sharded, reduced gradients (per-parameter sums of squares all-reduced) then
    step() == the unsharded AdamBridge's clip_grad_norm_ + step(), on every rank."""
    steps = 3
    want_w, _ = _reference("adamw", "bf16", steps, "cuda:0", clip=2e-3)
    mp.start_processes(_rank, args=(2, _free_port(), "adamw", "bf16", steps, str(tmp_path), gather, 2e-3), nprocs=2,
                       start_method="spawn", join=True)
    for r in range(2):
        got = pickle.load(open(tmp_path / f"rank{r}.pkl", "rb"))
        for g, w in zip(got, want_w):
            assert torch.equal(g, w.cpu())


# ---------------------------------------------------------------------------------------------- checkpoints

def _bits(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().cpu().reshape(-1)
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])


def _assert_same_state(a: dict, b: dict) -> None:
    """Two checkpoints in the AdamBridge format hold the same bits for every parameter."""
    assert sorted(a["state"]) == sorted(b["state"])
    for i in a["state"]:
        sa, sb = a["state"][i], b["state"][i]
        assert int(sa["step"]) == int(sb["step"])
        for key in ("master", "exp_avg", "exp_avg_sq"):
            if key not in sa:
                assert key not in sb
                continue
            xa, xb = sa[key], sb[key]
            if isinstance(xa, torch.Tensor):
                assert torch.equal(_bits(xa), _bits(xb)), (i, key)
                continue
            assert {k for k in xa if isinstance(xa[k], torch.Tensor)} == {k for k in xb if isinstance(xb[k], torch.Tensor)}
            for k, v in xa.items():
                if isinstance(v, torch.Tensor):
                    assert torch.equal(_bits(v), _bits(xb[k])), (i, key, k)
                else:
                    assert v == xb[k], (i, key, k)


def _run_steps(opt, params, first, last, device):
    for step in range(first, last + 1):
        for p, g in zip(params, _grads(step, device)):
            p.grad = g
        opt.step()
    torch.cuda.synchronize()


@pytest.mark.parametrize("algo,precision,master", [("adamw", "bf16", "fp32"), ("adamw", "fp8", "fp24"),
                                                    ("adamw", "fp32", "fp32"), ("lion", "fp8", "fp32")])
def test_zero_checkpoint_is_the_adambridge_checkpoint(algo, precision, master):
    """A world-1 ZeRO optimizer (3 rounds, so tensors are cut into pieces) gathers exactly the checkpoint the
    unsharded AdamBridge writes; loading that checkpoint into a fresh ZeRO optimizer and continuing equals the
    AdamBridge continuing."""
    cls_a = ab.LionBridge if algo == "lion" else ab.AdamBridge
    cls_z = ZeroLionBridge if algo == "lion" else ZeroAdamBridge
    kw = dict(lr=1e-3, precision=precision, master_precision=master, seed=3)
    pa = _params("cuda")
    oa = cls_a(pa, small_param_threshold=0, **kw)
    _run_steps(oa, pa, 1, 3, "cuda")
    pz = _params("cuda")
    oz = cls_z(pz, rounds=3, **kw)
    _run_steps(oz, pz, 1, 3, "cuda")
    sd_a, sd_z = oa.state_dict(), oz.state_dict()
    _assert_same_state(sd_a, sd_z)
    assert sd_z["adambridge"] == sd_a["adambridge"]

    # resume: fresh ZeRO optimizer over the AdamBridge's current weights, loaded from its checkpoint
    pr = [torch.nn.Parameter(p.detach().clone()) for p in pa]
    orr = cls_z(pr, rounds=2, **kw)
    orr.load_state_dict(sd_a)
    _run_steps(oa, pa, 4, 5, "cuda")
    _run_steps(orr, pr, 4, 5, "cuda")
    for x, y in zip(pa, pr):
        assert torch.equal(x, y)
    _assert_same_state(oa.state_dict(), orr.state_dict())
    oa.close()


def test_zero_checkpoint_converts_precision_and_checks_shapes():
    pa = _params("cuda")
    oa = ab.AdamBridge(pa, lr=1e-3, precision="fp32", small_param_threshold=0, seed=3)
    _run_steps(oa, pa, 1, 2, "cuda")
    sd = oa.state_dict()
    oz = ZeroAdamBridge(_params("cuda"), lr=1e-3, precision="bf16", seed=3)
    oz.load_state_dict(sd)
    got = oz.state_dict()
    for i, st in sd["state"].items():
        want = st["exp_avg"]["data"].to(torch.bfloat16)
        assert torch.equal(got["state"][i]["exp_avg"]["data"], want.cpu())
    bad = {"state": {i: dict(st) for i, st in sd["state"].items()}, "param_groups": sd["param_groups"]}
    bad["state"][3]["exp_avg"] = {"precision": "fp32", "data": torch.zeros(7)}
    before = oz.state_dict()
    with pytest.raises(ValueError, match="7 elements"):
        oz.load_state_dict(bad)
    _assert_same_state(before, oz.state_dict())      # a rejected checkpoint changes nothing
    partial = {"state": {0: sd["state"][0]}, "param_groups": sd["param_groups"]}
    with pytest.raises(ValueError, match="every parameter"):
        oz.load_state_dict(partial)
    oa.close()


def _ckpt_rank(rank, world, port, out_dir, gather, saved_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        dev = f"cuda:{rank}"
        params = _params(dev)
        opt = ZeroAdamBridge(params, lr=1e-3, precision="fp8", seed=3, rounds=2, gather=gather)
        _run_steps(opt, params, 1, 3, dev)
        sd = opt.state_dict(rank0_only=True)
        if rank == 0:
            torch.save(sd, os.path.join(out_dir, "gathered.pt"))
        else:
            assert sd["state"] == {}
        # resume from the unsharded optimizer's checkpoint on fresh weights, and continue
        saved = torch.load(saved_path, map_location="cpu", weights_only=False)
        fresh = [torch.nn.Parameter(w.to(dev)) for w in saved["weights"]]
        opt2 = ZeroAdamBridge(fresh, lr=1e-3, precision="fp8", seed=3, rounds=3, gather=gather)
        opt2.load_state_dict(saved["optimizer"])
        _run_steps(opt2, fresh, 4, 5, dev)
        with open(os.path.join(out_dir, f"resumed{rank}.pkl"), "wb") as f:
            pickle.dump([p.detach().cpu() for p in fresh], f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("gather", ["nccl", "p2p", "ce"])
def test_zero_two_gpus_checkpoint_gather_and_resume(tmp_path, gather):
    """2 ranks: the gathered checkpoint equals the unsharded AdamBridge's; an unsharded checkpoint loaded into
    2 ranks and continued equals the unsharded optimizer continuing."""
    pa = _params("cuda:0")
    oa = ab.AdamBridge(pa, lr=1e-3, precision="fp8", small_param_threshold=0, seed=3)
    _run_steps(oa, pa, 1, 3, "cuda:0")
    sd_a = oa.state_dict()
    saved_path = str(tmp_path / "unsharded.pt")
    torch.save({"optimizer": sd_a, "weights": [p.detach().cpu() for p in pa]}, saved_path)
    mp.start_processes(_ckpt_rank, args=(2, _free_port(), str(tmp_path), gather, saved_path), nprocs=2,
                       start_method="spawn", join=True)
    _assert_same_state(sd_a, torch.load(tmp_path / "gathered.pt", weights_only=False))
    _run_steps(oa, pa, 4, 5, "cuda:0")
    for r in range(2):
        got = pickle.load(open(tmp_path / f"resumed{r}.pkl", "rb"))
        for g, w in zip(got, pa):
            assert torch.equal(g, w.detach().cpu())
    oa.close()


# ---------------------------------------------------------------------------------- gradients reduced in backward

class _Mlp(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.layers = torch.nn.ModuleList(torch.nn.Linear(96, 96) for _ in range(4))
        self.head = torch.nn.Linear(96, 7)

    def forward(self, x):
        for layer in self.layers:
            x = torch.nn.functional.gelu(layer(x))
        return self.head(x)


def _mlp_pair(device):
    torch.manual_seed(0)
    a = _Mlp().to(device, torch.bfloat16)
    b = _Mlp().to(device, torch.bfloat16)
    b.load_state_dict(a.state_dict())
    return a, b


def _mlp_loss(model, step, rank, device):
    g = torch.Generator(device=device).manual_seed(100 * step + rank)
    x = torch.randn(32, 96, device=device, generator=g).to(torch.bfloat16)
    return model(x).float().square().mean()


def _hooks_vs_step(rank, world, device, gather, clip, steps=3):
    """The same model trained by a hooked and by a step-mode ZeRO optimizer: identical weights."""
    ma, mb = _mlp_pair(device)
    kw = dict(lr=2e-3, precision="bf16", seed=3, rounds=3)
    if gather is not None:
        kw["gather"] = gather
    # with clipping, the hooks only reduce-scatter (the clip needs every gradient before any update); without,
    # each round is also updated during backward
    oa = ZeroAdamBridge(list(ma.parameters()), **kw).attach_hooks(ma, update_in_backward=clip is None)
    ob = ZeroAdamBridge(list(mb.parameters()), **kw)
    for step in range(1, steps + 1):
        for model, opt in ((ma, oa), (mb, ob)):
            _mlp_loss(model, step, rank, device).backward()
            if clip is not None:
                opt.clip_grad_norm_(clip)
            opt.step()
            opt.zero_grad()
    torch.cuda.synchronize()
    return [p.detach().cpu() for p in ma.parameters()], [p.detach().cpu() for p in mb.parameters()]


@pytest.mark.parametrize("clip", [None, 0.05])
def test_zero_hooks_equal_step_world1(clip):
    got, want = _hooks_vs_step(0, 1, "cuda", None, clip)
    assert all(torch.equal(a, b) for a, b in zip(got, want))


@pytest.mark.parametrize("in_backward", [True, False])
def test_zero_hooks_update_during_backward(in_backward):
    """With update_in_backward every round's update is enqueued by the hooks (the weights change before step()
    on the GPU timeline); step() only ends the step.  Either way the weights equal step()'s."""
    ma, mb = _mlp_pair("cuda")
    oa = ZeroAdamBridge(list(ma.parameters()), lr=2e-3, precision="bf16", seed=3, rounds=3)
    oa.attach_hooks(ma, update_in_backward=in_backward)
    ob = ZeroAdamBridge(list(mb.parameters()), lr=2e-3, precision="bf16", seed=3, rounds=3)
    for step in range(1, 4):
        _mlp_loss(ma, step, 0, "cuda").backward()
        assert len(oa._rounds_updated) == (3 if in_backward else 0)
        oa.step()
        oa.zero_grad()
        assert not oa._rounds_updated
        _mlp_loss(mb, step, 0, "cuda").backward()
        ob.step()
        ob.zero_grad()
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(ma.parameters(), mb.parameters()))
    if in_backward:
        _mlp_loss(ma, 9, 0, "cuda").backward()
        with pytest.raises(RuntimeError, match="update_in_backward=False"):
            oa.clip_grad_norm_(1.0)


def test_zero_hooks_reject_a_second_gradient():
    ma, _ = _mlp_pair("cuda")
    opt = ZeroAdamBridge(list(ma.parameters()), lr=1e-3, precision="bf16", rounds=2).attach_hooks(ma)
    _mlp_loss(ma, 1, 0, "cuda").backward()
    with pytest.raises(RuntimeError, match="second gradient"):
        _mlp_loss(ma, 2, 0, "cuda").backward()


def _hooks_rank(rank, world, port, out_dir, gather, clip):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        got, want = _hooks_vs_step(rank, world, f"cuda:{rank}", gather, clip)
        with open(os.path.join(out_dir, f"hooks{rank}.pkl"), "wb") as f:
            pickle.dump((got, want), f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("gather,clip", [("nccl", None), ("p2p", None), ("p2p", 0.05), ("ce", None)])
def test_zero_two_gpus_hooks_equal_step(tmp_path, gather, clip):
    """Reduce-scatters issued from the backward hooks, round by round, give the weights of step()'s
    reduce-scatters on every rank (ranks see different data, so the average matters)."""
    mp.start_processes(_hooks_rank, args=(2, _free_port(), str(tmp_path), gather, clip), nprocs=2,
                       start_method="spawn", join=True)
    ranks = [pickle.load(open(tmp_path / f"hooks{r}.pkl", "rb")) for r in range(2)]
    for got, want in ranks:
        assert all(torch.equal(a, b) for a, b in zip(got, want))
    assert all(torch.equal(a, b) for a, b in zip(ranks[0][0], ranks[1][0]))   # replicas agree


def test_zero_host_streamed_step_equals_device_step():
    """step_shard(pinned host gradient shard, weights_out=pinned host buffer) -- copies overlapping the rounds'
    updates -- gives the device path's weights, and weights_out holds this rank's updated weight shard."""
    pa, pb = _params("cuda"), _params("cuda")
    oa = ZeroAdamBridge(pa, lr=1e-3, precision="fp8", seed=3, rounds=3)
    ob = ZeroAdamBridge(pb, lr=1e-3, precision="fp8", seed=3, rounds=3)
    L = ob.layout
    out = torch.empty(L.shard_numel, dtype=torch.bfloat16, pin_memory=True)
    gen = torch.Generator().manual_seed(9)
    for _ in range(3):
        g = (torch.randn(L.shard_numel, generator=gen) * 1e-3).to(torch.bfloat16).pin_memory()
        oa.step_shard(g.cuda())
        ob.step_shard(g, weights_out=out)
    torch.cuda.synchronize()
    for a, b in zip(pa, pb):
        assert torch.equal(a, b)
    mine = torch.cat([ob.flat_weights[slice(*L.rank_range(r, 0))] for r in range(L.rounds)]).cpu()
    assert torch.equal(out, mine)
    with pytest.raises(ValueError):
        ob.step_shard(g[:-1])


# ---------------------------------------------------------------------------------------------- delayed updates

def _delayed_run(opt, model, steps, rank, device, hooks):
    if hooks:
        opt.attach_hooks(model)
    for step in range(1, steps + 1):
        _mlp_loss(model, step, rank, device).backward()
        opt.step()
        opt.zero_grad()
    opt.flush()
    torch.cuda.synchronize()
    return [p.detach().cpu() for p in model.parameters()]


@pytest.mark.parametrize("warmup", [0, 2])
@pytest.mark.parametrize("hooks", [False, True])
def test_zero_delayed_updates_equal_adambridge_delayed(warmup, hooks):
    """delay_updates: each step's update lands one step late, as in AdamBridge's (the reference's) delayed mode --
    identical weights after flush(), with and without backward hooks, with and without warm-up steps."""
    ma, mb = _mlp_pair("cuda")
    oa = ab.AdamBridge(list(ma.parameters()), lr=2e-3, precision="bf16", seed=3, small_param_threshold=0,
                       delay_updates=True, delay_warmup_steps=warmup)
    ob = ZeroAdamBridge(list(mb.parameters()), lr=2e-3, precision="bf16", seed=3, rounds=3,
                        delay_updates=True, delay_warmup_steps=warmup)
    want = _delayed_run(oa, ma, 5, 0, "cuda", False)
    got = _delayed_run(ob, mb, 5, 0, "cuda", hooks)
    assert all(torch.equal(a, b) for a, b in zip(got, want))
    oa.close()


def test_zero_delayed_weights_lag_one_step():
    """Before flush() the parameters hold the previous step's update: after two delayed steps they equal a
    synchronous optimizer's after one step on the same gradients."""
    ma, mb = _mlp_pair("cuda")
    o_sync = ZeroAdamBridge(list(ma.parameters()), lr=2e-3, precision="bf16", seed=3, rounds=2)
    o_del = ZeroAdamBridge(list(mb.parameters()), lr=2e-3, precision="bf16", seed=3, rounds=2, delay_updates=True)
    grads = []
    for step in (1, 2):
        g = torch.Generator().manual_seed(step)
        grads.append([(torch.randn(p.shape, generator=g) * 1e-2).to("cuda", torch.bfloat16) for p in ma.parameters()])
    for p, g in zip(ma.parameters(), grads[0]):
        p.grad = g
    o_sync.step()
    after_one = [p.detach().clone() for p in ma.parameters()]
    for gs in grads:
        for p, g in zip(mb.parameters(), gs):
            p.grad = g
        o_del.step()
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(mb.parameters(), after_one))
    o_del.flush()
    assert not all(torch.equal(a, b) for a, b in zip(mb.parameters(), after_one))


def _delayed_rank(rank, world, port, out_dir, gather):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        dev = f"cuda:{rank}"
        ma, mb = _mlp_pair(dev)
        kw = dict(lr=2e-3, precision="bf16", seed=3, rounds=3, delay_updates=True)
        oa = ZeroAdamBridge(list(ma.parameters()), gather=gather, **kw)
        ob = ZeroAdamBridge(list(mb.parameters()), gather="nccl", **kw)
        got = _delayed_run(oa, ma, 4, rank, dev, True)
        want = _delayed_run(ob, mb, 4, rank, dev, False)
        with open(os.path.join(out_dir, f"delayed{rank}.pkl"), "wb") as f:
            pickle.dump((got, want), f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("gather", ["p2p", "ce"])
def test_zero_two_gpus_delayed_updates(gather):
    """2 ranks, delayed updates: the gather through symmetric memory (peer stores or copy-engine copies) with
    hooks and NCCL's gather with step() end with the same weights on every rank."""
    import tempfile
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_delayed_rank, args=(2, _free_port(), tmp, gather), nprocs=2, start_method="spawn",
                           join=True)
        ranks = [pickle.load(open(os.path.join(tmp, f"delayed{r}.pkl"), "rb")) for r in range(2)]
    for got, want in ranks:
        assert all(torch.equal(a, b) for a, b in zip(got, want))
    assert all(torch.equal(a, b) for a, b in zip(ranks[0][0], ranks[1][0]))
