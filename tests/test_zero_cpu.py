"""ZeRO-1 sharding logic on CPU: the flat layout, the per-rank pieces, and a world-size-2 gloo run in which
each rank updates only its shard (with the oracle standing in for the kernel) and the bf16 weights are
all-gathered -- bit-identical to the unsharded update.  This is the property the GPU path relies on: a piece
of a tensor at a 128-aligned tensor-local offset rounds exactly like the whole tensor
(tests/native/selftest.c:304-336)."""

from __future__ import annotations

import os
import pickle
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from adambridge_b200.zero import ALIGN, FlatLayout, ZeroAdamBridge
from oracle import oracle as O

SIZES = [5000, 128, 37, 70001, 4096, 300, 129, 20000]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("rounds", [None, 1, 4])
def test_layout_covers_every_element_once(world, rounds):
    L = FlatLayout(SIZES, world, rounds)
    assert L.total == L.rounds * L.world * L.chunk and L.chunk % ALIGN == 0
    assert all(o % ALIGN == 0 for o in L.offsets)
    seen = [np.zeros(n, np.int32) for n in SIZES]
    for rank in range(world):
        locals_ = []
        for r, pieces in enumerate(L.pieces(rank)):
            lo, hi = L.rank_range(r, rank)
            for pc in pieces:
                assert lo <= pc.flat_lo and pc.flat_lo + pc.n <= hi
                assert pc.flat_lo == L.offsets[pc.index] + pc.t_lo
                assert pc.local_lo == r * L.chunk + (pc.flat_lo - lo)
                assert pc.t_lo % ALIGN == 0 and pc.local_lo % ALIGN == 0   # FP8 blocks and scales line up
                seen[pc.index][pc.t_lo:pc.t_hi] += 1
                locals_.append((pc.local_lo, pc.local_lo + pc.n))
        locals_.sort()
        assert all(a[1] <= b[0] for a, b in zip(locals_, locals_[1:]))   # shard storage does not overlap
        assert all(b <= L.shard_numel for _, b in locals_)
    assert all((s == 1).all() for s in seen)


def test_one_round_without_peers():
    assert FlatLayout(SIZES, 1).rounds == 1


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_order_starts_at_the_next_rank(world):
    """Each rank lists its peers from the next rank on, so at any moment of the gather every GPU receives from a
    different sender; the distances are those of the peers' buffers."""
    from types import SimpleNamespace
    ptrs = [1000 * (r + 1) + 7 * r * r for r in range(world)]
    firsts = []
    for rank in range(world):
        d = ZeroAdamBridge._rotated_deltas(SimpleNamespace(rank=rank, world=world), ptrs)
        peers = [(rank + j) % world for j in range(1, world)]
        assert d == [ptrs[p] - ptrs[rank] for p in peers]
        firsts.append(peers[0])
    assert sorted(firsts) == list(range(world))


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("rounds", [None, 1, 4, 16])
def test_rounds_of_lists_exactly_the_rounds_a_parameter_touches(world, rounds):
    """The backward hooks start a round's reduce-scatter when every parameter listed for it has its gradient:
    rounds_of must list exactly the rounds whose flat range intersects the parameter, and every piece of a
    rank's shard must belong to a parameter listed for that piece's round."""
    L = FlatLayout(SIZES, world, rounds)
    for i in range(len(SIZES)):
        a, b = L.flat_slice(i)
        want = [r for r in range(L.rounds) if max(a, L.round_range(r)[0]) < min(b, L.round_range(r)[1])]
        assert L.rounds_of(i) == want
    for rank in range(world):
        for r, pieces in enumerate(L.pieces(rank)):
            assert all(r in L.rounds_of(pc.index) for pc in pieces)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("rounds", [None, 1, 4])
@pytest.mark.parametrize("unit,padded", [(1, False), (1, True), (ALIGN, True)])
def test_shard_runs_scatter_and_gather_round_trip(world, rounds, unit, padded):
    """The checkpoint mapping: per-parameter arrays (padded to whole 128-element blocks for FP8 codes, one
    entry per block for FP8 scales) scattered into every rank's shard by ``shard_runs`` and gathered back
    are unchanged, and every entry of every parameter lands in exactly one shard."""
    L = FlatLayout(SIZES, world, rounds)
    lengths = [(-(-n // ALIGN) * ALIGN if padded else n) // unit for n in SIZES]
    rng = np.random.default_rng(world * 100 + (rounds or 0))
    full = [rng.integers(1, 1 << 30, n) for n in lengths]
    shards = [np.zeros(L.shard_numel // unit, np.int64) for _ in range(world)]
    hits = [np.zeros(n, np.int64) for n in lengths]
    for r in range(world):
        for index, p_lo, s_lo, length in L.shard_runs(r, unit, padded):
            shards[r][s_lo:s_lo + length] = full[index][p_lo:p_lo + length]
            hits[index][p_lo:p_lo + length] += 1
    assert all((h == 1).all() for h in hits)
    back = [np.zeros(n, np.int64) for n in lengths]
    for r in range(world):
        for index, p_lo, s_lo, length in L.shard_runs(r, unit, padded):
            back[index][p_lo:p_lo + length] = shards[r][s_lo:s_lo + length]
    assert all((a == b).all() for a, b in zip(full, back))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


GROUP = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, seed=3, stochastic=1)


def _inputs(steps):
    rng = np.random.default_rng(5)
    params = [(rng.standard_normal(n) * 0.02).astype(np.float32) for n in SIZES]
    grads = [[(rng.standard_normal(n) * 1e-3).astype(np.float32) for n in SIZES] for _ in range(steps)]
    return [O.bf16_to_f32(O.bf16_bits(p)) for p in params], grads


def _unsharded(mv, steps):
    params, grads = _inputs(steps)
    orc = O.load_oracle()
    segs = []
    for i, p in enumerate(params):
        hs = O.HostSegment.random(len(p), O.DT_BF16, mv, O.DT_BF16, O.DT_F32, O.ADAMW, index=i)
        hs.buffers["p"][:] = p
        segs.append(hs)
    for step in range(1, steps + 1):
        for hs, g in zip(segs, grads[step - 1]):
            hs.buffers["g"][:] = O.bf16_bits(g)
            hs.step = step
        assert orc.multi_step([hs.ctype(O.Group(**GROUP)) for hs in segs], O.SIMD_AVX512) == 0
    return segs


def _rank_main(rank, world, port, mv, steps, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        params, grads = _inputs(steps)
        orc = O.load_oracle()
        L = FlatLayout(SIZES, world, rounds=3)
        pieces = L.pieces(rank)
        mb = {O.DT_BF16: np.uint16, O.DT_FP8: np.uint8}[mv]
        master = np.zeros(L.shard_numel, np.float32)
        m = np.zeros(L.shard_numel, mb)
        v = np.zeros(L.shard_numel, mb)
        m_scale = np.ones(L.shard_numel // ALIGN, np.float32)
        v_scale = np.ones(L.shard_numel // ALIGN, np.float32)
        gshard = np.zeros(L.shard_numel, np.uint16)
        flat_w = np.zeros(L.total, np.uint16)
        for i, p in enumerate(params):
            a, b = L.flat_slice(i)
            flat_w[a:b] = O.bf16_bits(p)
        for r in range(L.rounds):
            lo, hi = L.rank_range(r, rank)
            master[r * L.chunk:(r + 1) * L.chunk] = O.bf16_to_f32(flat_w[lo:hi])
        for step in range(1, steps + 1):
            segs = []
            for rp in pieces:
                for pc in rp:
                    gshard[pc.local_lo:pc.local_lo + pc.n] = O.bf16_bits(grads[step - 1][pc.index][pc.t_lo:pc.t_hi])
                    s = O.Segment(p=master.ctypes.data + 4 * pc.local_lo, g=gshard.ctypes.data + 2 * pc.local_lo,
                                  m=m.ctypes.data + m.itemsize * pc.local_lo, v=v.ctypes.data + v.itemsize * pc.local_lo,
                                  out=flat_w.ctypes.data + 2 * pc.flat_lo, n=pc.n, step=step, index=pc.index,
                                  offset=pc.t_lo, g_dtype=O.DT_BF16, mv_dtype=mv, out_dtype=O.DT_BF16,
                                  algorithm=O.ADAMW, p_dtype=O.DT_F32)
                    if mv == O.DT_FP8:
                        s.m_scale = m_scale.ctypes.data + 4 * (pc.local_lo // ALIGN)
                        s.v_scale = v_scale.ctypes.data + 4 * (pc.local_lo // ALIGN)
                    segs.append(s)
            grp = O.Group(**GROUP)
            for s in segs:
                s.group = O.ctypes.pointer(grp)
            assert orc.multi_step(segs, O.SIMD_AVX512) == 0
            for r in range(L.rounds):   # the all-gather of each round's bf16 weights
                lo, hi = L.round_range(r)
                # bf16 bit patterns widened to int32 (gloo has no 16-bit integer type)
                mine = torch.from_numpy(flat_w[slice(*L.rank_range(r, rank))].astype(np.int32))
                parts = [torch.empty_like(mine) for _ in range(world)]
                dist.all_gather(parts, mine)
                flat_w[lo:hi] = torch.cat(parts).numpy().astype(np.uint16)
        with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
            pickle.dump({"flat_w": flat_w, "master": master, "m": m, "pieces": pieces, "chunk": L.chunk,
                         "offsets": L.offsets, "m_scale": m_scale}, f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mv", [O.DT_BF16, O.DT_FP8])
def test_two_rank_gloo_sharded_update_is_bit_exact(tmp_path, mv):
    steps, world = 3, 2
    mp.start_processes(_rank_main, args=(world, _free_port(), mv, steps, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    want = _unsharded(mv, steps)
    results = [pickle.load(open(tmp_path / f"rank{r}.pkl", "rb")) for r in range(world)]
    for res in results:   # every rank holds the same, complete bf16 weights
        for i, hs in enumerate(want):
            a = res["offsets"][i]
            assert np.array_equal(res["flat_w"][a:a + hs.n], hs.buffers["out"]), i
    for res in results:   # and its shard of the master and moments equals the unsharded state
        for rp in res["pieces"]:
            for pc in rp:
                hs = want[pc.index]
                assert np.array_equal(res["master"][pc.local_lo:pc.local_lo + pc.n].view(np.uint32),
                                      hs.buffers["p"][pc.t_lo:pc.t_hi].view(np.uint32))
                assert np.array_equal(res["m"][pc.local_lo:pc.local_lo + pc.n], hs.buffers["m"][pc.t_lo:pc.t_hi])
                if mv == O.DT_FP8:
                    nb = -(-pc.n // ALIGN)
                    assert np.array_equal(res["m_scale"][pc.local_lo // ALIGN:pc.local_lo // ALIGN + nb],
                                          hs.buffers["m_scale"][pc.t_lo // ALIGN:pc.t_lo // ALIGN + nb])
