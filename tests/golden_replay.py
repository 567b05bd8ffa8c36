"""Replay a golden fixture (tests/golden/*.npz, made by tests/golden/make_golden.py from the reference's own
library) through a checker or through libabx, and compare with the reference's final buffers."""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def fixtures() -> list[Path]:
    return sorted(GOLDEN.glob("*.npz"))


def load(path: Path):
    d = np.load(path)
    meta = json.loads(str(d["meta"]))
    segs, grads, finals = [], [], []
    for i, s in enumerate(meta["segments"]):
        hs = O.HostSegment(s["n"], s["g_dtype"], s["mv_dtype"], s["out_dtype"], s["p_dtype"], s["algorithm"],
                           index=s["index"])
        hs.buffers = {k[len(f"s{i}_init_"):]: d[k].copy() for k in d.files if k.startswith(f"s{i}_init_")}
        g = d[f"s{i}_grads"]
        hs.buffers["g"] = g[0].copy()
        segs.append(hs)
        grads.append(g)
        final = O.HostSegment(hs.n, hs.g_dtype, hs.mv_dtype, hs.out_dtype, hs.p_dtype, hs.algorithm, index=hs.index)
        final.buffers = {k[len(f"s{i}_final_"):]: d[k].copy() for k in d.files if k.startswith(f"s{i}_final_")}
        finals.append(final)
    return meta, segs, grads, finals


def replay_oracle(path: Path, oracle) -> list[dict]:
    meta, segs, grads, finals = load(path)
    for step in range(1, meta["steps"] + 1):
        g = O.Group(**{**meta["group"], "lr": meta["lrs"][step - 1]}, seed=meta["seed"], stochastic=1)
        csegs = []
        for hs, gs in zip(segs, grads):
            hs.buffers["g"][:] = gs[step - 1]
            hs.step = step
            csegs.append(hs.ctype(g))
        assert oracle.multi_step(csegs, meta["level"]) == 0
    return [hs.mismatches(f) for hs, f in zip(segs, finals)]


def replay_gpu(path: Path, kernels) -> list[dict]:
    import torch

    from adambridge_b200 import native
    from conftest import device_segment, from_device, to_device

    meta, segs, grads, finals = load(path)
    kernels.set_simd_level(O.SIMD_NAMES[meta["level"]])
    devs = [to_device(hs) for hs in segs]
    for step in range(1, meta["steps"] + 1):
        g = native.Group(**{**meta["group"], "lr": meta["lrs"][step - 1]}, seed=meta["seed"], stochastic=1)
        ptrs, keep = [], []
        for hs, gs, dev in zip(segs, grads, devs):
            a = gs[step - 1]
            dev["g"].copy_(torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda())
            hs.step = step
            s = device_segment(hs, dev, g)
            keep.append(s)
            ptrs.append(ctypes.pointer(s))
        kernels.multi_step(None, kernels.segment_array(ptrs))
    torch.cuda.synchronize()
    kernels.set_simd_level(None)
    return [from_device(hs, dev).mismatches(f) for hs, dev, f in zip(segs, devs, finals)]
