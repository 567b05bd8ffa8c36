"""Generate the golden fixtures in this folder from the reference's own kernel library.

    make -C oracle ref && python tests/golden/make_golden.py

Each fixture is a small seeded case shaped after one of the benchmark configurations, run for
several steps through ``adambridge_multi_step`` of oracle/_ref/libadambridge_ref.so (the reference's
adambridge/csrc/adambridge_kernels.c compiled from its sources) at a given SIMD level.  The npz holds
the starting buffers, every step's gradient and learning rate, and the final buffers, so that
tests can replay the same steps through the oracle (CPU) and through libabx (GPU) and compare
bit for bit, without the reference being present.
"""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import oracle as O  # noqa: E402

# name: (segments [(n, g_dtype, mv_dtype, out_dtype, p_dtype, algorithm)], steps, group, lr schedule, grad kind)
CONFIGS = {
    # config 1 shape, scaled down: one flat fp32 tensor, fp32 grad, no out, fp32 moments, 10 steps
    "c1_adamw_fp32": ([(4099, O.DT_F32, O.DT_F32, O.DT_NONE, O.DT_F32, O.ADAMW)], 10,
                      dict(lr=1e-4, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01), "const", "normal"),
    # config 2: bf16 moments, bf16 grad and weights, per-tensor grad scale, cosine LR from 2e-5
    "c2_adamw_bf16": ([(3000, O.DT_BF16, O.DT_BF16, O.DT_BF16, O.DT_F32, O.ADAMW),
                       (896, O.DT_BF16, O.DT_BF16, O.DT_BF16, O.DT_F32, O.ADAMW),
                       (1000, O.DT_BF16, O.DT_BF16, O.DT_BF16, O.DT_F32, O.ADAMW)], 8,
                      dict(lr=2e-5, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01), "cosine", "lognormal"),
    # config 3: fp8 moments, grads with 1% outliers x100
    "c3_adamw_fp8": ([(2560, O.DT_BF16, O.DT_FP8, O.DT_BF16, O.DT_F32, O.ADAMW),
                      (333, O.DT_BF16, O.DT_FP8, O.DT_BF16, O.DT_F32, O.ADAMW)], 6,
                     dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01), "const", "outliers"),
    # config 4: Lion, one bf16 moment
    "c4_lion_bf16": ([(2000, O.DT_BF16, O.DT_BF16, O.DT_BF16, O.DT_F32, O.LION),
                      (515, O.DT_BF16, O.DT_BF16, O.DT_BF16, O.DT_F32, O.LION)], 6,
                     dict(lr=1e-5, beta1=0.9, beta2=0.99, eps=0.0, weight_decay=0.1), "const", "normal"),
    # fp24 master with fp8 moments (AdamW) and with an fp8 moment (Lion)
    "fp24_adamw_fp8": ([(1537, O.DT_BF16, O.DT_FP8, O.DT_BF16, O.DT_F24, O.ADAMW)], 5,
                       dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01), "const", "normal"),
    "fp24_lion_fp8": ([(1537, O.DT_F32, O.DT_FP8, O.DT_F32, O.DT_F24, O.LION)], 5,
                      dict(lr=1e-4, beta1=0.9, beta2=0.99, eps=0.0, weight_decay=0.1), "const", "normal"),
}
LEVELS = {"avx512": O.SIMD_AVX512, "avx2": O.SIMD_AVX2, "scalar": O.SIMD_SCALAR}


def grads(kind: str, n: int, rng: np.random.Generator, sigma: float) -> np.ndarray:
    g = rng.standard_normal(n).astype(np.float32)
    if kind == "normal":
        return g * np.float32(1e-3)
    if kind == "lognormal":
        return g * np.float32(sigma)
    if kind == "outliers":
        g = g * np.float32(1e-3)
        g[rng.random(n) < 0.01] *= np.float32(100.0)
        return g
    raise ValueError(kind)


def lr_at(schedule: str, base: float, step: int, total: int) -> float:
    if schedule == "cosine":   # torch CosineAnnealingLR(T_max=total), eta_min 0, value used at step `step`
        return base * (1 + math.cos(math.pi * (step - 1) / total)) / 2
    return base


def make(name: str, level_name: str) -> dict:
    segs_spec, steps, group, schedule, gkind = CONFIGS[name]
    rng = np.random.default_rng(sum(map(ord, name)))
    segs = [O.HostSegment.random(n, gt, mv, ot, pt, algo, seed=1000 + i, index=i, p_scale=0.02)
            for i, (n, gt, mv, ot, pt, algo) in enumerate(segs_spec)]
    sigmas = [float(10 ** rng.uniform(-4, -2)) for _ in segs]
    initial = [{k: v.copy() for k, v in hs.buffers.items()} for hs in segs]
    all_grads = [[] for _ in segs]
    lrs = []
    ref = O.load_reference()
    if ref is None:
        raise SystemExit("oracle/_ref/libadambridge_ref.so is missing: run `make -C oracle ref` first")
    ref.set_simd_level(LEVELS[level_name])
    if ref.simd_level != LEVELS[level_name]:
        raise SystemExit(f"this CPU cannot run the reference at level {level_name}")
    for step in range(1, steps + 1):
        lr = lr_at(schedule, group["lr"], step, steps)
        lrs.append(lr)
        g = O.Group(**{**group, "lr": lr}, seed=11, stochastic=1)
        csegs = []
        for i, hs in enumerate(segs):
            gv = grads(gkind, hs.n, rng, sigmas[i])
            hs.buffers["g"][:] = O.bf16_bits(gv) if hs.g_dtype == O.DT_BF16 else gv
            all_grads[i].append(hs.buffers["g"].copy())
            hs.step = step
            csegs.append(hs.ctype(g))
        rc = ref.multi_step(csegs, 1)
        if rc != 0:
            raise RuntimeError(f"reference rejected {name}: {rc}")
    ref.set_simd_level(None)
    out = {"meta": json.dumps({"name": name, "level": LEVELS[level_name], "steps": steps, "group": group,
                               "seed": 11, "lrs": lrs,
                               "segments": [dict(n=s.n, g_dtype=s.g_dtype, mv_dtype=s.mv_dtype,
                                                 out_dtype=s.out_dtype, p_dtype=s.p_dtype, algorithm=s.algorithm,
                                                 index=s.index) for s in segs]})}
    for i, hs in enumerate(segs):
        for k, v in initial[i].items():
            if k != "g":
                out[f"s{i}_init_{k}"] = v
            out[f"s{i}_final_{k}"] = hs.buffers[k]
        out[f"s{i}_grads"] = np.stack(all_grads[i])
    return out


def main() -> None:
    for name in CONFIGS:
        levels = ("avx512", "avx2", "scalar") if name == "c2_adamw_bf16" else ("avx512",)
        for level in levels:
            data = make(name, level)
            path = HERE / f"{name}_{level}.npz"
            np.savez_compressed(path, **data)
            print(path.name, path.stat().st_size)


if __name__ == "__main__":
    main()
