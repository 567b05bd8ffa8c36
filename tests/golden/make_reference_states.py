"""Generate fixtures from the reference's own Python package: state-format conversions and optimizer checkpoints.

    ABX_REFERENCE=<reference checkout> python tests/golden/make_reference_states.py

(ABX_REFERENCE defaults to a ``reference`` directory beside this repository.)  The reference is imported from
its checkout with its native backend (its C library, built by its own loader into a temporary cache) and run on
the CPU.  Two kinds of fixture land next to this script:

* ``convert/conversions.npz`` -- seeded values (ordinary, zero, negative zero, tiny, huge, infinite and NaN)
  written into the reference's stores by its own code (adambridge/precision.py: BF16Store, FP8Store for both
  roles, FP24Store, an FP8 store saved under one role and loaded under the other, a 64-element-block FP8 store)
  and read back.  libabx's conversion kernel and the CPU checker in oracle/convert.py are compared with them.
* ``checkpoints/<case>.pt`` -- a few small parameters trained for three steps by the reference's AdamBridge /
  LionBridge (CPU parameters, its native update at the SIMD level recorded in the file), its ``state_dict()``
  then, the gradients of a fourth step, and the weights and ``state_dict()`` after that step.  A test loads
  the checkpoint into adambridge_b200 on the GPU, takes the fourth step and compares bit for bit.
"""

from __future__ import annotations

import copy
import io
import os
import sys
import tempfile
import zlib
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def reference_tree() -> Path:
    env = os.environ.get("ABX_REFERENCE")
    tree = Path(env) if env else REPO.parent / "reference"
    if not (tree / "adambridge" / "precision.py").exists():
        sys.exit(f"the reference checkout is not at {tree}: set ABX_REFERENCE")
    return tree


def special_values(rng: np.random.Generator, n: int, nonneg: bool) -> np.ndarray:
    x = (rng.standard_normal(n) * 10.0 ** rng.uniform(-12, 4, n)).astype(np.float32)
    if nonneg:
        x = np.abs(x)
    specials = np.array([0.0, -0.0, 1e-45, -1e-45, 1e-38, 3e38, -3e38, np.inf, -np.inf, np.nan, 448.0, 460.0,
                         57344.0, 60000.0, 1.0, -1.0], np.float32)
    idx = rng.choice(n, size=specials.size, replace=False)
    x[idx] = specials
    # one block with no special value at all, one all-zero block
    x[256:384] = (rng.standard_normal(128) * 1e-3).astype(np.float32)
    x[384:512] = 0.0
    return x


def conversions(precision) -> dict:
    rng = np.random.default_rng(20261202)
    n = 1000                              # 8 blocks, the last one partial
    xm = special_values(rng, n, nonneg=False)
    xv = special_values(rng, n, nonneg=True)
    xv[rng.choice(n, 5, replace=False)] = -rng.uniform(0, 1, 5).astype(np.float32)   # negative v: sqrt(max(v, 0))
    out = {"x_m": xm, "x_v": xv}
    tm, tv = torch.from_numpy(xm.copy()), torch.from_numpy(xv.copy())

    bf = precision.BF16Store(n, init=tm.clone())
    out["bf16_data"] = bf.data.view(torch.int16).numpy().view(np.uint16)
    out["bf16_read"] = bf.to_fp32().numpy()
    for role, t in (("m", tm), ("v", tv)):
        st = precision.FP8Store(n, role, init=t.clone())
        out[f"fp8_{role}_q"] = st.q.view(torch.uint8).numpy()
        out[f"fp8_{role}_scale"] = st.scale.numpy()
        out[f"fp8_{role}_read"] = st.to_fp32().numpy()
    f24 = precision.FP24Store(n, init=tm.clone())
    out["fp24_hi"] = f24.hi.view(torch.int16).numpy().view(np.uint16)
    out["fp24_lo"] = f24.lo.numpy()
    out["fp24_read"] = f24.to_fp32().numpy()
    # an m store loaded as a v store: decoded as E4M3, re-encoded as E5M2 of sqrt
    m_store = precision.FP8Store(n, "m", init=tv.clone())
    out["m_as_v_src_q"] = m_store.q.view(torch.uint8).numpy()
    out["m_as_v_src_scale"] = m_store.scale.numpy()
    moved = precision.store_from_state_dict(m_store.state_dict(), n, "v")
    out["m_as_v_q"] = moved.q.view(torch.uint8).numpy()
    out["m_as_v_scale"] = moved.scale.numpy()
    # a 64-element-block store (a block size the reference's torch path accepts) and its values
    b64 = precision.FP8Store(n, "m", init=tm.clone(), block=64)
    out["fp8_b64_q"] = b64.q.view(torch.uint8).numpy()
    out["fp8_b64_scale"] = b64.scale.numpy()
    out["fp8_b64_read"] = b64.to_fp32().numpy()
    return {k: np.ascontiguousarray(v) for k, v in out.items()}


# case: (algorithm, moment precision, master precision, weight dtype)
CASES = {
    "adamw_fp32_bf16w": ("adamw", "fp32", "fp32", torch.bfloat16),
    "adamw_bf16_bf16w": ("adamw", "bf16", "fp32", torch.bfloat16),
    "adamw_fp8_bf16w": ("adamw", "fp8", "fp32", torch.bfloat16),
    "adamw_bf16_fp24_bf16w": ("adamw", "bf16", "fp24", torch.bfloat16),
    "adamw_bf16_fp32w": ("adamw", "bf16", "fp32", torch.float32),
    "lion_bf16_bf16w": ("lion", "bf16", "fp32", torch.bfloat16),
    "lion_fp8_fp24_bf16w": ("lion", "fp8", "fp24", torch.bfloat16),
}
SHAPES = [(40, 50), (256,), (130, 20)]   # 2000, 256, 2600 elements: whole and partial FP8 blocks


def checkpoint(adambridge, native, case: str) -> bytes:
    algo, prec, master, wdtype = CASES[case]
    gen = torch.Generator().manual_seed(zlib.crc32(case.encode()) & 0xFFFF)
    params = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(wdtype)) for s in SHAPES]
    kw = dict(precision=prec, master_precision=master, seed=11)
    if algo == "lion":
        opt = adambridge.LionBridge(params, lr=1e-3, betas=(0.9, 0.99), weight_decay=0.1, **kw)
    else:
        opt = adambridge.AdamBridge(params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, **kw)

    def grads():
        return [(torch.randn(s, generator=gen) * 10.0 ** float(torch.empty(1).uniform_(-4, -2, generator=gen)))
                .to(wdtype) for s in SHAPES]

    for _ in range(3):
        for p, g in zip(params, grads()):
            p.grad = g
        opt.step()
        opt.zero_grad(set_to_none=True)
    # the state dict holds the live state tensors: copy them before the next step changes them in place
    before = {"weights": [p.detach().clone() for p in params], "state_dict": copy.deepcopy(opt.state_dict())}
    g4 = grads()
    for p, g in zip(params, g4):
        p.grad = g.clone()
    opt.step()
    after = {"weights": [p.detach().clone() for p in params], "state_dict": copy.deepcopy(opt.state_dict())}
    blob = {"case": case, "algorithm": algo, "precision": prec, "master_precision": master,
            "weight_dtype": str(wdtype), "shapes": SHAPES, "simd_level": native.load().simd_level,
            "hyper": {"lr": 1e-3, "betas": (0.9, 0.99) if algo == "lion" else (0.9, 0.999),
                      "weight_decay": 0.1 if algo == "lion" else 0.01, "seed": 11},
            "before": before, "grads": g4, "after": after}
    buf = io.BytesIO()
    torch.save(blob, buf)
    opt.close()
    return buf.getvalue()


def main() -> None:
    tree = reference_tree()
    os.environ.setdefault("ADAMBRIDGE_CACHE_DIR", tempfile.mkdtemp(prefix="abx-ref-cache-"))
    sys.path.insert(0, str(tree))
    import adambridge
    from adambridge import native, precision

    if native.load() is None:
        sys.exit("the reference's native backend did not build")
    (HERE / "convert").mkdir(exist_ok=True)
    np.savez_compressed(HERE / "convert" / "conversions.npz", **conversions(precision))
    (HERE / "checkpoints").mkdir(exist_ok=True)
    for case in CASES:
        (HERE / "checkpoints" / f"{case}.pt").write_bytes(checkpoint(adambridge, native, case))
    print(f"wrote convert/conversions.npz and {len(CASES)} checkpoints (simd {native.load().simd_level})")


if __name__ == "__main__":
    main()
