"""Generate checkpoints written by adambridge_b200, for the reference to load (needs a GPU).

    python tests/golden/make_b200_checkpoints.py [output directory]

For each case -- the moment precisions, fp32 and fp24 masters, bf16 and fp32 weights, AdamW and Lion -- a few
small CUDA parameters take three steps of adambridge_b200's AdamBridge / LionBridge; the file keeps the weights
and the ``state_dict()`` (moved to the host), the gradients of a fourth step, and the weights and
``state_dict()`` after adambridge_b200 took that step.  tests/test_checkpoint_to_reference_cpu.py loads each
into the reference's own optimizer on the CPU, takes the fourth step there and compares bit for bit.  The
output lands in tests/golden/checkpoints_b200/ unless a directory is given.
"""

from __future__ import annotations

import io
import sys
import zlib
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

import adambridge_b200 as ab  # noqa: E402

# case: (algorithm, moment precision, master precision, weight dtype)
CASES = {
    "adamw_fp32_bf16w": ("adamw", "fp32", "fp32", torch.bfloat16),
    "adamw_bf16_bf16w": ("adamw", "bf16", "fp32", torch.bfloat16),
    "adamw_fp8_bf16w": ("adamw", "fp8", "fp32", torch.bfloat16),
    "adamw_fp8_fp24_bf16w": ("adamw", "fp8", "fp24", torch.bfloat16),
    "adamw_bf16_fp32w": ("adamw", "bf16", "fp32", torch.float32),
    "lion_bf16_bf16w": ("lion", "bf16", "fp32", torch.bfloat16),
    "lion_fp8_fp24_bf16w": ("lion", "fp8", "fp24", torch.bfloat16),
}
SHAPES = [(40, 50), (256,), (130, 20)]
HYPER = {"adamw": dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01),
         "lion": dict(lr=1e-3, betas=(0.9, 0.99), weight_decay=0.1)}


def to_host(obj):
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu().clone()
    if isinstance(obj, dict):
        return {k: to_host(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(to_host(v) for v in obj)
    return obj


def case_blob(case: str) -> bytes:
    algo, prec, master, wdtype = CASES[case]
    gen = torch.Generator().manual_seed(zlib.crc32(case.encode()) & 0xFFFF)
    params = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(wdtype).cuda()) for s in SHAPES]
    cls = ab.LionBridge if algo == "lion" else ab.AdamBridge
    opt = cls(params, precision=prec, master_precision=master, seed=11, **HYPER[algo])

    def grads():
        scale = 10.0 ** float(torch.empty(1).uniform_(-4, -2, generator=gen))
        return [(torch.randn(s, generator=gen) * scale).to(wdtype) for s in SHAPES]

    for _ in range(3):
        for p, g in zip(params, grads()):
            p.grad = g.cuda()
        opt.step()
        opt.zero_grad(set_to_none=True)
    before = {"weights": to_host(list(params)), "state_dict": to_host(opt.state_dict())}
    g4 = grads()
    for p, g in zip(params, g4):
        p.grad = g.cuda()
    opt.step()
    after = {"weights": to_host(list(params)), "state_dict": to_host(opt.state_dict())}
    blob = {"case": case, "algorithm": algo, "precision": prec, "master_precision": master,
            "weight_dtype": str(wdtype), "shapes": SHAPES, "simd_level": ab.native.load().simd_level,
            "hyper": {**HYPER[algo], "seed": 11}, "before": before, "grads": g4, "after": after}
    opt.close()
    buf = io.BytesIO()
    torch.save(blob, buf)
    return buf.getvalue()


def main() -> None:
    out = Path(sys.argv[1]) if len(sys.argv) > 1 else HERE / "checkpoints_b200"
    out.mkdir(parents=True, exist_ok=True)
    for case in CASES:
        (out / f"{case}.pt").write_bytes(case_blob(case))
    print(f"wrote {len(CASES)} checkpoints to {out}")


if __name__ == "__main__":
    main()
