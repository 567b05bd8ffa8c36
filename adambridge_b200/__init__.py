"""adambridge_b200: adambridge's fused AdamW / Lion optimizer-update hot path on B200.

The optimizer state (FP32 or FP24 master weights, FP32 / BF16 / block-scaled FP8
moments) lives in HBM and is updated by hand-written sm_100a kernels (libabx, C ABI in
include/abx.h), behind the reference's ``AdamBridge`` / ``OptiComputeAdamW`` /
``LionBridge`` API.  ``ZeroAdamBridge`` / ``ZeroLionBridge`` (``adambridge_b200.zero``) shard
the state ZeRO-1 style over the ranks of a process group; the all-gather of the new bf16
weights is fused into the update as NVLink stores into the peers' copies, or run by NCCL.
``clip_coefficient`` computes torch's gradient-clipping norm and coefficient on the device.
"""

from . import native, precision
from .clip import clip_coefficient
from .engine import StepStats
from .optimizer import AdamBridge, LionBridge, OptiComputeAdamW
from .precision import bytes_per_param

__version__ = "0.1.0"

__all__ = [
    "AdamBridge",
    "LionBridge",
    "OptiComputeAdamW",
    "StepStats",
    "bytes_per_param",
    "clip_coefficient",
    "native",
    "precision",
    "__version__",
]
