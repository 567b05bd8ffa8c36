"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on a CPU-only machine.

The parity checker is the oracle (oracle/abx_oracle.c, a C restatement of the reference's
update arithmetic) and, where it was built, the reference's own kernel library
(oracle/_ref/libadambridge_ref.so).  GPU tests run one seeded case through the CUDA kernels
and through the checker and compare every buffer bit for bit.
"""

from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402

CUDA = torch.cuda.is_available()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


def pytest_collection_modifyitems(config, items):
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords and not CUDA:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    return O.load_oracle()


@pytest.fixture(scope="session")
def reference():
    return O.load_reference()


@pytest.fixture(scope="session")
def kernels():
    from adambridge_b200 import native
    return native.load()


# ---------------------------------------------------------------- device copies of HostSegments

_TORCH = {np.dtype(np.float32): torch.float32, np.dtype(np.uint16): torch.int16, np.dtype(np.uint8): torch.uint8}


def to_device(hs: O.HostSegment, device="cuda") -> dict[str, torch.Tensor]:
    """Device tensors holding the same bytes as ``hs``'s buffers."""
    out = {}
    for k, a in hs.buffers.items():
        t = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a)
        out[k] = t.to(device)
    return out


def from_device(hs: O.HostSegment, dev: dict[str, torch.Tensor]) -> O.HostSegment:
    """A copy of ``hs`` whose buffers hold the device tensors' bytes."""
    c = hs.clone()
    for k, t in dev.items():
        a = t.cpu().numpy()
        c.buffers[k][:] = a.view(np.uint16) if c.buffers[k].dtype == np.uint16 else a
    return c


def device_segment(hs: O.HostSegment, dev: dict[str, torch.Tensor], group=None, elem_offset: int = 0):
    """A product Segment (adambridge_b200.native.Segment) over the device buffers."""
    from adambridge_b200 import native
    ptr = (lambda k: dev[k].data_ptr() if k in dev else None)
    s = native.Segment(p=ptr("p"), p_lo=ptr("p_lo"), g=ptr("g"), m=ptr("m"), v=ptr("v"), m_scale=ptr("m_scale"),
                       v_scale=ptr("v_scale"), out=ptr("out"), n=hs.n, step=hs.step, index=hs.index,
                       offset=hs.offset, g_dtype=hs.g_dtype, mv_dtype=hs.mv_dtype, out_dtype=hs.out_dtype,
                       algorithm=hs.algorithm, p_dtype=hs.p_dtype)
    if group is not None:
        s.group = ctypes.cast(ctypes.pointer(group), ctypes.POINTER(native.Group))
    return s


def product_group(**kw):
    from adambridge_b200 import native
    return native.Group(**kw)


def oracle_group(**kw):
    return O.Group(**kw)
