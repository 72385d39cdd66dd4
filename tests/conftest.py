"""Shared pytest configuration: the `gpu` marker and repository import path."""
from __future__ import annotations

import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


import pytest  # noqa: E402


@pytest.fixture(scope="session")
def model_image():
    """Seeded synthetic PBTQW25 v1 image (config 0 weights), cached on disk."""
    from promptboot_b200 import pbtqw25
    return pbtqw25.load_or_synthesize(0)


@pytest.fixture(scope="session")
def model_view(model_image):
    from promptboot_b200 import api
    view = api.ModelView(model_image, device=0)
    yield view
    view.close()


def dev(array):
    """Copy a numpy array to a new cuda:0 tensor (test plumbing only)."""
    import numpy as np
    import torch
    a = np.ascontiguousarray(array).copy()
    signed = {np.dtype(np.uint16): np.int16, np.dtype(np.uint32): np.int32,
              np.dtype(np.uint64): np.int64}
    if a.dtype in signed:
        a = a.view(signed[a.dtype])
    return torch.from_numpy(a).to("cuda:0")


def ptr(t):
    import ctypes
    return ctypes.c_void_p(t.data_ptr())
