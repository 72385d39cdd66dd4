"""pb_qmatvec_device_noalloc: the matvec operator for callers that cannot
allocate device memory (hosts whose own allocator owns the GPU's memory budget,
latency-critical loops, fixed-arena integrations).  It must give the same
binary32 results as pb_qmatvec_device -- bit for bit, the bar every matvec test
here uses -- on consecutive calls that share its fixed device scratch, and it
must reject sizes beyond that scratch.  This file is collected last and also
passes on its own in a fresh process (the first call sets the scratch up)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from promptboot_b200 import _lib

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _weights(rng, wtype, rows, cols):
    nb = rows * cols // 32
    scales = (np.abs(rng.standard_normal(nb) * 0.02) / 8).astype(np.float16)
    width = 18 if wtype == 2 else 34
    w = np.empty((nb, width), dtype=np.uint8)
    w[:, :2] = scales.view(np.uint8).reshape(nb, 2)
    if wtype == 2:
        w[:, 2:] = rng.integers(0, 256, size=(nb, 16), dtype=np.uint8)
    else:
        w[:, 2:] = rng.integers(-128, 128, size=(nb, 32), dtype=np.int8).view(np.uint8)
    return torch.from_numpy(w.reshape(-1)).to("cuda")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _run(fn, wtype, w, rows, cols, x, batch):
    y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
    status = fn(wtype, _ptr(w), rows, cols, _ptr(x), batch, _ptr(y), None)
    torch.cuda.synchronize()
    return status, y.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("wtype,rows,cols", [(2, 896, 896), (2, 896, 4864), (3, 1024, 896)])
def test_noalloc_matches_allocating_operator_on_consecutive_calls(wtype, rows, cols):
    lib = _lib.load()
    rng = np.random.default_rng(rows + cols + wtype)
    w = _weights(rng, wtype, rows, cols)
    for call, batch in enumerate((32, 5)):
        x = torch.from_numpy(rng.standard_normal((batch, cols)).astype(np.float32)).to("cuda")
        st_ref, ref = _run(lib.pb_qmatvec_device, wtype, w, rows, cols, x, batch)
        st, got = _run(lib.pb_qmatvec_device_noalloc, wtype, w, rows, cols, x, batch)
        assert st_ref == 0 and st == 0, (call, _lib.last_error())
        assert np.array_equal(got, ref), f"call {call}: no-alloc result differs"


def test_noalloc_back_to_back_calls_on_a_side_stream():
    """Two calls queued on one non-default stream with no synchronisation
    between them (the second overwrites the shared scratch only after the
    first's kernels are done, by stream order); each output equals the
    allocating operator's."""
    lib = _lib.load()
    rng = np.random.default_rng(11)
    w = _weights(rng, 2, 896, 4864)
    xs = [torch.from_numpy(rng.standard_normal((b, 4864)).astype(np.float32)).to("cuda")
          for b in (32, 3)]
    refs = [_run(lib.pb_qmatvec_device, 2, w, 896, 4864, x, x.shape[0])[1] for x in xs]
    side = torch.cuda.Stream()
    ys = [torch.full((x.shape[0], 896), float("nan"), device="cuda") for x in xs]
    torch.cuda.synchronize()
    handle = ctypes.c_void_p(side.cuda_stream)
    for x, y in zip(xs, ys):
        assert lib.pb_qmatvec_device_noalloc(2, _ptr(w), 896, 4864, _ptr(x), x.shape[0], _ptr(y),
                                             handle) == 0
    side.synchronize()
    for i, (y, ref) in enumerate(zip(ys, refs)):
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref), i


def test_noalloc_allocates_nothing_after_setup():
    lib = _lib.load()
    rng = np.random.default_rng(7)
    w = _weights(rng, 2, 896, 896)
    x = torch.from_numpy(rng.standard_normal((8, 896)).astype(np.float32)).to("cuda")
    y = torch.empty((8, 896), dtype=torch.float32, device="cuda")
    assert lib.pb_qmatvec_device_noalloc(2, _ptr(w), 896, 896, _ptr(x), 8, _ptr(y), None) == 0
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert lib.pb_qmatvec_device_noalloc(2, _ptr(w), 896, 896, _ptr(x), 8, _ptr(y), None) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    rng = np.random.default_rng(3)
    w = _weights(rng, 2, 896, 896)
    x = torch.zeros((33, 896), dtype=torch.float32, device="cuda")
    y = torch.zeros((33, 896), dtype=torch.float32, device="cuda")
    assert lib.pb_qmatvec_device_noalloc(2, _ptr(w), 896, 896, _ptr(x), 33, _ptr(y), None) == 4
    assert "32" in _lib.last_error()
    assert lib.pb_qmatvec_device_noalloc(2, _ptr(w), 896, 8960, _ptr(x), 1, _ptr(y), None) == 4
    torch.cuda.synchronize()
    assert not y.any()
