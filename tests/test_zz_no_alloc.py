"""mb_op_mesh_backward_noalloc: the allocation-free mesh stack backward.

Callers that must not allocate device memory per call (a service with a
fixed device-memory budget, a host whose caching allocator must see every
allocation) use this variant; it keeps its gradient partials in a static
device array instead of cudaMallocAsync scratch.  This test calls it through
the C ABI twice in a row and checks both results against the allocating
entry point mb_op_mesh_backward, with the tolerances of the mesh op tests.
It lives in a file pytest collects last, and passes alone or after the rest.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call(fn, x, dy, w, conn):
    import torch
    rows, width = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    status = fn(p(x), p(dy), p(dx), p(dw), rows, width, w.shape[0], conn, p(w), stream)
    return status, dx, dw


@pytest.mark.parametrize("width,depth,conn,rows", [(512, 4, 0, 4097), (128, 6, 1, 3000), (256, 16, 0, 65536)])
def test_noalloc_matches_allocating_entry_point(width, depth, conn, rows):
    import torch

    from grokking_abmod_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(width + depth)
    x = torch.from_numpy(rng.standard_normal((rows, width)).astype(np.float32)).cuda()
    dy = torch.from_numpy(rng.standard_normal((rows, width)).astype(np.float32)).cuda()
    w_np = np.empty((depth, width, 2), dtype=np.float32)
    w_np[..., 0] = 0.7 + 0.2 * (rng.random((depth, width)) - 0.5)
    w_np[..., 1] = 0.4 * (rng.random((depth, width)) - 0.5)
    w = torch.from_numpy(w_np).cuda()
    status, ref_dx, ref_dw = _call(lib.mb_op_mesh_backward, x, dy, w, conn)
    assert status == 0
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        status, dx, dw = _call(lib.mb_op_mesh_backward_noalloc, x, dy, w, conn)
        assert status == 0
        torch.cuda.synchronize()
        rdx, rdw = ref_dx.cpu().numpy(), ref_dw.cpu().numpy()
        assert np.abs(dx.cpu().numpy() - rdx).max() <= 1e-5 * (1 + np.abs(rdx).max())
        assert np.abs(dw.cpu().numpy() - rdw).max() <= 1e-4 * np.abs(rdw).max()


def test_noalloc_rejects_invalid_requests():
    import torch

    from grokking_abmod_b200 import _lib
    lib = _lib.load()
    x = torch.zeros((8, 128), device="cuda")
    w = torch.zeros((17, 128, 2), device="cuda")
    status, _, _ = _call(lib.mb_op_mesh_backward_noalloc, x, x, w, 0)
    assert status == _lib.MB_ERR_INVALID
