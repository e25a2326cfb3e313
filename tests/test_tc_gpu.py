"""tcgen05 3xTF32 GEMM (the tensor-core building blocks) against f64 numpy:
K-major and K-outer (transposed) A and B operands, including strides that
rule out a TMA tensor map (the cp.async staging path); A is staged through
tensor memory."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layout", [0, 1, 2, 3, 4, 5])
@pytest.mark.parametrize("m,n,k", [(128, 64, 32), (300, 130, 200), (4656, 128, 97), (97, 384, 194), (1, 1, 1)])
def test_gemm_tf32x3_is_fp32_accurate(m, n, k, layout):
    import torch

    from grokking_abmod_b200 import ops
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    bb = np.ascontiguousarray(b.T) if layout & 1 else b
    aa = np.ascontiguousarray(a.T) if layout & 4 else a
    c = ops.gemm_tf32x3(torch.from_numpy(aa).cuda(), torch.from_numpy(bb).cuda(), layout).cpu().numpy()
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    scale = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64).T
    # FP32-level accuracy: a plain TF32 product would miss this by ~1000x.
    err = np.abs(c - ref) / (scale + 1e-30)
    assert err.max() <= 2e-6, (err.max(), np.unravel_index(err.argmax(), err.shape))


@pytest.mark.parametrize("lost_block", [0, 3])
def test_gemm_wait_that_gives_up_reports_and_leaves_the_context_usable(lost_block):
    """A K block whose hand-over to the MMA warp never arrives: the bounded
    waits give up (short limit), every CTA drains its copies, skips its
    epilogue and frees its tensor memory, the status flag reads 1, and a
    normal GEMM right after it on the same stream is still FP32-exact."""
    import ctypes

    import torch

    from grokking_abmod_b200 import _lib, ops
    lib = _lib.load()
    m, n, k = 256, 128, 256
    rng = np.random.default_rng(5)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    c = torch.full((m, n), 7.0, dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.mb_test_gemm_lost_arrival(ctypes.c_void_p(da.data_ptr()), ctypes.c_void_p(db.data_ptr()),
                                       ctypes.c_void_p(c.data_ptr()), m, n, k, lost_block, 1 << 12,
                                       ctypes.c_void_p(status.data_ptr()), stream)
    assert rc == _lib.MB_OK
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    # Every CTA skipped its epilogue: the output is untouched.
    assert bool((c == 7.0).all())
    # A K block that does not exist is rejected on the host.
    assert lib.mb_test_gemm_lost_arrival(ctypes.c_void_p(da.data_ptr()), ctypes.c_void_p(db.data_ptr()),
                                         ctypes.c_void_p(c.data_ptr()), m, n, k, 8, 1 << 12,
                                         ctypes.c_void_p(status.data_ptr()), stream) == _lib.MB_ERR_INVALID
    out = ops.gemm_tf32x3(da, db, 0).cpu().numpy()
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    scale = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64).T
    assert (np.abs(out - ref) / scale).max() <= 2e-6
