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
