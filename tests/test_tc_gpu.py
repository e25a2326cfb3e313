"""tcgen05 3xTF32 GEMM (the tensor-core building block) against f64 numpy."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k", [(128, 64, 32), (300, 130, 200), (4656, 128, 97), (97, 384, 194), (1, 1, 1)])
def test_gemm_tf32x3_is_fp32_accurate(m, n, k):
    import torch

    from grokking_abmod_b200 import ops
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    c = ops.gemm_tf32x3(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    scale = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64).T
    # FP32-level accuracy: a plain TF32 product would miss this by ~1000x.
    assert np.all(np.abs(c - ref) <= 2e-6 * scale + 1e-30), np.max(np.abs(c - ref) / (scale + 1e-30))
