"""Op-level mesh stack entry points against the f64 oracle (GPU)."""

import numpy as np
import pytest

from oracle.gpt_ref import mesh_backward as ref_backward
from oracle.gpt_ref import mesh_forward as ref_forward

pytestmark = pytest.mark.gpu

CASES = [(64, 1, 0, 5), (128, 4, 0, 1000), (256, 6, 1, 333), (384, 3, 0, 70), (512, 4, 0, 4097), (512, 6, 1, 64)]


def _data(width, depth, rows, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, width)).astype(np.float32)
    dy = rng.standard_normal((rows, width)).astype(np.float32)
    w = np.empty((depth, width, 2), dtype=np.float32)
    w[..., 0] = 0.7 + 0.2 * (rng.random((depth, width)) - 0.5)
    w[..., 1] = 0.4 * (rng.random((depth, width)) - 0.5)
    return x, dy, w


def _strides(width, depth, conn):
    if conn == 0:
        return [1] * depth
    return [1 << (l % (width.bit_length() - 1)) for l in range(depth)]


@pytest.mark.parametrize("case", CASES)
def test_mesh_stack_matches_oracle(case):
    import torch

    from grokking_abmod_b200 import ops
    width, depth, conn, rows = case
    x, dy, w = _data(width, depth, rows, width + depth)
    s = _strides(width, depth, conn)
    acts = ref_forward(x.astype(np.float64), w.astype(np.float64), s)
    rdx, rdw = ref_backward(acts, w.astype(np.float64), s, dy.astype(np.float64))
    tx, tdy, tw = (torch.from_numpy(a).cuda() for a in (x, dy, w))
    y = ops.mesh_forward(tx, tw, conn).cpu().numpy()
    dx, dw = ops.mesh_backward(tx, tdy, tw, conn)
    dx, dw = dx.cpu().numpy(), dw.cpu().numpy()
    assert np.abs(y - acts[-1]).max() <= 1e-5 * (1 + np.abs(acts[-1]).max())
    assert np.abs(dx - rdx).max() <= 1e-5 * (1 + np.abs(rdx).max())
    assert np.abs(dw - rdw).max() <= 1e-4 * np.abs(rdw).max()
    dx2, dw2 = ops.mesh_backward(tx, tdy, tw, conn)
    assert np.array_equal(dx2.cpu().numpy(), dx) and np.array_equal(dw2.cpu().numpy(), dw)


def test_mesh_ops_reject_bad_shapes():
    import torch

    from grokking_abmod_b200 import MeshError, ops
    x = torch.zeros((4, 100), device="cuda")
    w = torch.zeros((2, 100, 2), device="cuda")
    with pytest.raises(MeshError):
        ops.mesh_forward(x, w)
    x = torch.zeros((4, 128), device="cuda")
    w = torch.zeros((17, 128, 2), device="cuda")
    with pytest.raises(MeshError):
        ops.mesh_backward(x, x, w)
