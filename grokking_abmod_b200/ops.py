"""Op-level entry points over device buffers (torch CUDA tensors as plumbing).

``mesh_forward`` / ``mesh_backward`` wrap ``mb_op_mesh_forward`` /
``mb_op_mesh_backward``: one two-parent mesh stack, the per-op boundary of
the reference's ``gpt_mesh`` and ``gpt_mesh_gradient`` kernels
(src/gpt/gpu.rs:103-146, :1087-1149).
"""

import ctypes

from . import _lib
from ._lib import check


def _dev(t, name):
    if not (t.is_cuda and t.is_contiguous() and str(t.dtype) == "torch.float32"):
        raise ValueError(f"{name} must be a contiguous float32 CUDA tensor")
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def mesh_forward(x, weights, connectivity: int = 0):
    """y = stack(x); x [rows][width], weights [depth][width][2]."""
    import torch
    rows, width = x.shape
    depth = weights.shape[0]
    y = torch.empty_like(x)
    check(_lib.load().mb_op_mesh_forward(_dev(x, "x"), _dev(y, "y"), rows, width, depth, connectivity,
                                         _dev(weights, "weights"), _stream()))
    return y


def mesh_backward(x, dy, weights, connectivity: int = 0):
    """(dx, dweights) of a stack from its input x and output gradient dy."""
    import torch
    rows, width = x.shape
    depth = weights.shape[0]
    dx = torch.empty_like(x)
    dw = torch.empty_like(weights)
    check(_lib.load().mb_op_mesh_backward(_dev(x, "x"), _dev(dy, "dy"), _dev(dx, "dx"), _dev(dw, "dweights"), rows,
                                          width, depth, connectivity, _dev(weights, "weights"), _stream()))
    return dx, dw


def gemm_tf32x3(a, b, layout: int = 0):
    """FP32 GEMM via tcgen05 3xTF32, C [m][n] = A . B^T over k.  Layout bits:
    1 = b given [k][n] (else [n][k]); 2 = accepted, the same as 0 (A is always
    staged through tensor memory);
    4 = a given [k][m] (else [m][k]; not with 2)."""
    import torch
    m, k = (a.shape[1], a.shape[0]) if layout & 4 else a.shape
    n, k2 = (b.shape[1], b.shape[0]) if layout & 1 else b.shape
    if k != k2:
        raise ValueError("inner dimensions differ")
    c = torch.empty((m, n), dtype=torch.float32, device=a.device)
    status = torch.zeros(1, dtype=torch.int32, device=a.device)
    check(_lib.load().mb_op_gemm_tf32x3(_dev(a, "a"), _dev(b, "b"), _dev(c, "c"), m, n, k, layout,
                                        ctypes.c_void_p(status.data_ptr()), _stream()))
    if int(status.item()) != 0:
        raise RuntimeError("tensor-core completion wait timed out")
    return c
