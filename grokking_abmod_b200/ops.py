"""Op-level entry points over device buffers (torch CUDA tensors as plumbing).

``mesh_forward`` / ``mesh_backward`` wrap ``mb_op_mesh_forward`` /
``mb_op_mesh_backward``: one two-parent mesh stack, the per-op boundary of
the reference's ``gpt_mesh`` and ``gpt_mesh_gradient`` kernels
(src/gpt/gpu.rs:103-146, :1087-1149).  The other wrappers follow the
remaining ``mb_op_*`` entry points: RMSNorm (:65-94, :1035-1077), RoPE
(:175-208), causal attention (:381-779), XSA (:781-897), the tied head and
cross-entropy (:927-1021) and AdamW (:1369-1391).  Operands are [rows][width]
row-major float32 CUDA tensors; each call runs on torch's current stream.
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


def _u32(t, name):
    if not (t.is_cuda and t.is_contiguous() and str(t.dtype) in ("torch.int32", "torch.uint32")):
        raise ValueError(f"{name} must be a contiguous 32-bit integer CUDA tensor")
    return ctypes.c_void_p(t.data_ptr())


def _status(device):
    import torch
    return torch.zeros(1, dtype=torch.int32, device=device)


def _raise_status(status, what):
    code = int(status.item())
    if code:
        raise RuntimeError(f"{what}: device status {code}")


def rmsnorm_forward(x, heads: int = 1):
    """(y, inv): per-(row, head) RMSNorm and 1/rms [rows][heads]."""
    import torch
    rows, width = x.shape
    y = torch.empty_like(x)
    inv = torch.empty((rows, heads), dtype=torch.float32, device=x.device)
    check(_lib.load().mb_op_rmsnorm_forward(_dev(x, "x"), _dev(y, "y"), _dev(inv, "inv"), rows, width, heads,
                                            _stream()))
    return y, inv


def rmsnorm_backward(x, dy, heads: int = 1):
    import torch
    rows, width = x.shape
    dx = torch.empty_like(x)
    check(_lib.load().mb_op_rmsnorm_backward(_dev(x, "x"), _dev(dy, "dy"), _dev(dx, "dx"), rows, width, heads,
                                             _stream()))
    return dx


def rope(x, sequence: int, heads: int, inverse: bool = False):
    import torch
    rows, width = x.shape
    y = torch.empty_like(x)
    check(_lib.load().mb_op_rope(_dev(x, "x"), _dev(y, "y"), rows, sequence, width, heads, int(inverse), _stream()))
    return y


def attention_forward(q, k, v, sequence: int, heads: int):
    """(o, lse2): causal attention per head; lse2 [heads][rows] is the
    base-2 log-sum-exp of each row's scores scaled by log2(e) / sqrt(hd)."""
    import torch
    rows, width = q.shape
    o = torch.empty_like(q)
    lse = torch.empty((heads, rows), dtype=torch.float32, device=q.device)
    status = _status(q.device)
    check(_lib.load().mb_op_attn_forward(_dev(q, "q"), _dev(k, "k"), _dev(v, "v"), _dev(o, "o"), _dev(lse, "lse"),
                                         rows, sequence, width, heads, ctypes.c_void_p(status.data_ptr()), _stream()))
    _raise_status(status, "attention forward")
    return o, lse


def attention_backward(q, k, v, o, dout, lse, sequence: int, heads: int):
    import torch
    rows, width = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    status = _status(q.device)
    check(_lib.load().mb_op_attn_backward(_dev(q, "q"), _dev(k, "k"), _dev(v, "v"), _dev(o, "o"),
                                          _dev(dout, "dout"), _dev(lse, "lse"), _dev(dq, "dq"), _dev(dk, "dk"),
                                          _dev(dv, "dv"), rows, sequence, width, heads,
                                          ctypes.c_void_p(status.data_ptr()), _stream()))
    _raise_status(status, "attention backward")
    return dq, dk, dv


def xsa_forward(y, v, heads: int):
    import torch
    rows, width = y.shape
    z = torch.empty_like(y)
    check(_lib.load().mb_op_xsa_forward(_dev(y, "y"), _dev(v, "v"), _dev(z, "z"), rows, width, heads, _stream()))
    return z


def xsa_backward(y, v, dz, heads: int):
    import torch
    rows, width = y.shape
    dy, dv = torch.empty_like(y), torch.empty_like(v)
    check(_lib.load().mb_op_xsa_backward(_dev(y, "y"), _dev(v, "v"), _dev(dz, "dz"), _dev(dy, "dy"), _dev(dv, "dv"),
                                         rows, width, heads, _stream()))
    return dy, dv


def head_ce(h, embeddings, targets, backward: bool = True):
    """(logits, loss, dh, dembeddings) of the tied head and mean
    cross-entropy; dh and dembeddings are None without ``backward``."""
    import torch
    rows, width = h.shape
    vocab = embeddings.shape[0]
    logits = torch.empty((rows, vocab), dtype=torch.float32, device=h.device)
    loss = torch.empty(1, dtype=torch.float64, device=h.device)
    dh = torch.empty_like(h) if backward else None
    de = torch.empty_like(embeddings) if backward else None
    status = _status(h.device)
    check(_lib.load().mb_op_head_ce(_dev(h, "h"), _dev(embeddings, "embeddings"), _u32(targets, "targets"), rows,
                                    width, vocab, _dev(logits, "logits"), ctypes.c_void_p(loss.data_ptr()),
                                    _dev(dh, "dh") if backward else None,
                                    _dev(de, "dembeddings") if backward else None,
                                    ctypes.c_void_p(status.data_ptr()), _stream()))
    _raise_status(status, "head cross-entropy")
    return logits, float(loss.item()), dh, de


def adamw(weights, m, v, gradient, options, step: int):
    """One AdamW update of float32 CUDA tensors in place (update number ``step``)."""
    o = options.to_c()
    check(_lib.load().mb_op_adamw(_dev(weights, "weights"), _dev(m, "m"), _dev(v, "v"), _dev(gradient, "gradient"),
                                  weights.numel(), ctypes.byref(o), step, _stream()))
