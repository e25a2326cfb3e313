"""Per-op entry points of the Mesh GPT operators (mb_op_*) against the f64
oracle's operators (oracle/gpt_ref.py), through the C ABI.

Tolerances: elementwise 1e-5 * (1 + |ref|) for the row operators (norms,
RoPE, XSA: a handful of f32 roundings); attention within 1e-4 of the largest
reference magnitude (the north-star gradient bound) and 5e-4 * (1 + |ref|)
elementwise (the reference verifier's bound, src/bin/mesh-gpt.rs:335-383);
the head's loss within 1e-5 relative; AdamW within 1e-6 * (1 + |p|) of the
f32 host optimizer (src/bin/mesh-gpt.rs:448-481)."""

import numpy as np
import pytest

from grokking_abmod_b200 import AdamWOptions, Context, GptConfig, IGNORE_TARGET, MeshGpt, ops
from oracle import gpt_ref as ref

pytestmark = pytest.mark.gpu


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def _np(t):
    return t.detach().cpu().numpy().astype(np.float64)


def _close(name, want, got, tol):
    want, got = np.asarray(want, np.float64), np.asarray(got, np.float64)
    assert np.all(np.isfinite(got)), name
    err = np.abs(got - want) - tol * (1 + np.abs(want))
    assert err.max() <= 0, f"{name}: worst excess {err.max():.3e}"


def _rows(rows, width, seed, scale=1.0):
    return np.random.default_rng(seed).normal(0.0, scale, (rows, width)).astype(np.float32)


@pytest.mark.parametrize("rows,width,heads", [(1000, 512, 1), (777, 512, 8), (64, 256, 4), (33, 96, 3), (8, 4, 2)])
def test_rmsnorm_forward_and_backward(rows, width, heads):
    x, dy = _rows(rows, width, 1, 2.0), _rows(rows, width, 2)
    y, inv = ops.rmsnorm_forward(_t(x), heads)
    want, winv = ref.rmsnorm(x.astype(np.float64), heads)
    _close("rmsnorm", want, _np(y), 1e-5)
    _close("inv", winv, _np(inv), 1e-5)
    dx = ops.rmsnorm_backward(_t(x), _t(dy), heads)
    _close("rmsnorm backward", ref.rmsnorm_backward(want, winv, dy.astype(np.float64), heads), _np(dx), 1e-5)


@pytest.mark.parametrize("rows,seq,width,heads", [(2048, 1024, 512, 8), (130, 65, 256, 4), (12, 3, 8, 2)])
def test_rope_and_its_inverse(rows, seq, width, heads):
    x = _rows(rows, width, 3)
    y = ops.rope(_t(x), seq, heads)
    _close("rope", ref.rope(x.astype(np.float64), seq, heads), _np(y), 1e-5)
    back = ops.rope(y, seq, heads, inverse=True)
    _close("rope inverse", x, _np(back), 1e-5)


@pytest.mark.parametrize("rows,width,heads", [(1024, 512, 8), (50, 128, 4), (7, 64, 1)])
def test_xsa_forward_and_backward(rows, width, heads):
    y, v, dz = _rows(rows, width, 4), _rows(rows, width, 5), _rows(rows, width, 6)
    v[3, :width // heads] = 0.0  # a head with |v| below the floor
    z = ops.xsa_forward(_t(y), _t(v), heads)
    y64, v64 = y.astype(np.float64), v.astype(np.float64)
    _close("xsa", ref.exclusive_forward(y64, v64, heads), _np(z), 1e-5)
    dy, dv = ops.xsa_backward(_t(y), _t(v), _t(dz), heads)
    wdy, wdv = ref.exclusive_backward(y64, v64, dz.astype(np.float64), heads)
    _close("xsa dy", wdy, _np(dy), 1e-5)
    _close("xsa dv", wdv, _np(dv), 1e-5)


def _lse2(q, k, seq, heads):
    """Base-2 log-sum-exp of each row's causal scores, [heads][rows]."""
    n, w = q.shape
    hd = w // heads
    out = np.empty((heads, n))
    mask = np.tril(np.ones((seq, seq), dtype=bool))
    for s0 in range(0, n, seq):
        for h in range(heads):
            qs, ks = q[s0:s0 + seq, h * hd:(h + 1) * hd], k[s0:s0 + seq, h * hd:(h + 1) * hd]
            sc = np.where(mask, qs @ ks.T / np.sqrt(hd), -np.inf)
            m = sc.max(-1)
            out[h, s0:s0 + seq] = (np.log(np.exp(sc - m[:, None]).sum(-1)) + m) / np.log(2.0)
    return out


def _attention_case(rows, seq, width, heads, large):
    rng = np.random.default_rng(rows + seq)
    q, k, v = (rng.normal(0.0, 1.0, (rows, width)) for _ in range(3))
    if large:
        # Scores that climb along the keys, from about -6 to +6: every query
        # is aligned with a direction whose weight in the keys grows with the
        # key's position, so a late row's running maximum rises by more than
        # 2^8 over its first key tile and the online softmax must rescale.
        hd = width // heads
        alpha = np.sqrt(6.0 / np.sqrt(hd))
        a = rng.normal(0.0, 1.0, (heads, hd))
        pos = 2.0 * (np.arange(rows) % seq) / (seq - 1) - 1.0
        q, k = 0.3 * q, 0.3 * k
        for h in range(heads):
            q[:, h * hd:(h + 1) * hd] += alpha * a[h]
            k[:, h * hd:(h + 1) * hd] += alpha * pos[:, None] * a[h]
    return [x.astype(np.float32) for x in (q, k, v)] + [rng.normal(0.0, 1e-3, (rows, width)).astype(np.float32)]


def _max_growth(q, k, seq, heads):
    """log2 growth of the last row's running score maximum after its first
    64 keys, per head, in the first sequence."""
    hd = q.shape[1] // heads
    out = []
    for h in range(heads):
        s = k[:seq, h * hd:(h + 1) * hd] @ q[seq - 1, h * hd:(h + 1) * hd] / np.sqrt(hd)
        out.append((s.max() - s[:64].max()) / np.log(2.0))
    return np.array(out)


@pytest.mark.parametrize("rows,seq,width,heads,large", [
    (2048, 1024, 512, 8, False),  # the cfg4 shape: hd 64, two 1024-token sequences
    (1024, 1024, 512, 8, True),   # large, growing logits: the lazy-rescale path
    (768, 256, 256, 4, False),    # the cfg3 shape
    (390, 130, 128, 4, True),     # hd 32, ragged tiles
    (96, 32, 64, 8, False),       # hd 8 on the FP32 SIMT kernels
    (256, 128, 256, 2, False),    # hd 128 on the FP32 SIMT kernels
])
def test_attention_forward_and_backward(rows, seq, width, heads, large):
    q, k, v, do = _attention_case(rows, seq, width, heads, large)
    o, lse = ops.attention_forward(_t(q), _t(k), _t(v), seq, heads)
    q64, k64, v64 = (x.astype(np.float64) for x in (q, k, v))
    want, probs = ref.attention_forward(q64, k64, v64, seq, heads)
    got = _np(o)
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()
    _close("attention", want, got, 5e-4)
    wlse = _lse2(q64, k64, seq, heads)
    if large:
        assert (_max_growth(q64, k64, seq, heads) > 8).any(), "case lacks growing maxima"
    _close("lse", wlse, _np(lse), 1e-5)
    dq, dk, dv = ops.attention_backward(_t(q), _t(k), _t(v), o, _t(do), lse, seq, heads)
    wq, wk, wv = ref.attention_backward(q64, k64, v64, probs, do.astype(np.float64), seq, heads)
    for name, w, g in (("dq", wq, dq), ("dk", wk, dk), ("dv", wv, dv)):
        g = _np(g)
        assert np.abs(g - w).max() <= 1e-4 * np.abs(w).max(), (name, np.abs(g - w).max() / np.abs(w).max())
        _close(name, w, g, 5e-4)


def test_head_cross_entropy():
    rows, width, vocab = 600, 256, 64
    rng = np.random.default_rng(8)
    h = _rows(rows, width, 9, 3.0)
    emb = rng.normal(0.0, 1.0, (vocab, width)).astype(np.float32)
    targets = rng.integers(0, vocab, rows).astype(np.uint32)
    targets[::3] = IGNORE_TARGET
    import torch
    tt = torch.from_numpy(targets.view(np.int32)).cuda()
    logits, loss, dh, de = ops.head_ce(_t(h), _t(emb), tt)
    h64, e64 = h.astype(np.float64), emb.astype(np.float64)
    nf, inv = ref.rmsnorm(h64, 1)
    wl = nf @ e64.T
    # the 3xTF32 GEMM's bound: 2e-6 of the sum of the products' magnitudes
    assert np.all(np.abs(_np(logits) - wl) <= 2e-6 * (np.abs(nf) @ np.abs(e64).T))
    rows_ce, sup = ref.ReferenceGpt.row_losses(wl, targets)
    count = sup.sum()
    assert abs(loss - rows_ce.sum() / count) <= 1e-5 * abs(rows_ce.sum() / count)
    p = np.exp(wl - wl.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    t = np.where(sup, targets, 0).astype(np.int64)
    p[np.arange(rows), t] -= 1.0
    dlog = np.where(sup[:, None], p / count, 0.0)
    wdh = ref.rmsnorm_backward(nf, inv, dlog @ e64, 1)
    wde = dlog.T @ nf
    for name, w, g in (("dh", wdh, dh), ("dE", wde, de)):
        g = _np(g)
        assert np.abs(g - w).max() <= 1e-4 * np.abs(w).max(), name
    # forward only, and the status for a target outside the vocabulary
    _, loss2, none_dh, none_de = ops.head_ce(_t(h), _t(emb), tt, backward=False)
    assert loss2 == loss and none_dh is None and none_de is None
    bad = tt.clone()
    bad[5] = vocab
    with pytest.raises(RuntimeError, match="status 2"):
        ops.head_ce(_t(h), _t(emb), bad)


def test_adamw_matches_f32_host_optimizer():
    n = 10007
    rng = np.random.default_rng(10)
    p = rng.normal(0.0, 1.0, n).astype(np.float32)
    w, m, v = _t(p), _t(np.zeros(n)), _t(np.zeros(n))
    hp, hm, hv = p.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    opt = AdamWOptions(learning_rate=1e-3, weight_decay=0.1, beta1=0.9, beta2=0.98)
    b1 = b2 = np.float32(1.0)
    for step in range(1, 4):
        g = rng.normal(0.0, 1e-2, n).astype(np.float32)
        ops.adamw(w, m, v, _t(g), opt, step)
        b1, b2 = np.float32(b1 * np.float32(opt.beta1)), np.float32(b2 * np.float32(opt.beta2))
        ref.adamw_step(hp, hm, hv, g, step, opt.learning_rate, opt.weight_decay, opt.beta1, opt.beta2, opt.epsilon,
                       (b1, b2))
        _close("adamw", hp, _np(w), 1e-6)


def test_invalid_op_arguments_are_rejected():
    from grokking_abmod_b200 import MeshError, UnsupportedShape
    x = _t(np.zeros((12, 8)))
    with pytest.raises(MeshError):
        ops.rmsnorm_forward(x, 3)  # heads must divide the width
    with pytest.raises(MeshError):
        ops.rope(x, 5, 2)  # rows must hold whole sequences
    with pytest.raises(UnsupportedShape):
        big = _t(np.zeros((4, 512)))
        ops.attention_forward(big, big, big, 4, 2)  # head width 256


def test_models_share_a_context_stream():
    kw = dict(vocab_size=17, context=8, width=128, heads=4, layers=1)
    ctx = Context(0)
    a = MeshGpt(ctx, GptConfig(**kw), 7)
    b = MeshGpt(0, GptConfig(**kw), 7)
    assert a.stream() == ctx.stream and b.stream() != ctx.stream
    x = np.arange(32, dtype=np.uint32) % 17
    la, ga = a.loss_and_gradient(x, x[::-1].copy(), 8)
    lb, gb = b.loss_and_gradient(x, x[::-1].copy(), 8)
    assert la == lb and ga.tobytes() == gb.tobytes()
    a.close()
    b.close()
    ctx.close()
