"""Mesh GPT on the GPU through the C ABI, checked against the f64 oracle.

Tolerances: the reference's own verifier bound 5e-4*(1+|ref|) on every logit,
loss and gradient (src/bin/mesh-gpt.rs:335-383) and, tighter, the north-star
bounds: loss within 1e-5 relative, gradients within 1e-4 of the largest
gradient magnitude.  AdamW updates are checked against the f32 host optimizer
applied to the GPU's own gradients at 1e-6*(1+|p|) (src/bin/mesh-gpt.rs:448-481).
"""

import json
import os

import numpy as np
import pytest

from grokking_abmod_b200 import AdamWOptions, GptConfig, IGNORE_TARGET, MeshError, MeshGpt
from oracle import gpt_config as ocfg
from oracle.data import EquationDataset, EquationSampler, warmed_learning_rate
from oracle.gpt_ref import ReferenceGpt, adamw_step

pytestmark = pytest.mark.gpu

PINS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_pins.json")))

CASES = [
    # (config kwargs, sequences, sequence length)
    (dict(vocab_size=9, context=3, width=64, heads=8, layers=1, attention_mesh_depth=1, ffn_mesh_depth=1), 4, 3),
    (dict(vocab_size=9, context=3, width=128, heads=4, layers=2, attention_mesh_depth=2, ffn_mesh_depth=2), 5, 3),
    (dict(vocab_size=99, context=4, width=128, heads=4, layers=2), 40, 4),
    (dict(vocab_size=17, context=8, width=128, heads=4, layers=1, connectivity="butterfly"), 6, 8),
    (dict(vocab_size=64, context=70, width=256, heads=4, layers=2), 3, 70),
    (dict(vocab_size=64, context=130, width=512, heads=8, layers=1), 2, 130),
    (dict(vocab_size=33, context=64, width=384, heads=6, layers=1, attention_mesh_depth=2, ffn_mesh_depth=3), 2, 64),
    (dict(vocab_size=17, context=8, width=128, heads=4, layers=1, embedding="table"), 6, 8),
    (dict(vocab_size=64, context=70, width=256, heads=4, layers=2, embedding="table", connectivity="butterfly"), 3,
     70),
    # head width 128: a head spans two warps of the row kernels (QK-Norm, XSA
    # sums and the RoPE partner cross warps); FP32 SIMT attention
    (dict(vocab_size=33, context=40, width=256, heads=2, layers=2), 3, 40),
    (dict(vocab_size=64, context=70, width=512, heads=4, layers=1), 2, 70),
    (dict(vocab_size=17, context=16, width=128, heads=1, layers=1, connectivity="butterfly"), 4, 16),
]


def _pair(kw, seed=7):
    oc = ocfg.GptConfig(**kw)
    pc = GptConfig(**kw)
    return ReferenceGpt(oc, seed=seed), MeshGpt(0, pc, seed)


def _batch(cfg, seqs, seq, seed=0, answer_only=False):
    rng = np.random.default_rng(seed)
    x = rng.integers(0, cfg.vocab_size, seqs * seq).astype(np.uint32)
    y = rng.integers(0, cfg.vocab_size, seqs * seq).astype(np.uint32)
    if answer_only:
        y[np.arange(y.size) % seq != seq - 1] = IGNORE_TARGET
    return x, y


def _close(name, ref, got, tol=5e-4):
    ref, got = np.asarray(ref, np.float64), np.asarray(got, np.float64)
    err = np.abs(ref - got) - tol * (1 + np.abs(ref))
    assert np.all(np.isfinite(got)), name
    assert err.max() <= 0, f"{name}: worst excess {err.max():.3e}"


@pytest.mark.parametrize("case", range(len(CASES)))
def test_logits_loss_gradients_match_oracle(case):
    kw, seqs, seq = CASES[case]
    ref, gpu = _pair(kw)
    assert gpu.parameters().tobytes() == ref.parameters.tobytes()
    _close("embeddings", ref.token_embeddings(), gpu.token_embeddings())
    for answer_only in (False, True):
        x, y = _batch(ref.config, seqs, seq, seed=case, answer_only=answer_only)
        _close("logits", ref.logits(x, seq), gpu.logits(x, seq))
        rl, rg = ref.loss_and_gradient(x, y, seq)
        gl, gg = gpu.loss_and_gradient(x, y, seq)
        assert abs(rl - gl) <= 1e-5 * abs(rl), (rl, gl)
        _close("gradients", rg, gg)
        assert np.abs(rg - gg).max() <= 1e-4 * np.abs(rg).max(), np.abs(rg - gg).max() / np.abs(rg).max()
        assert abs(gpu.cross_entropy(x, y, seq) - rl) <= 1e-5 * abs(rl)
    gpu.close()


def test_hidden_states_and_causality():
    kw = dict(vocab_size=9, context=8, width=128, heads=4, layers=2)
    ref, gpu = _pair(kw, seed=11)
    x = np.array([0, 1, 2, 3, 1, 2, 3, 4], dtype=np.uint32)
    _close("hidden", ref.hidden_states(x, 4), gpu.hidden_states(x, 4))
    a = gpu.logits(x, 4)
    b = gpu.logits(np.array([0, 1, 4, 0, 4, 4, 4, 4], dtype=np.uint32), 4)
    assert np.array_equal(a[:2], b[:2]), "causal mask leaked future tokens"
    assert np.array_equal(a[:2], gpu.logits(np.array([0, 1], dtype=np.uint32), 2))


def test_gradients_are_bitwise_repeatable():
    kw = dict(vocab_size=64, context=64, width=256, heads=4, layers=2)
    _, gpu = _pair(kw)
    x, y = _batch(GptConfig(**kw), 8, 64, seed=3)
    l1, g1 = gpu.loss_and_gradient(x, y, 64)
    l2, g2 = gpu.loss_and_gradient(x, y, 64)
    assert l1 == l2 and g1.tobytes() == g2.tobytes()


def test_workspace_capacity():
    """set_workspace_capacity / workspace_capacity (src/gpt/gpu.rs:1779-1791;
    the reference's CLI checks 0 and 4 are refused, src/bin/mesh-gpt.rs:600-606):
    results do not depend on which batch shapes stay cached."""
    kw = dict(vocab_size=64, context=64, width=256, heads=4, layers=2)
    _, gpu = _pair(kw)
    assert gpu.workspace_capacity() == 1
    for bad in (0, 4):
        with pytest.raises(MeshError):
            gpu.set_workspace_capacity(bad)
    assert gpu.workspace_capacity() == 1
    xa, ya = _batch(GptConfig(**kw), 4, 64, seed=3)
    xb, yb = _batch(GptConfig(**kw), 2, 32, seed=4)
    want_a, want_b = gpu.loss_and_gradient(xa, ya, 64), gpu.loss_and_gradient(xb, yb, 32)
    for cap in (3, 2, 1):
        gpu.set_workspace_capacity(cap)
        assert gpu.workspace_capacity() == cap
        for _ in range(2):
            for (x, y, s), want in (((xa, ya, 64), want_a), ((xb, yb, 32), want_b)):
                loss, grad = gpu.loss_and_gradient(x, y, s)
                assert loss == want[0] and grad.tobytes() == want[1].tobytes()


@pytest.mark.parametrize("opt", [AdamWOptions(learning_rate=0.002, weight_decay=0.01),
                                 AdamWOptions(learning_rate=0.001, weight_decay=1.0, beta2=0.98)])
def test_adamw_matches_f32_host_optimizer_and_resets(opt):
    kw = dict(vocab_size=5, context=4, width=64, heads=2, layers=1, attention_mesh_depth=2, ffn_mesh_depth=2)
    ref, gpu = _pair(kw)
    x = np.array([0, 1, 3, 2, 4, 1], dtype=np.uint32)
    y = np.array([1, 3, 2, 4, 1, 0], dtype=np.uint32)
    p = ref.parameters.copy()
    m, v = np.zeros_like(p), np.zeros_like(p)
    b1 = b2 = np.float32(1.0)
    first = None
    for step in range(1, 4):
        p = gpu.parameters()
        _, g = gpu.loss_and_gradient(x, y, 3)
        b1, b2 = np.float32(b1 * np.float32(opt.beta1)), np.float32(b2 * np.float32(opt.beta2))
        adamw_step(p, m, v, g, step, opt.learning_rate, opt.weight_decay, opt.beta1, opt.beta2, opt.epsilon, (b1, b2))
        if step == 1:
            first = p.copy()
        gpu.train_batch_with_optimizer(x, y, 3, opt)
        _close("adamw", p, gpu.parameters(), tol=1e-6)
    gpu.set_parameters(ref.parameters)
    gpu.train_batch_with_optimizer(x, y, 3, opt)
    _close("adamw reset", first, gpu.parameters(), tol=1e-6)


def test_device_batches_match_host_batches():
    import torch
    kw = dict(vocab_size=64, context=32, width=128, heads=4, layers=2)
    _, a = _pair(kw)
    _, b = _pair(kw)
    x, y = _batch(GptConfig(**kw), 16, 32, seed=5)
    opt = AdamWOptions(learning_rate=3e-4, weight_decay=0.1)
    dx = torch.from_numpy(x.astype(np.int32)).cuda()
    dy = torch.from_numpy(y.astype(np.int32)).cuda()
    dl = torch.zeros(1, dtype=torch.float64, device="cuda")
    torch.cuda.synchronize()
    for _ in range(3):
        la = a.train_batch_with_optimizer(x, y, 32, opt)
        b.train_batch_device(dx.data_ptr(), dy.data_ptr(), x.size, 32, opt, dl.data_ptr())
        b.check()
        assert la == float(dl.item())
    assert a.parameters().tobytes() == b.parameters().tobytes()
    bad = torch.full_like(dx, 64)
    b.train_batch_device(bad.data_ptr(), dy.data_ptr(), x.size, 32, opt, 0)
    with pytest.raises(MeshError):
        b.check()


def test_invalid_batches_and_parameters_are_rejected():
    kw = dict(vocab_size=5, context=4, width=64, heads=2, layers=1)
    _, gpu = _pair(kw)
    with pytest.raises(MeshError):
        gpu.logits([], 1)
    with pytest.raises(MeshError):
        gpu.logits([5], 1)
    with pytest.raises(MeshError):
        gpu.logits([0], 0)
    with pytest.raises(MeshError):
        gpu.logits([0, 1, 2], 2)
    with pytest.raises(MeshError):
        gpu.loss_and_gradient([0], [IGNORE_TARGET], 1)
    with pytest.raises(MeshError):
        gpu.loss_and_gradient([0, 1], [9, 9], 2)
    with pytest.raises(MeshError):
        gpu.set_parameters([0.0])
    bad = gpu.parameters()
    bad[3] = np.nan
    with pytest.raises(MeshError):
        gpu.set_parameters(bad)
    with pytest.raises(MeshError):
        gpu.train_batch_with_optimizer([0, 1], [1, 2], 2, AdamWOptions(beta1=1.0))


def test_zero_embeddings_give_zero_logits():
    kw = dict(vocab_size=9, context=4, width=64, heads=4, layers=1, attention_mesh_depth=2, ffn_mesh_depth=2)
    _, gpu = _pair(kw)
    p = np.full(gpu.parameter_count(), 0.5, dtype=np.float32)
    p[:2 * 64 * 2] = 0.0
    gpu.set_parameters(p)
    assert np.all(gpu.logits(np.arange(8) % 9, 4) == 0.0)


def test_grok_epoch_reproduces_archived_reference_run():
    """One mod-97 epoch through the GPU path reproduces the reference's archived
    f32 CUDA run (train CE 7.419670094 -> 6.532873894)."""
    pin = PINS["grok_epoch"]
    c = pin["config"]
    ds = EquationDataset(c["modulus"], c["operation"], c["train_fraction"], c["seed"])
    cfg = GptConfig(vocab_size=c["vocab_size"], context=4, width=c["width"], heads=c["heads"], layers=c["layers"])
    gpu = MeshGpt(0, cfg, c["seed"])

    def evaluate(val):
        x, y = ds.batch(val, range(len(ds.split(val))))
        logits = gpu.logits(x, 4).astype(np.float64)[3::4]
        t = y[3::4].astype(np.int64)
        m = logits.max(-1)
        lse = np.log(np.exp(logits - m[:, None]).sum(-1)) + m
        return float((lse - logits[np.arange(len(t)), t]).mean())

    got = [evaluate(False), evaluate(True)]
    sampler = EquationSampler(len(ds.training), c["seed"])
    for step in range(1, c["steps"] + 1):
        x, y = ds.batch(False, sampler.sample(c["batch"]))
        lr = float(warmed_learning_rate(c["learning_rate"], step))
        gpu.train_batch_with_optimizer(x, y, 4, AdamWOptions(learning_rate=lr, weight_decay=c["weight_decay"],
                                                             beta1=c["beta1"], beta2=c["beta2"],
                                                             epsilon=c["epsilon"]))
    got += [evaluate(False), evaluate(True)]
    want = [pin["train_cross_entropy"][0], pin["validation_cross_entropy"][0],
            pin["train_cross_entropy"][1], pin["validation_cross_entropy"][1]]
    for g, w in zip(got, want):
        assert abs(g - w) <= 2e-6 * abs(w), (got, want)


def test_benchmark_shape_step_is_finite_and_learns():
    """Size-independent properties at the cfg3 shape (W256 L4 H4 T256 B64):
    finite loss, identical reruns, and a decreasing loss over a few steps."""
    from grokking_abmod_b200.data import zipf_batch
    cfg = GptConfig(vocab_size=64, context=256, width=256, heads=4, layers=4)
    gpu = MeshGpt(0, cfg, 7)
    x, y = zipf_batch(7, 0, 0, 64, 256)
    opt = AdamWOptions(learning_rate=3e-4, weight_decay=0.1)
    losses = [gpu.train_batch_with_optimizer(x, y, 256, opt) for _ in range(6)]
    assert all(np.isfinite(losses)) and losses[-1] < losses[0]
    assert np.isfinite(gpu.parameters()).all()


def _adamw_first_step_close(name, params, ref_grad, got, opt, grad_tol):
    """Parameters after one AdamW step from `params` against the f32 host
    optimizer applied to the oracle's gradient.  The first step moves each
    weight by lr * g / (|g| + eps) (+ decay), so a gradient error d changes
    it by at most lr * min(2, 2 d / |g|): the bound is tight where gradients
    are well determined and a full step where they sit at the error level."""
    want, m, v = params.copy(), np.zeros_like(params), np.zeros_like(params)
    adamw_step(want, m, v, ref_grad, 1, opt.learning_rate, opt.weight_decay, opt.beta1, opt.beta2, opt.epsilon,
               (np.float32(opt.beta1), np.float32(opt.beta2)))
    g = np.abs(ref_grad)
    bound = opt.learning_rate * np.minimum(2.0, 2.0 * grad_tol / np.maximum(g, 1e-30)) + 1e-6 * (1 + np.abs(want))
    err = np.abs(got.astype(np.float64) - want)
    assert np.all(err <= bound), f"{name}: worst excess {(err - bound).max():.3e}"
    # and most weights move by the oracle's step to FP32 accuracy
    assert np.mean(err <= 1e-6 * (1 + np.abs(want))) > 0.99


@pytest.mark.parametrize("name,kw,seqs", [
    # BASELINE configs[4]'s model and context (one 1024-token sequence; the
    # timed step runs 32 of them, which are independent until the loss mean)
    ("cfg4", dict(vocab_size=64, context=1024, width=512, heads=8, layers=8), 1),
    # BASELINE configs[3]'s model and context, 4 of its 64 sequences
    ("cfg3", dict(vocab_size=64, context=256, width=256, heads=4, layers=4), 4),
])
def test_timed_shapes_match_oracle(name, kw, seqs):
    """Loss, every gradient and one AdamW step at the shapes the bench times,
    on its seeded Zipf(1.1) tokens: the attention's long-row paths (1024-key
    online softmax, the 16-tile causal work order) run here."""
    from grokking_abmod_b200.data import zipf_batch
    ref, gpu = _pair(kw)
    T = kw["context"]
    x, y = zipf_batch(7, 0, 0, seqs, T)
    rl, rg = ref.loss_and_gradient(x, y, T)
    gl, gg = gpu.loss_and_gradient(x, y, T)
    assert abs(rl - gl) <= 1e-5 * abs(rl), (rl, gl)
    assert np.abs(rg - gg).max() <= 1e-4 * np.abs(rg).max(), np.abs(rg - gg).max() / np.abs(rg).max()
    _close("gradients", rg, gg)
    opt = AdamWOptions(learning_rate=3e-4, weight_decay=0.1)
    params = gpu.parameters()
    assert gpu.train_batch_with_optimizer(x, y, T, opt) == gl
    _adamw_first_step_close(name, params, rg, gpu.parameters(), opt, 1e-4 * np.abs(rg).max())
    gpu.close()
