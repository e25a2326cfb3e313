"""The CPU oracle against the reference's own known answers (no GPU).

Every check here pins ``oracle/`` to a constant that the reference's unit tests
or archived runs publish (``tests/golden/reference_pins.json``), or to the
reference's differentiation rules through the tape port."""

import json
import math
import os

import numpy as np
import pytest

from oracle.data import (IGNORE_TARGET, EquationDataset, EquationSampler, residue_permutation,
                         warmed_learning_rate, zipf_batch, zipf_cdf)
from oracle.gpt_config import GptConfig, Layout, parameter_count, token_codes
from oracle.gpt_ref import (ReferenceGpt, adamw_step, exclusive_backward, exclusive_forward,
                            rmsnorm, rmsnorm_backward, rope)
from oracle.rng import Random
from oracle.tape import tape_loss_and_gradient

PINS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_pins.json")))
TINY = GptConfig(vocab_size=5, context=4, width=4, heads=2, layers=1,
                 attention_mesh_depth=2, ffn_mesh_depth=2)


def test_parameter_counts_match_reference_and_configs():
    assert parameter_count(GptConfig()) == PINS["default_parameter_count"]["value"]
    for vocab in (2, 26, 256, 65536):
        layout = Layout(GptConfig(vocab_size=vocab))
        assert layout.count() == 3072 and len(layout.groups) == 1 + 5 * 2
    # BASELINE shapes: P = 2W(A + L(4A+F))
    assert parameter_count(GptConfig(vocab_size=64, context=256, width=256, heads=4, layers=4)) == 47104
    assert parameter_count(GptConfig(vocab_size=64, context=1024, width=512, heads=8, layers=8)) == 184320


def test_butterfly_strides():
    c = GptConfig(width=128, connectivity="butterfly")
    assert [c.stride(l) for l in range(16)] == PINS["butterfly_strides_w128"]["value"]
    for w in (2, 3, 7, 64, 100, 4096):
        for l in range(16):
            s = GptConfig(width=w, heads=1, connectivity="butterfly").stride(l)
            assert 1 <= s < w and s & (s - 1) == 0


def test_token_codes_are_injective_signed_and_nonzero():
    for width in (2, 4, 6, 16, 64, 128):
        for vocab in (2, 3, 5, 26, 129, 255, 256):
            codes = token_codes(GptConfig(width=width, vocab_size=vocab, heads=1))
            assert codes.shape == (vocab, width)
            assert np.all(np.abs(codes) <= 1) and np.all(codes != 0)
            assert len({c.tobytes() for c in codes}) == vocab


def test_configuration_validation():
    bad = [dict(vocab_size=1), dict(context=0), dict(heads=3), dict(width=6, heads=2),
           dict(width=8, heads=8), dict(layers=65), dict(ffn_mesh_depth=0)]
    for kw in bad:
        with pytest.raises(ValueError):
            GptConfig(**kw).validate()


def test_splitmix_unit_and_index():
    r = Random(0)
    # unit() is the top 24 bits over 2^24, in [0, 1)
    vals = [float(r.unit()) for _ in range(1000)]
    assert all(0.0 <= v < 1.0 for v in vals)
    assert all(float(np.float32(v) * 16777216.0).is_integer() for v in vals)
    r = Random(5)
    assert all(0 <= r.index(7) < 7 for _ in range(1000))


def test_equation_splits_match_reference():
    pins = PINS["add97_seed7_split"]
    ds = EquationDataset(97, "add", 0.5, 7)
    assert (len(ds.training), len(ds.validation)) == (pins["training"], pins["validation"])
    changed = EquationDataset(97, "add", 0.5, 8)
    assert ds.training != changed.training and ds.residue_tokens != changed.residue_tokens
    for op in ("add", "mul", "sub", "div", "mixed", "square-sum", "quadratic",
               "quadratic-linear", "cubic-product", "cubic-mixed"):
        d = EquationDataset(7, op, 0.5, 7)
        pairs = {(a, b) for a, b, _ in d.training + d.validation}
        assert len(pairs) == (PINS["mod7_pairs"]["div"] if op == "div" else PINS["mod7_pairs"]["other"])
        assert d.residue_tokens != list(range(7))
    div = EquationDataset(97, "div", 0.5, 11)
    assert len(div.training) == 4656 and len(div.validation) == 4656
    x, y = ds.batch(False, [0, 0, 1])
    assert list(x[:4]) == [ds.residue_tokens[ds.training[0][0]], 97,
                           ds.residue_tokens[ds.training[0][1]], 98]
    assert list(y[:3]) == [IGNORE_TARGET] * 3


def test_sampler_epochs_without_replacement():
    s, d = EquationSampler(24, 7), EquationSampler(24, 7)
    seen = set()
    for _ in range(100):
        idx = s.sample(12)
        assert idx == d.sample(12) and len(set(idx)) == 12
        seen.update(idx)
    assert seen == set(range(24))
    e = EquationSampler(25, 7)
    assert [len(e.sample(12)) for _ in range(4)] == [12, 12, 1, 12]


def test_warmup():
    for step in range(1, 20):
        assert abs(float(warmed_learning_rate(1e-3, step)) - 1e-3 * min(step, 10) / 10) < 1e-9


def test_zipf_stream_is_reproducible_and_zipfian():
    x1, y1 = zipf_batch(7, 0, 3, 4, 16)
    x2, y2 = zipf_batch(7, 0, 3, 4, 16)
    assert np.array_equal(x1, x2) and np.array_equal(y1, y2)
    assert np.array_equal(x1.reshape(4, 16)[:, 1:], y1.reshape(4, 16)[:, :-1])
    x3, _ = zipf_batch(7, 1, 3, 4, 16)
    assert not np.array_equal(x1, x3)
    big, _ = zipf_batch(1, 0, 0, 64, 256)
    freq = np.bincount(big, minlength=64) / big.size
    expected = np.diff(np.concatenate([[0.0], zipf_cdf(64)]))
    assert np.abs(freq - expected).max() < 0.01


def test_xsa_known_answer_and_floor():
    kat = PINS["xsa_kat"]
    z = exclusive_forward(np.array([kat["y"]]), np.array([kat["v"]]), kat["heads"])
    assert np.allclose(z[0], kat["z"], atol=1e-15)
    y = np.array([[1.5, -0.25, 0.8, -1.2]])
    g = np.array([[0.3, -0.5, 0.7, 0.9]])
    eps = 1e-12
    for v, heads in (([2.0, -1.0, 0.3, 0.7], 2), ([0.0] * 4, 2),
                     ([0.2 * eps, -0.3 * eps, 2 * eps, -eps], 2), ([1.0, -2.0, 0.7, 0.8], 4)):
        v = np.array([v])
        dy, dv = exclusive_backward(y, v, g, heads)
        loss = lambda yy, vv: (exclusive_forward(yy, vv, heads) * g).sum()
        for t, d in ((0, dy), (1, dv)):
            for ch in range(4):
                step = eps * 1e-4 if t == 1 and abs(v[0, ch]) < 1e-10 else 1e-6
                a, b = [y.copy(), v.copy()], [y.copy(), v.copy()]
                a[t][0, ch] += step
                b[t][0, ch] -= step
                num = (loss(*a) - loss(*b)) / (2 * step)
                assert abs(d[0, ch] - num) < 1e-5 * (1 + abs(d[0, ch]))


def test_rope_known_answer_and_inverse():
    x = np.array([[1.0, 2.0, 3.0, 4.0]] * 2)
    out = rope(x, 2, 1)
    assert np.allclose(out[0], x[0])
    exp1 = [1 * math.cos(1) - 3 * math.sin(1), 2 * math.cos(0.01) - 4 * math.sin(0.01),
            3 * math.cos(1) + 1 * math.sin(1), 4 * math.cos(0.01) + 2 * math.sin(0.01)]
    assert np.allclose(out[1], exp1, atol=1e-12)
    r = np.random.default_rng(0).standard_normal((12, 8))
    assert np.allclose(rope(rope(r, 6, 2), 6, 2, inverse=True), r, atol=1e-12)


def test_rmsnorm_zero_input_and_gradient():
    eps = float(np.float32(1e-5))
    y, inv = rmsnorm(np.zeros((1, 4)), 1)
    g = rmsnorm_backward(y, inv, np.array([[0.3, -0.7, 0.5, 1.0]]), 1)
    assert np.allclose(g, np.array([[0.3, -0.7, 0.5, 1.0]]) / math.sqrt(eps))
    x = np.array([[3.0, 4.0, 5.0, 12.0]])
    y, _ = rmsnorm(x, 2)
    assert np.allclose(y[0, :2], x[0, :2] / math.sqrt(12.5 + eps))


@pytest.mark.parametrize("connectivity", ["neighbor", "butterfly"])
def test_hand_adjoints_match_reference_tape(connectivity):
    c = TINY.with_(connectivity=connectivity)
    m = ReferenceGpt(c, seed=7)
    x = [0, 1, 3, 2, 4, 1]
    for y in ([1, 3, 2, 4, 1, 0], [IGNORE_TARGET, IGNORE_TARGET, 2, IGNORE_TARGET, IGNORE_TARGET, 0]):
        loss, grad = m.loss_and_gradient(x, y, 3)
        tl, tg, tlog = tape_loss_and_gradient(c, m.parameters, x, y, 3)
        assert abs(loss - tl) < 1e-12
        assert np.abs(grad - tg).max() < 1e-12
        assert np.abs(m.logits(x, 3) - tlog).max() < 1e-12


def test_finite_differences_tiny():
    m = ReferenceGpt(TINY, seed=7)
    x, y = [0, 1, 3, 2, 4, 1], [1, 3, 2, 4, 1, 0]
    _, grad = m.loss_and_gradient(x, y, 3)
    for p in range(0, len(grad), 3):
        plus, minus = m.parameters.copy(), m.parameters.copy()
        plus[p] += np.float32(1e-4)
        minus[p] -= np.float32(1e-4)
        step = float(plus[p]) - float(minus[p])
        a = ReferenceGpt(TINY, plus).loss_and_gradient(x, y, 3)[0]
        b = ReferenceGpt(TINY, minus).loss_and_gradient(x, y, 3)[0]
        assert abs(grad[p] - (a - b) / step) < 4e-4 * (1 + abs(grad[p]))


def test_causality_and_batch_isolation():
    m = ReferenceGpt(TINY, seed=11)
    a = m.logits([0, 1, 2, 3, 1, 2, 3, 4], 4)
    b = m.logits([0, 1, 4, 0, 4, 4, 4, 4], 4)
    assert np.array_equal(a[:2], b[:2])
    assert np.allclose(a[:2], m.logits([0, 1], 2), atol=1e-14)


def test_answer_only_loss_averages_sequences():
    m = ReferenceGpt(TINY, seed=7)
    x = [0, 1, 3, 2, 4, 1]
    y = [IGNORE_TARGET, IGNORE_TARGET, 2, IGNORE_TARGET, IGNORE_TARGET, 0]
    l, g = m.loss_and_gradient(x, y, 3)
    l1, g1 = m.loss_and_gradient(x[:3], y[:3], 3)
    l2, g2 = m.loss_and_gradient(x[3:], y[3:], 3)
    assert abs(l - (l1 + l2) / 2) < 1e-12 and np.abs(g - (g1 + g2) / 2).max() < 1e-12
    with pytest.raises(ValueError):
        m.loss_and_gradient(x, [IGNORE_TARGET] * 6, 3)
    with pytest.raises(ValueError):
        m.loss_and_gradient(x, [99] * 6, 3)


def test_zero_embeddings_give_zero_logits():
    for conn in ("neighbor", "butterfly"):
        c = TINY.with_(connectivity=conn)
        p = np.full(parameter_count(c), 0.5, dtype=np.float32)
        p[:2 * c.width * c.attention_mesh_depth] = 0.0
        assert np.all(ReferenceGpt(c, p).logits([0, 1, 2, 3, 4, 0], 3) == 0.0)


@pytest.mark.slow
def test_grok_epoch_reproduces_archived_reference_run():
    """One mod-97 epoch (10 steps at batch 512, 96-row tail) reproduces the
    reference's archived train/validation cross-entropies."""
    pin = PINS["grok_epoch"]
    cfgd = pin["config"]
    ds = EquationDataset(cfgd["modulus"], cfgd["operation"], cfgd["train_fraction"], cfgd["seed"])
    cfg = GptConfig(vocab_size=cfgd["vocab_size"], context=4, width=cfgd["width"], heads=cfgd["heads"],
                    layers=cfgd["layers"], attention_mesh_depth=4, ffn_mesh_depth=6)
    m = ReferenceGpt(cfg, seed=cfgd["seed"])

    def evaluate(val):
        x, y = ds.batch(val, range(len(ds.split(val))))
        rows, sup = m.row_losses(m.logits(x, 4), y)
        return rows.sum() / sup.sum()

    start = (evaluate(False), evaluate(True))
    sampler = EquationSampler(len(ds.training), cfgd["seed"])
    p, mo, ve = m.parameters.copy(), np.zeros_like(m.parameters), np.zeros_like(m.parameters)
    b1 = b2 = np.float32(1.0)
    for step in range(1, cfgd["steps"] + 1):
        x, y = ds.batch(False, sampler.sample(cfgd["batch"]))
        _, g = m.loss_and_gradient(x, y, 4)
        b1, b2 = np.float32(b1 * np.float32(0.9)), np.float32(b2 * np.float32(0.98))
        adamw_step(p, mo, ve, g, step, warmed_learning_rate(1e-3, step), 1.0, 0.9, 0.98, 1e-8, (b1, b2))
        m.parameters = p
    end = (evaluate(False), evaluate(True))
    # f64 oracle vs the reference's f32 CUDA run: agreement to ~1e-7 relative.
    for got, want in zip(start + end, pin["train_cross_entropy"][:1] + pin["validation_cross_entropy"][:1]
                         + pin["train_cross_entropy"][1:] + pin["validation_cross_entropy"][1:]):
        assert abs(got - want) < 1e-6 * abs(want), (got, want)


def test_table_embedding_starts_as_the_tabulated_mesh():
    """src/gpt/config.rs:810-840: a table has vocab * width embedding
    parameters and no embedding mesh, its initial table is the mesh model's
    embedding tabulated over the token codes, and the blocks are the mesh
    model's own; so the two models start as one function."""
    from oracle.gpt_config import Layout, parameter_count, tabulated
    for connectivity in ("neighbor", "butterfly"):
        mesh = GptConfig(vocab_size=99, width=16, attention_mesh_depth=6, connectivity=connectivity)
        table = mesh.with_(embedding="table")
        blocks = parameter_count(mesh) - 2 * 16 * 6
        assert parameter_count(table) == 99 * 16 + blocks
        layout = Layout(table)
        assert layout.groups[layout.embedding].size == 99 * 16 and layout.groups[layout.embedding].depth == 0
        assert all(g.size == 2 * 16 * g.depth for g in layout.groups[1:])
        init_mesh = Layout(mesh).initialize(5)
        init_table = layout.initialize(5)
        assert np.array_equal(init_table, tabulated(mesh, init_mesh))
        assert np.array_equal(init_table[99 * 16:], init_mesh[2 * 16 * 6:])
        rm, rt = ReferenceGpt(mesh, init_mesh), ReferenceGpt(table, init_table)
        assert np.abs(rm.token_embeddings() - rt.token_embeddings()).max() < 1e-7
        tokens = np.arange(24) % 99
        targets = (tokens * 7 + 3) % 99
        lm, gm = rm.loss_and_gradient(tokens, targets, 8)
        lt, gt = rt.loss_and_gradient(tokens, targets, 8)
        assert abs(lm - lt) < 1e-7 and np.abs(gm[2 * 16 * 6:] - gt[99 * 16:]).max() < 1e-7


def test_table_gradient_matches_finite_differences():
    from oracle.gpt_config import Layout
    config = GptConfig(vocab_size=7, context=4, width=8, heads=2, layers=1, attention_mesh_depth=2,
                       ffn_mesh_depth=2, embedding="table")
    model = ReferenceGpt(config, seed=3)
    tokens = np.array([1, 2, 3, 4, 5, 6, 0, 1])
    targets = np.array([2, 3, 4, 5, 6, 0, 1, 2])
    _, grad = model.loss_and_gradient(tokens, targets, 4)
    p0 = model.parameters.astype(np.float64).copy()
    for i in range(0, 7 * 8, 5):  # table entries
        h = 1e-4
        model.parameters = p0.copy(); model.parameters[i] += h
        lp = model.loss_and_gradient(tokens, targets, 4)[0]
        model.parameters = p0.copy(); model.parameters[i] -= h
        lm = model.loss_and_gradient(tokens, targets, 4)[0]
        model.parameters = p0.copy()
        assert abs((lp - lm) / (2 * h) - grad[i]) <= 1e-6 + 1e-4 * abs(grad[i])
