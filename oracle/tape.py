"""Pure-Python port of the reference's scalar f64 tape autodiff (test
infrastructure only; tiny configurations only).

Restates ``Tape`` (``src/gpt/reference.rs:244-390``) and the model assembly of
``ReferenceGpt::forward`` / ``loss_and_gradient`` (``:61-88``, ``:104-229``)
node for node, so the vectorised hand-derived oracle in ``gpt_ref.py`` can be
checked against the reference's own differentiation rules.
"""

import math

import numpy as np

from .data import IGNORE_TARGET
from .gpt_config import GptConfig, Layout, RMSNORM_EPSILON, ROPE_BASE, XSA_EPSILON, token_codes

NONE = -1


class Tape:
    def __init__(self, values):
        self.values = [float(v) for v in values]
        self.edges = [((NONE, 0.0), (NONE, 0.0)) for _ in self.values]

    def node(self, value, edges):
        self.values.append(value)
        self.edges.append(edges)
        return len(self.values) - 1

    def constant(self, value):
        return self.node(float(value), ((NONE, 0.0), (NONE, 0.0)))

    def add(self, a, b):
        return self.node(self.values[a] + self.values[b], ((a, 1.0), (b, 1.0)))

    def subtract(self, a, b):
        return self.node(self.values[a] - self.values[b], ((a, 1.0), (b, -1.0)))

    def multiply(self, a, b):
        va, vb = self.values[a], self.values[b]
        return self.node(va * vb, ((a, vb), (b, va)))

    def divide(self, a, b):
        r = 1.0 / self.values[b]
        va = self.values[a]
        return self.node(va * r, ((a, r), (b, -va * r * r)))

    def scale(self, a, s):
        return self.node(self.values[a] * s, ((a, s), (NONE, 0.0)))

    def shift(self, a, o):
        return self.node(self.values[a] + o, ((a, 1.0), (NONE, 0.0)))

    def exp(self, a):
        v = math.exp(self.values[a])
        return self.node(v, ((a, v), (NONE, 0.0)))

    def log(self, a):
        return self.node(math.log(self.values[a]), ((a, 1.0 / self.values[a]), (NONE, 0.0)))

    def inverse_sqrt(self, a):
        v = 1.0 / math.sqrt(self.values[a])
        return self.node(v, ((a, -0.5 * v * v * v), (NONE, 0.0)))

    def clamp_min(self, a, m):
        x = self.values[a]
        return self.node(max(x, m), ((a, 1.0 if x >= m else 0.0), (NONE, 0.0)))

    def elu(self, a):
        x = self.values[a]
        if x >= 0.0:
            return self.scale(a, 1.0)
        return self.node(math.expm1(x), ((a, math.exp(x)), (NONE, 0.0)))

    def sum(self, ids):
        total = ids[0]
        for i in ids[1:]:
            total = self.add(total, i)
        return total

    def dot(self, left, right):
        return self.sum([self.multiply(a, b) for a, b in zip(left, right)])

    def shifted_exponentials(self, ids):
        maximum = max(self.values[i] for i in ids)
        ex = [self.exp(self.shift(i, -maximum)) for i in ids]
        return maximum, self.sum(ex), ex

    def backward(self, loss, count):
        adj = [0.0] * len(self.values)
        adj[loss] = 1.0
        for i in range(len(self.values) - 1, -1, -1):
            for parent, d in self.edges[i]:
                if parent != NONE:
                    adj[parent] += adj[i] * d
        return adj[:count]


def _rmsnorm(t, x, heads):
    hw = len(x[0]) // heads
    out = []
    for row in x:
        r = []
        for h in range(heads):
            head = row[h * hw:(h + 1) * hw]
            ms = t.scale(t.dot(head, head), 1.0 / hw)
            inv = t.inverse_sqrt(t.shift(ms, float(RMSNORM_EPSILON)))
            r += [t.multiply(i, inv) for i in head]
        out.append(r)
    return out


def _mesh(t, x, offset, depth, config):
    w = len(x[0])
    for layer in range(depth):
        s = config.stride(layer)
        nxt = []
        for row in x:
            r = []
            for c in range(w):
                p = offset + layer * 2 * w + 2 * c
                total = t.add(t.multiply(row[c], p), t.multiply(row[(c + s) % w], p + 1))
                r.append(total if layer + 1 == depth else t.elu(total))
            nxt.append(r)
        x = nxt
    return x


def _rotary(t, x, sequence, heads):
    out = []
    for rowi, row in enumerate(x):
        pos = rowi % sequence
        hw = len(row) // heads
        half = hw // 2
        o = list(row)
        for h in range(heads):
            for pair in range(half):
                angle = pos / float(ROPE_BASE) ** (pair / half)
                sn, cs = math.sin(angle), math.cos(angle)
                l = h * hw + pair
                r = l + half
                o[l] = t.subtract(t.scale(row[l], cs), t.scale(row[r], sn))
                o[r] = t.add(t.scale(row[r], cs), t.scale(row[l], sn))
        out.append(o)
    return out


def _attention(t, q, k, v, sequence, heads):
    w = len(q[0])
    hw = w // heads
    out = []
    for rowi, query in enumerate(q):
        pos = rowi % sequence
        first = rowi - pos
        o = []
        for h in range(heads):
            b = h * hw
            scores = [t.scale(t.dot(query[b:b + hw], k[first + j][b:b + hw]), 1.0 / math.sqrt(hw))
                      for j in range(pos + 1)]
            _, total, ex = t.shifted_exponentials(scores)
            probs = [t.divide(e, total) for e in ex]
            for ch in range(b, b + hw):
                o.append(t.sum([t.multiply(p, v[first + j][ch]) for j, p in enumerate(probs)]))
        out.append(o)
    return out


def _exclusive(t, y, v, heads):
    hw = len(y[0]) // heads
    out = []
    for yr, vr in zip(y, v):
        o = []
        for h in range(heads):
            yy, vv = yr[h * hw:(h + 1) * hw], vr[h * hw:(h + 1) * hw]
            sq = t.dot(vv, vv)
            inv = t.inverse_sqrt(t.clamp_min(sq, float(XSA_EPSILON) ** 2))
            u = [t.multiply(i, inv) for i in vv]
            proj = t.dot(yy, u)
            o += [t.subtract(a, t.multiply(proj, b)) for a, b in zip(yy, u)]
        out.append(o)
    return out


def tape_loss_and_gradient(config: GptConfig, parameters, tokens, targets, sequence):
    """Loss and f64 gradient exactly as the reference tape computes them."""
    layout = Layout(config)
    t = Tape(np.asarray(parameters, dtype=np.float32).astype(np.float64))
    codes = [[t.constant(float(x)) for x in row] for row in token_codes(config)]
    emb = _mesh(t, codes, layout.groups[layout.embedding].offset,
                config.attention_mesh_depth, config)
    x = [list(emb[int(tok)]) for tok in tokens]
    A, F, H = config.attention_mesh_depth, config.ffn_mesh_depth, config.heads
    for block in layout.blocks:
        n = _rmsnorm(t, x, 1)
        q, k, v = (_mesh(t, n, layout.groups[block[nm]].offset, A, config)
                   for nm in ("query", "key", "value"))
        q = _rotary(t, _rmsnorm(t, q, H), sequence, H)
        k = _rotary(t, _rmsnorm(t, k, H), sequence, H)
        att = _exclusive(t, _attention(t, q, k, v, sequence, H), v, H)
        proj = _mesh(t, att, layout.groups[block["projection"]].offset, A, config)
        x = [[t.add(a, b) for a, b in zip(r1, r2)] for r1, r2 in zip(x, proj)]
        n = _rmsnorm(t, x, 1)
        ff = _mesh(t, n, layout.groups[block["ffn"]].offset, F, config)
        x = [[t.add(a, b) for a, b in zip(r1, r2)] for r1, r2 in zip(x, ff)]
    n = _rmsnorm(t, x, 1)
    logits = [[t.dot(row, emb[tok]) for tok in range(config.vocab_size)] for row in n]
    losses = []
    for row, target in zip(logits, targets):
        if int(target) == IGNORE_TARGET:
            continue
        m, total, _ = t.shifted_exponentials(row)
        losses.append(t.subtract(t.shift(t.log(total), m), row[int(target)]))
    loss_id = t.scale(t.sum(losses), 1.0 / len(losses))
    grad = t.backward(loss_id, layout.count())
    return t.values[loss_id], np.array(grad), np.array([[t.values[i] for i in r] for r in logits])
