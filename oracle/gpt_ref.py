"""f64 Mesh GPT forward / backward with hand-derived adjoints (test
infrastructure only).

Restates the model of ``src/gpt/reference.rs:104-229`` (embeddings, blocks,
tied head) and the loss of ``:61-88`` (mean cross-entropy over supervised rows,
IGNORE = u32::MAX).  The operators follow ``rmsnorm`` (``:392-409``), ``mesh``
(``:422-453``, ELU on every layer but the last of a stack), ``rotary``
(``:462-490``, split-half pairs, position = row mod sequence), ``attention``
(``:510-554``, causal including the diagonal, scale 1/sqrt(head width)) and
``exclusive`` (``:577-603``, z = y - (y.u)u, u = v / max(|v|, 1e-12)).  The
adjoints are derived by hand and checked against ``tape.py`` (a direct port of
the reference tape, ``:244-390``) and finite differences.

Rows are vectorised with numpy; attention runs in chunks of whole sequences.
"""

import numpy as np

from .data import IGNORE_TARGET
from .gpt_config import GptConfig, Layout, RMSNORM_EPSILON, ROPE_BASE, XSA_EPSILON, token_codes

EPS_RMS = float(RMSNORM_EPSILON)
EPS_XSA = float(XSA_EPSILON)


# ----------------------------------------------------------------- operators
def rmsnorm(x, heads):
    n, w = x.shape
    hd = w // heads
    xh = x.reshape(n, heads, hd)
    inv = 1.0 / np.sqrt((xh * xh).sum(-1) / hd + EPS_RMS)
    return (xh * inv[..., None]).reshape(n, w), inv


def rmsnorm_backward(y, inv, dy, heads):
    n, w = y.shape
    hd = w // heads
    yh, dyh = y.reshape(n, heads, hd), dy.reshape(n, heads, hd)
    dot = (dyh * yh).sum(-1, keepdims=True)
    return (inv[..., None] * (dyh - yh * dot / hd)).reshape(n, w)


def mesh_forward(x, weights, strides):
    """weights [depth][W][2]; returns the list [input, y_1, ..., y_depth]."""
    acts = [x]
    depth = len(strides)
    for layer, s in enumerate(strides):
        z = x * weights[layer, :, 0] + np.roll(x, -s, axis=1) * weights[layer, :, 1]
        x = z if layer + 1 == depth else np.where(z >= 0.0, z, np.expm1(np.minimum(z, 0.0)))
        acts.append(x)
    return acts


def mesh_backward(acts, weights, strides, dy):
    """Returns (dx, dweights[depth][W][2])."""
    depth = len(strides)
    dw = np.zeros(weights.shape)
    for layer in reversed(range(depth)):
        s = strides[layer]
        x, y = acts[layer], acts[layer + 1]
        dz = dy if layer + 1 == depth else dy * np.where(y >= 0.0, 1.0, y + 1.0)
        neighbor = np.roll(x, -s, axis=1)
        dw[layer, :, 0] = (dz * x).sum(0)
        dw[layer, :, 1] = (dz * neighbor).sum(0)
        dy = dz * weights[layer, :, 0] + np.roll(dz * weights[layer, :, 1], s, axis=1)
    return dy, dw


def rope_tables(sequence, head_width):
    half = head_width // 2
    pair = np.arange(half, dtype=np.float64)
    freq = float(ROPE_BASE) ** (pair / half)
    angle = np.arange(sequence, dtype=np.float64)[:, None] / freq[None, :]
    return np.cos(angle), np.sin(angle)


def rope(x, sequence, heads, inverse=False):
    n, w = x.shape
    hd = w // heads
    half = hd // 2
    cos, sin = rope_tables(sequence, hd)
    pos = np.arange(n) % sequence
    c, s = cos[pos][:, None, :], sin[pos][:, None, :]
    if inverse:
        s = -s
    xh = x.reshape(n, heads, hd)
    a, b = xh[..., :half], xh[..., half:]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=-1).reshape(n, w)


def _chunks(n, sequence, heads):
    """Sequence chunks of at most ~8M score entries each."""
    seqs = n // sequence
    per = max(1, (1 << 23) // max(1, heads * sequence * sequence))
    for first in range(0, seqs, per):
        yield first * sequence, min(seqs, first + per) * sequence


def _heads(x, sequence, heads):
    n, w = x.shape
    return x.reshape(n // sequence, sequence, heads, w // heads).transpose(0, 2, 1, 3)


def _rows(x):
    s, h, t, d = x.shape
    return x.transpose(0, 2, 1, 3).reshape(s * t, h * d)


def attention_forward(q, k, v, sequence, heads):
    """Returns (o, probabilities per chunk [S][H][T][T])."""
    n, w = q.shape
    hd = w // heads
    scale = 1.0 / np.sqrt(hd)
    mask = np.tril(np.ones((sequence, sequence), dtype=bool))
    o = np.empty_like(q)
    probs = []
    for a, b in _chunks(n, sequence, heads):
        qh, kh, vh = (_heads(t[a:b], sequence, heads) for t in (q, k, v))
        s = np.where(mask, qh @ kh.transpose(0, 1, 3, 2) * scale, -np.inf)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        o[a:b] = _rows(p @ vh)
        probs.append(p)
    return o, probs


def attention_backward(q, k, v, probs, do, sequence, heads):
    n, w = q.shape
    hd = w // heads
    scale = 1.0 / np.sqrt(hd)
    dq, dk, dv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
    for i, (a, b) in enumerate(_chunks(n, sequence, heads)):
        qh, kh, vh, doh = (_heads(t[a:b], sequence, heads) for t in (q, k, v, do))
        p = probs[i]
        dv[a:b] = _rows(p.transpose(0, 1, 3, 2) @ doh)
        dp = doh @ vh.transpose(0, 1, 3, 2)
        ds = p * (dp - (dp * p).sum(-1, keepdims=True)) * scale
        dq[a:b] = _rows(ds @ kh)
        dk[a:b] = _rows(ds.transpose(0, 1, 3, 2) @ qh)
    return dq, dk, dv


def exclusive_forward(y, v, heads):
    n, w = y.shape
    hd = w // heads
    yh, vh = y.reshape(n, heads, hd), v.reshape(n, heads, hd)
    norm = np.sqrt((vh * vh).sum(-1, keepdims=True))
    inv = 1.0 / np.maximum(norm, EPS_XSA)
    u = vh * inv
    proj = (yh * u).sum(-1, keepdims=True)
    return (yh - proj * u).reshape(n, w)


def exclusive_backward(y, v, dz, heads):
    n, w = y.shape
    hd = w // heads
    yh, vh, gh = y.reshape(n, heads, hd), v.reshape(n, heads, hd), dz.reshape(n, heads, hd)
    sq = (vh * vh).sum(-1, keepdims=True)
    norm = np.sqrt(sq)
    inv = 1.0 / np.maximum(norm, EPS_XSA)
    u = vh * inv
    proj = (yh * u).sum(-1, keepdims=True)
    gproj = (gh * u).sum(-1, keepdims=True)
    dy = gh - gproj * u
    du = -gproj * yh - proj * gh
    # The norm is differentiated only above the floor (tape clamp_min, :591).
    above = sq >= EPS_XSA * EPS_XSA
    dv = inv * (du + np.where(above, 2.0 * proj * gproj * u, 0.0))
    return dy.reshape(n, w), dv.reshape(n, w)


# --------------------------------------------------------------------- model
class ReferenceGpt:
    """f64 restatement of ``ReferenceGpt`` (``src/gpt/reference.rs:14-229``)."""

    def __init__(self, config: GptConfig, parameters=None, seed: int = 7):
        self.config = config.validate()
        self.layout = Layout(config)
        if parameters is None:
            parameters = self.layout.initialize(seed)
        parameters = np.asarray(parameters, dtype=np.float32)
        if parameters.shape != (self.layout.count(),):
            raise ValueError("parameter count does not match GPT configuration")
        self.parameters = parameters
        self.codes = token_codes(config).astype(np.float64)

    def _w(self, gid):
        return self.layout.group_weights(self.parameters, gid).astype(np.float64)

    def _strides(self, depth):
        return [self.config.stride(l) for l in range(depth)]

    def forward(self, tokens, sequence):
        c = self.config
        tokens = np.asarray(tokens, dtype=np.int64)
        if sequence < 1 or sequence > c.context or len(tokens) == 0 or len(tokens) % sequence:
            raise ValueError("tokens must form equal sequences within context")
        if (tokens >= c.vocab_size).any() or (tokens < 0).any():
            raise ValueError("token ID is outside the vocabulary")
        A, F, H = c.attention_mesh_depth, c.ffn_mesh_depth, c.heads
        cache = {"tokens": tokens, "sequence": sequence, "blocks": []}
        if c.embedding == "table":
            emb_acts = None
            E = self._table()
        else:
            emb_acts = mesh_forward(self.codes, self._w(self.layout.embedding), self._strides(A))
            E = emb_acts[-1]
        cache["emb_acts"], cache["E"] = emb_acts, E
        x = E[tokens]
        for block in self.layout.blocks:
            bc = {"x": x}
            n1, inv1 = rmsnorm(x, 1)
            bc["n1"], bc["inv1"] = n1, inv1
            acts = {}
            for name in ("query", "key", "value"):
                acts[name] = mesh_forward(n1, self._w(block[name]), self._strides(A))
            bc["acts"] = acts
            qn, invq = rmsnorm(acts["query"][-1], H)
            kn, invk = rmsnorm(acts["key"][-1], H)
            bc.update(qn=qn, invq=invq, kn=kn, invk=invk)
            qr, kr = rope(qn, sequence, H), rope(kn, sequence, H)
            v = acts["value"][-1]
            o, probs = attention_forward(qr, kr, v, sequence, H)
            bc.update(qr=qr, kr=kr, v=v, o=o, probs=probs)
            z = exclusive_forward(o, v, H)
            pacts = mesh_forward(z, self._w(block["projection"]), self._strides(A))
            xm = x + pacts[-1]
            n2, inv2 = rmsnorm(xm, 1)
            facts = mesh_forward(n2, self._w(block["ffn"]), self._strides(F))
            x = xm + facts[-1]
            bc.update(pacts=pacts, xm=xm, n2=n2, inv2=inv2, facts=facts)
            cache["blocks"].append(bc)
        nf, invf = rmsnorm(x, 1)
        cache.update(x_final=x, nf=nf, invf=invf)
        logits = nf @ E.T
        return logits, cache

    def logits(self, tokens, sequence):
        return self.forward(tokens, sequence)[0]

    def hidden_states(self, tokens, sequence):
        return self.forward(tokens, sequence)[1]["x_final"]

    def _table(self):
        g = self.layout.groups[self.layout.embedding]
        return self.parameters[g.offset:g.offset + g.size].astype(np.float64).reshape(
            self.config.vocab_size, self.config.width)

    def token_embeddings(self):
        if self.config.embedding == "table":
            return self._table()
        return mesh_forward(self.codes, self._w(self.layout.embedding),
                            self._strides(self.config.attention_mesh_depth))[-1]

    @staticmethod
    def row_losses(logits, targets):
        """Per-row cross-entropy (0 for ignored rows) and the supervised mask."""
        targets = np.asarray(targets, dtype=np.int64)
        sup = targets != IGNORE_TARGET
        m = logits.max(-1, keepdims=True)
        lse = np.log(np.exp(logits - m).sum(-1)) + m[:, 0]
        t = np.where(sup, targets, 0)
        rows = np.where(sup, lse - logits[np.arange(len(t)), t], 0.0)
        return rows, sup

    def loss_and_gradient(self, tokens, targets, sequence):
        """(mean supervised CE, f64 gradient of every parameter) —
        ``src/gpt/reference.rs:61-88``."""
        c = self.config
        targets = np.asarray(targets, dtype=np.int64)
        if len(targets) != len(tokens):
            raise ValueError("inputs and targets must have equal lengths")
        sup = targets != IGNORE_TARGET
        if not sup.any():
            raise ValueError("batch must contain at least one supervised target")
        if (targets[sup] >= c.vocab_size).any():
            raise ValueError("target ID is outside the vocabulary")
        logits, cache = self.forward(tokens, sequence)
        rows, sup = self.row_losses(logits, targets)
        count = int(sup.sum())
        loss = rows.sum() / count
        grad = np.zeros(self.layout.count())
        # head
        p = np.exp(logits - logits.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        t = np.where(sup, targets, 0)
        p[np.arange(len(t)), t] -= 1.0
        dlogits = np.where(sup[:, None], p / count, 0.0)
        emb_acts, E = cache["emb_acts"], cache["E"]
        dE = dlogits.T @ cache["nf"]
        dx = rmsnorm_backward(cache["nf"], cache["invf"], dlogits @ E, 1)
        H, A, F = c.heads, c.attention_mesh_depth, c.ffn_mesh_depth
        seq = cache["sequence"]
        for block, bc in zip(reversed(self.layout.blocks), reversed(cache["blocks"])):
            dxm = dx.copy()
            dn2, dw = mesh_backward(bc["facts"], self._w(block["ffn"]), self._strides(F), dx)
            self._add(grad, block["ffn"], dw)
            dxm += rmsnorm_backward(bc["n2"], bc["inv2"], dn2, 1)
            dz, dw = mesh_backward(bc["pacts"], self._w(block["projection"]), self._strides(A), dxm)
            self._add(grad, block["projection"], dw)
            do, dv_x = exclusive_backward(bc["o"], bc["v"], dz, H)
            dqr, dkr, dv_a = attention_backward(bc["qr"], bc["kr"], bc["v"], bc["probs"], do, seq, H)
            dq = rmsnorm_backward(bc["qn"], bc["invq"], rope(dqr, seq, H, inverse=True), H)
            dk = rmsnorm_backward(bc["kn"], bc["invk"], rope(dkr, seq, H, inverse=True), H)
            dn1 = np.zeros_like(dx)
            for name, d in (("query", dq), ("key", dk), ("value", dv_x + dv_a)):
                dni, dw = mesh_backward(bc["acts"][name], self._w(block[name]), self._strides(A), d)
                self._add(grad, block[name], dw)
                dn1 += dni
            dx = dxm + rmsnorm_backward(bc["n1"], bc["inv1"], dn1, 1)
        np.add.at(dE, cache["tokens"], dx)
        if c.embedding == "table":
            self._add(grad, self.layout.embedding, dE)  # the table's gradient is dE itself
        else:
            _, dw = mesh_backward(emb_acts, self._w(self.layout.embedding), self._strides(A), dE)
            self._add(grad, self.layout.embedding, dw)
        return loss, grad

    def _add(self, grad, gid, dw):
        g = self.layout.groups[gid]
        grad[g.offset:g.offset + g.size] += dw.reshape(-1)


def adamw_step(parameters, m, v, gradient, step, lr, wd, beta1=0.9, beta2=0.999, eps=1e-8,
               powers=None):
    """AdamW with decoupled decay in FP32 host semantics
    (``src/bin/mesh-gpt.rs:448-470``; device kernel ``src/gpt/gpu.rs:1369-1391``).
    ``powers`` = (beta1^t, beta2^t) accumulated in f32 by the caller
    (``src/gpt/gpu.rs:1980-1981``).  Updates in place."""
    f = np.float32
    b1p, b2p = powers
    g = gradient.astype(np.float32)
    m[:] = f(beta1) * m + (f(1.0) - f(beta1)) * g
    v[:] = f(beta2) * v + (f(1.0) - f(beta2)) * g * g
    mh = m / (f(1.0) - b1p)
    vh = v / (f(1.0) - b2p)
    parameters[:] = parameters - f(lr) * (mh / (np.sqrt(vh) + f(eps)) + f(wd) * parameters)
