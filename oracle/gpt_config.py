"""Mesh GPT configuration, parameter layout, seeded init and token codes
(test infrastructure only).

Restates ``src/gpt/config.rs``: ``GptConfig`` defaults (``:38-56``),
validation (``:144-172``), connectivity strides (``:117-122``), ``Layout``
(``:358-414``), ``Layout::initialize`` (``:416-459``, default parity
geometry; a table embedding starts as the tabulated mesh embedding,
``tabulated`` at ``:515-546``) and ``token_codes`` (``:552-591``).
"""

from dataclasses import dataclass, replace

import numpy as np

from .rng import Random

RMSNORM_EPSILON = np.float32(1e-5)  # src/gpt/mod.rs:39
XSA_EPSILON = np.float32(1e-12)  # src/gpt/mod.rs:41
ROPE_BASE = np.float32(10000.0)  # src/gpt/mod.rs:37


@dataclass(frozen=True)
class GptConfig:
    vocab_size: int = 32
    context: int = 32
    width: int = 32
    heads: int = 4
    layers: int = 2
    attention_mesh_depth: int = 4
    ffn_mesh_depth: int = 6
    connectivity: str = "neighbor"  # or "butterfly"
    embedding: str = "mesh"  # or "table" (src/gpt/config.rs:60-67)

    def validate(self):
        # src/gpt/config.rs:144-172
        if not 2 <= self.vocab_size <= 65536:
            raise ValueError("vocab_size must be in 2..65536")
        if not 1 <= self.context <= 4096:
            raise ValueError("context must be in 1..4096")
        if not 2 <= self.width <= 4096:
            raise ValueError("width must be in 2..4096")
        if not 1 <= self.heads <= 64 or self.width % self.heads:
            raise ValueError("heads must be in 1..64 and divide width")
        if self.width // self.heads < 2:
            raise ValueError("each attention head requires at least two channels")
        if (self.width // self.heads) % 2:
            raise ValueError("slice RoPE requires an even number of channels per head")
        if not 1 <= self.layers <= 64:
            raise ValueError("layers must be in 1..64")
        if not (1 <= self.attention_mesh_depth <= 256 and 1 <= self.ffn_mesh_depth <= 256):
            raise ValueError("mesh depths must be in 1..256")
        if self.embedding not in ("mesh", "table"):
            raise ValueError("unknown token embedding")
        return self

    def stride(self, layer: int) -> int:
        # src/gpt/config.rs:117-122
        if self.connectivity == "neighbor":
            return 1
        return 1 << (layer % (self.width.bit_length() - 1))

    def with_(self, **kw):
        return replace(self, **kw)


@dataclass
class Group:
    offset: int
    size: int
    depth: int


class Layout:
    """``src/gpt/config.rs:352-414``: embedding group, then per block the
    query, key, value, projection and FFN meshes; each group is layer-major
    with (self, neighbor) weight pairs per channel."""

    def __init__(self, config: GptConfig):
        config.validate()
        self.config = config
        self.groups = []
        w, a, f = config.width, config.attention_mesh_depth, config.ffn_mesh_depth
        # A table has no mesh layers (src/gpt/config.rs:366-372).
        self.embedding = (self._push(2 * w * a, a) if config.embedding == "mesh"
                          else self._push(config.vocab_size * w, 0))
        self.blocks = []
        for _ in range(config.layers):
            q = self._push(2 * w * a, a)
            k = self._push(2 * w * a, a)
            v = self._push(2 * w * a, a)
            o = self._push(2 * w * a, a)
            ffn = self._push(2 * w * f, f)
            self.blocks.append(dict(query=q, key=k, value=v, projection=o, ffn=ffn))

    def _push(self, size, depth):
        self.groups.append(Group(self.count(), size, depth))
        return len(self.groups) - 1

    def count(self) -> int:
        return 0 if not self.groups else self.groups[-1].offset + self.groups[-1].size

    def group_weights(self, parameters, gid):
        """Group ``gid`` as an array [depth][width][2] (self, neighbor)."""
        g = self.groups[gid]
        return np.asarray(parameters[g.offset:g.offset + g.size]).reshape(
            g.depth, self.config.width, 2)

    def initialize(self, seed: int) -> np.ndarray:
        """``src/gpt/config.rs:416-459`` in f32 arithmetic, draw order
        group -> layer -> channel -> (self, neighbor).  A table embedding
        draws the mesh model's stream and stores its tabulated embedding, so
        both start as one function."""
        if self.config.embedding == "table":
            mesh = self.config.with_(embedding="mesh")
            return tabulated(mesh, Layout(mesh).initialize(seed))
        random = Random(seed)
        out = np.zeros(self.count(), dtype=np.float32)
        w = self.config.width
        f = np.float32
        for g in self.groups:
            for layer in range(g.depth):
                for channel in range(w):
                    o = g.offset + layer * 2 * w + channel * 2
                    a = f(0.7) + f(0.2) * (random.unit() - f(0.5))
                    b = f(0.4) * (random.unit() - f(0.5))
                    if layer + 1 == g.depth:
                        a = a * f(0.3)
                        b = b * f(0.3)
                    out[o], out[o + 1] = a, b
        return out


def tabulated(config: GptConfig, parameters) -> np.ndarray:
    """``src/gpt/config.rs:515-546``: the mesh embedding of every token code in
    f64 (ELU through expm1), cast to f32, followed by the block parameters."""
    w, depth = config.width, config.attention_mesh_depth
    p = np.asarray(parameters, dtype=np.float32)
    vectors = token_codes(config).astype(np.float64)
    for layer in range(depth):
        s = config.stride(layer)
        w0 = p[layer * 2 * w:(layer + 1) * 2 * w:2].astype(np.float64)
        w1 = p[layer * 2 * w + 1:(layer + 1) * 2 * w:2].astype(np.float64)
        total = vectors * w0 + np.roll(vectors, -s, axis=1) * w1
        vectors = np.where(total < 0.0, np.expm1(total), total) if layer + 1 != depth else total
    return np.concatenate([vectors.astype(np.float32).reshape(-1), p[2 * w * depth:]])


def parameter_count(config: GptConfig) -> int:
    return Layout(config).count()


def token_codes(config: GptConfig) -> np.ndarray:
    """Fixed signed injective codes, ``src/gpt/config.rs:552-591`` (parity
    form, token order)."""
    v, w = config.vocab_size, config.width
    bits = (v - 1).bit_length()
    lanes = min(w, bits)
    masks = [1 << b for b in range(bits)] + [m for m in range(1, 1 << bits) if m & (m - 1)]
    codes = np.zeros((v, w), dtype=np.float32)
    for token in range(v):
        for channel in range(w):
            if w >= bits:
                ones = bin(token & masks[channel % len(masks)]).count("1")
                codes[token, channel] = -1.0 if ones % 2 == 0 else 1.0
                continue
            digit = maximum = 0
            for bit in range(channel % lanes, bits, lanes):
                digit = 2 * digit + ((token >> bit) & 1)
                maximum = 2 * maximum + 1
            codes[token, channel] = np.float32(2.0) * np.float32(digit) / np.float32(maximum) - np.float32(1.0)
    return codes
