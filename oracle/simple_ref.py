"""grok-simple models: configuration, seeded init, one-hot encoding and an f64
restatement of the forward pass, loss and gradients (test infrastructure
only: the checker of the CUDA path, never the product).

Covers the three architectures of the benchmark configurations and three
more:

* ``mesh-mlp`` (``src/simple/mod.rs:42-46``): dense input layer, ``depth-1``
  two-parent mesh layers with the activation on their inputs, dense readout.
* ``tied-rotary-residual-dense-mlp`` (``:71-73``): shared operand embedding
  E with operand b rotated pairwise by 90 degrees, pre-RMSNorm residual
  blocks with one activated dense projection each, final RMSNorm, tied
  readout through E.
* ``shared-neighbor-mesh-mlp`` (``:51-53``): a linear Neighbor embedding
  chain shared by a, b and the transposed readout, Rotate90 roles,
  pre-RMSNorm residual two-parent blocks with biases, final RMSNorm.
* ``mlp`` (``:36-37``): concatenated operands, ``depth`` activated
  bias-free dense layers, dense readout.
* ``bilinear`` (``:77-78``): the elementwise product of separate ``a`` and
  ``b`` embeddings, read out by a dense layer.
* ``residual-mlp`` (``:60-62``): a dense operand embedding, ``depth``
  pre-RMSNorm feed-forward blocks (width -> width * expansion -> width)
  with residual sums, a final RMSNorm and a dense readout.
* the residual mesh family (``:57-70``): ``depth`` pre-RMSNorm residual
  blocks whose branches are ``mesh_depth`` fixed-width mesh layers
  (activated between layers, and after the last with
  ``mesh_output_activation``), a final RMSNorm and a readout; the operand
  embedding is a dense layer over ``[a | b]`` (``residual-mesh-mlp``), the
  concatenation ``[E a | E b]`` projected to ``width``
  (``tied-concat-residual-mesh-mlp``) or E's Rotate90 roles
  (``tied-rotary-residual-mesh-mlp``); the tied ones read out through E.
* ``tied-concat-mesh-mlp`` (``:54-56``): the tied concatenation embedding,
  ``depth-1`` mesh layers as in ``mesh-mlp``, readout through E.
* ``full-mesh-mlp`` (``:47-49``): an entirely two-parent network over the
  binary operand bits, every unit ``x[a] w0 + x[b] w1 + bias`` with the
  activation on the inputs of every layer after the first.

Sources: ``SimpleConfig`` validation / layout / init / encode
(``src/simple/mod.rs:500-1055``), the f64 tape model
(``src/simple/reference.rs:143-448``), AdamW of ``simple_adam``
(``src/simple/gpu.rs:787-812``) with f32 host beta powers
(``:2044-2047``), the record loop of ``grok-simple``
(``src/bin/mesh-gpt/simple.rs:242-652,757-860``) and ``row_metrics``
(``src/bin/mesh-gpt/grokking.rs:544-557``).  The tape is replaced by
hand-derived numpy gradients; ``tests/test_simple_oracle.py`` checks them by
finite differences and pins the archived step-0 and step-10 records.
"""

import math
from dataclasses import dataclass, replace

import numpy as np

from .data import EquationDataset, EquationSampler, warmed_learning_rate
from .gpt_ref import adamw_step
from .rng import Random

RMSNORM_EPSILON = 1e-5  # src/gpt/mod.rs:39 (f32 1e-5 widened)
EPS = float(np.float32(RMSNORM_EPSILON))
MAX_WIDTH, MAX_DEPTH, MAX_CLASSES = 16384, 64, 1024  # src/simple/mod.rs:25-31
ARCHITECTURES = ("mesh-mlp", "tied-rotary-residual-dense-mlp", "shared-neighbor-mesh-mlp", "mlp", "bilinear",
                 "residual-mlp", "residual-mesh-mlp", "tied-concat-residual-mesh-mlp",
                 "tied-rotary-residual-mesh-mlp", "tied-concat-mesh-mlp", "full-mesh-mlp")
ENCODINGS = ("one-hot", "binary", "scalar", "discrete-log")
RESIDUAL_MESH = ("residual-mesh-mlp", "tied-concat-residual-mesh-mlp", "tied-rotary-residual-mesh-mlp")
TIED_CONCAT = ("tied-concat-residual-mesh-mlp", "tied-concat-mesh-mlp")
ROTARY = ("tied-rotary-residual-dense-mlp", "shared-neighbor-mesh-mlp", "tied-rotary-residual-mesh-mlp")


def two_parents(inputs: int, outputs: int, stride: int):
    """``TwoParentLayer::parents`` (``src/simple/mod.rs:493-496``) for every
    output: the first parent o * inputs / outputs and (first + stride) mod
    inputs."""
    first = np.arange(outputs) * inputs // outputs
    return first, (first + stride) % inputs


def butterfly_stride(width: int, layer: int) -> int:
    """``src/gpt/config.rs:117-122``: 2^(layer mod floor(log2 width))."""
    return 1 << (layer % (width.bit_length() - 1))


@dataclass(frozen=True)
class SimpleConfig:
    """The subset of ``SimpleConfig`` (``src/simple/mod.rs:500-558``) these
    architectures read.  Encoding is one-hot (``scalar``, one feature per
    operand, is accepted by the dense architectures so that the reference's
    tiny known-answer models can be stated); the embedding initializers are
    the reference defaults (uniform fan-in E, near-identity shared chain)."""
    architecture: str = "mesh-mlp"
    activation: str = "relu"  # or "square"
    modulus: int = 97
    width: int = 128
    depth: int = 1
    connectivity: str = "neighbor"  # own | neighbor | butterfly
    embedding_mesh_depth: int = 4
    full_mesh_initialization: str = "kaiming"  # or "identity-hidden"
    mesh_learning_rate_multiplier: int = 1
    encoding: str = "one-hot"  # binary | scalar | discrete-log
    expansion: int = 4  # residual-mlp hidden width / width
    mesh_depth: int = 4  # mesh layers per residual mesh branch
    mesh_output_activation: bool = False  # activate the branch output too
    tied_mesh: bool = False  # every mesh layer uses the first one's weights
    decay_factors: int = 2  # factors per hidden channel the weight decay imitates

    def with_(self, **kw):
        return replace(self, **kw)

    # -------------------------------------------------------------- validation
    def validate(self):
        """``src/simple/mod.rs:561-694`` for these architectures."""
        a = self.architecture
        if a not in ARCHITECTURES:
            raise ValueError(f"unsupported architecture: {a}")
        if self.activation not in ("relu", "square"):
            raise ValueError("unknown activation")
        if self.connectivity not in ("own", "neighbor", "butterfly"):
            raise ValueError("unknown mesh connectivity")
        if not 2 <= self.modulus <= MAX_CLASSES:
            raise ValueError(f"modulus must be in 2..={MAX_CLASSES}")
        if not 1 <= self.width <= MAX_WIDTH:
            raise ValueError(f"width must be in 1..={MAX_WIDTH}")
        if a != "bilinear" and not 1 <= self.depth <= MAX_DEPTH:
            raise ValueError(f"depth must be in 1..={MAX_DEPTH}")
        if self.encoding not in ENCODINGS:
            raise ValueError("unknown encoding")
        if self.encoding == "discrete-log":
            primitive_root(self.modulus)
        if a == "residual-mlp" and not 1 <= self.width * self.expansion <= MAX_WIDTH:
            raise ValueError(f"residual hidden width must be in 1..={MAX_WIDTH}")
        if a in RESIDUAL_MESH and not 1 <= self.mesh_depth <= MAX_DEPTH:
            raise ValueError(f"mesh depth must be in 1..={MAX_DEPTH}")
        if self.mesh_output_activation and a not in RESIDUAL_MESH:
            raise ValueError("only residual mesh branches activate their final mesh output")
        if self.tied_mesh and a not in ("mesh-mlp", "tied-concat-mesh-mlp"):
            raise ValueError("only mesh MLPs tie mesh layers")
        if self.decay_factors < 2:
            raise ValueError("weight decay imitates at least two factors per channel")
        if self.decay_factors != 2 and (a != "mlp" or self.depth != 1):
            raise ValueError("only one-layer MLPs decay as more factors per channel")
        if a in TIED_CONCAT and (self.encoding != "one-hot" or 2 * self.width > MAX_WIDTH):
            raise ValueError(f"tied concatenation needs one-hot encoding and width <= {MAX_WIDTH // 2}")
        if self.encoding != "one-hot" and a not in ("mesh-mlp", "mlp", "bilinear", "residual-mlp",
                                                     "residual-mesh-mlp", "full-mesh-mlp"):
            raise ValueError("rotary roles need one-hot encoding and a positive even width")
        if a == "shared-neighbor-mesh-mlp" and not 1 <= self.embedding_mesh_depth <= MAX_DEPTH:
            raise ValueError("shared Neighbor embedding depth must be in 1..=64")
        if self.mesh_layers() > 0 and self.parents() == 2 and self.width < 2:
            raise ValueError("a second mesh parent needs a width of at least 2")
        if a in ROTARY and (self.width < 2 or self.width % 2):
            raise ValueError("rotary roles need one-hot encoding and a positive even width")
        if self.full_mesh_initialization not in ("kaiming", "identity-hidden"):
            raise ValueError("unknown full-mesh initialization")
        if a == "full-mesh-mlp" and (self.encoding != "binary" or self.connectivity == "own"):
            raise ValueError("a full mesh needs ordinary binary inputs and two-parent connectivity")
        if self.full_mesh_initialization != "kaiming" and a not in ("shared-neighbor-mesh-mlp", "full-mesh-mlp"):
            raise ValueError("only a full mesh configures its mesh initialization")
        if a == "shared-neighbor-mesh-mlp" and (
                self.width < self.modulus or self.width % 2 or self.connectivity == "own"):
            raise ValueError("shared Neighbor meshes need one-hot inputs, even width >= classes, "
                             "two core parents and embedding depth 1..=64")
        if self.mesh_learning_rate_multiplier < 1:
            raise ValueError("the mesh learning rate multiplier must be positive")
        if self.mesh_learning_rate_multiplier != 1 and self.mesh_layers() == 0:
            raise ValueError("only mesh layers multiply their learning rate")
        return self

    # -------------------------------------------------------------- structure
    def parents(self) -> int:
        return 1 if self.connectivity == "own" else 2

    def stride(self, layer: int) -> int:
        """``src/simple/mod.rs:178-186``."""
        if self.connectivity == "own":
            return 0
        if self.connectivity == "neighbor":
            return 1
        return butterfly_stride(self.width, layer)

    def operand_features(self) -> int:
        """``Encoding::features`` (``src/simple/mod.rs:362-370``)."""
        if self.encoding == "one-hot":
            return self.modulus
        if self.encoding == "binary":
            return max((self.modulus - 1).bit_length(), 1)
        return 1 if self.encoding == "scalar" else 2

    def input_features(self) -> int:
        return 2 * self.operand_features()

    def layers(self):
        """Dense (inputs, outputs) layers in parameter order (``:710-756``)."""
        m, w, f = self.modulus, self.width, self.operand_features()
        if self.architecture in ("mesh-mlp", "residual-mesh-mlp"):
            return [(2 * f, w), (w, m)]
        if self.architecture in TIED_CONCAT:
            return [(m, w), (2 * w, w)]
        if self.architecture == "tied-rotary-residual-mesh-mlp":
            return [(m, w)]
        if self.architecture == "mlp":
            return [(2 * f, w)] + [(w, w)] * (self.depth - 1) + [(w, m)]
        if self.architecture == "bilinear":
            return [(f, w), (f, w), (w, m)]
        if self.architecture == "residual-mlp":
            hidden = w * self.expansion
            return [(2 * f, w)] + [(w, hidden), (hidden, w)] * self.depth + [(w, m)]
        if self.architecture == "tied-rotary-residual-dense-mlp":
            return [(m, w)] + [(w, w)] * self.depth
        return []

    def two_parent_layers(self):
        """Full mesh layers as (inputs, outputs, stride) (``:766-800``)."""
        if self.architecture != "full-mesh-mlp":
            return []
        w = self.width
        layers = [(self.input_features(), w, self.operand_features())]
        layers += [(w, w, self.stride(layer - 1)) for layer in range(1, self.depth)]
        return layers + [(w, self.modulus, self.stride(self.depth - 1))]

    def mesh_layers(self) -> int:
        """``:758-765``."""
        if self.architecture in ("mesh-mlp", "tied-concat-mesh-mlp"):
            return self.depth - 1
        if self.architecture in RESIDUAL_MESH:
            return self.depth * self.mesh_depth
        if self.architecture == "full-mesh-mlp":
            return self.depth + 1
        if self.architecture == "shared-neighbor-mesh-mlp":
            return self.embedding_mesh_depth + self.depth
        return 0

    def stored_mesh_layers(self) -> int:
        """``:880-893``: one stored layer when the mesh layers are tied."""
        return min(self.mesh_layers(), 1) if self.tied_mesh else self.mesh_layers()

    def stored_mesh_layer(self, layer: int) -> int:
        return 0 if self.tied_mesh else layer

    def groups(self):
        """Parameter group sizes in storage order (``:871-889``)."""
        if self.architecture == "shared-neighbor-mesh-mlp":
            return [2 * self.width] * self.embedding_mesh_depth + [3 * self.width] * self.depth
        if self.architecture == "full-mesh-mlp":
            return [3 * o for _, o, _ in self.two_parent_layers()]
        g = [i * o for i, o in self.layers()]
        return g + [self.parents() * self.width] * self.stored_mesh_layers()

    def parameter_count(self) -> int:
        return sum(self.groups())

    def group_learning_rate_scale(self):
        """Per group: the learning-rate multiple (``src/simple/gpu.rs:2051-2064``)."""
        if self.architecture == "full-mesh-mlp":
            return [self.mesh_learning_rate_multiplier] * len(self.groups())
        n_dense = len(self.layers())
        return [1 if i < n_dense else self.mesh_learning_rate_multiplier
                for i in range(len(self.groups()))]


# ------------------------------------------------------------------- init
def _box_muller(random: Random):
    radius = math.sqrt(-2.0 * math.log(1.0 - float(random.unit())))
    angle = 2.0 * math.pi * float(random.unit())
    return radius, angle


def initial_parameters(config: SimpleConfig, seed: int) -> np.ndarray:
    """``SimpleConfig::initial_parameters`` (``src/simple/mod.rs:938-1036``)."""
    config.validate()
    random = Random(seed ^ 0x73696D706C650004)
    out = []
    w = config.width
    if config.architecture == "shared-neighbor-mesh-mlp":
        depth = config.embedding_mesh_depth
        ratio = 0.1 / math.sqrt(depth)  # near-identity (``:326-331``)
        own, deviation = 1.0, ratio
        for _ in range(depth * w):
            radius, angle = _box_muller(random)
            out += [np.float32(own), np.float32(deviation * radius * math.cos(angle))]
        for layer in range(config.depth):
            identity = config.full_mesh_initialization == "identity-hidden" and layer > 0
            for _ in range(w):
                if identity:
                    pair = [1.0, 0.0]
                else:
                    radius, angle = _box_muller(random)
                    pair = [radius * math.cos(angle), radius * math.sin(angle)]
                out += [np.float32(pair[0]), np.float32(pair[1]), np.float32(0.0)]
        return np.array(out, dtype=np.float32)
    if config.architecture == "full-mesh-mlp":
        # src/simple/mod.rs:979-1003
        for index, (_, outputs, _) in enumerate(config.two_parent_layers()):
            identity = config.full_mesh_initialization == "identity-hidden" and 0 < index < config.depth
            deviation = math.sqrt(0.5) if index == config.depth else 1.0
            for _ in range(outputs):
                if identity:
                    pair = [1.0, 0.0]
                else:
                    radius, angle = _box_muller(random)
                    pair = [deviation * radius * math.cos(angle), deviation * radius * math.sin(angle)]
                out += [np.float32(pair[0]), np.float32(pair[1]), np.float32(0.0)]
        return np.array(out, dtype=np.float32)
    for index, (inputs, outputs) in enumerate(config.layers()):
        count = inputs * outputs
        if config.architecture == "tied-rotary-residual-dense-mlp" and index > 0:
            deviation = math.sqrt(2.0 / inputs)  # Kaiming normal, fan-in, ReLU gain
            for offset in range(0, count, 2):
                radius, angle = _box_muller(random)
                out.append(np.float32(deviation * radius * math.cos(angle)))
                if offset + 1 < count:
                    out.append(np.float32(deviation * radius * math.sin(angle)))
            continue
        bound = np.float32(1.0) / np.sqrt(np.float32(inputs))
        for _ in range(count):
            out.append((np.float32(2.0) * random.unit() - np.float32(1.0)) * bound)
    unit = [1.0, 0.0][:config.parents()]
    for _ in range(config.stored_mesh_layers() * w):
        out += unit
    return np.array(out, dtype=np.float32)


def primitive_root(modulus: int) -> int:
    """The smallest primitive root (``src/simple/mod.rs:444-456``)."""
    for root in range(1, modulus):
        seen, value = [False] * modulus, 1
        for _ in range(modulus - 1):
            seen[value] = True
            value = value * root % modulus
        if all(seen[1:]):
            return root
    raise ValueError("discrete logarithms require a prime modulus")


def encoding_table(config: SimpleConfig) -> np.ndarray:
    """``Encoding::table`` (``src/simple/mod.rs:373-414``): one feature row
    per residue, float32 [modulus][operand_features]."""
    m, f = config.modulus, config.operand_features()
    table = np.zeros((m, f), dtype=np.float32)
    if config.encoding == "one-hot":
        table[np.arange(m), np.arange(m)] = 1.0
    elif config.encoding == "binary":
        for value in range(m):
            table[value] = [1.0 if value >> bit & 1 else -1.0 for bit in range(f)]
    elif config.encoding == "scalar":
        middle = (m - 1) / 2.0
        table[:, 0] = [np.float32((value - middle) / middle) for value in range(m)]
    else:
        root, logs, value = primitive_root(m), [0] * m, 1
        for exponent in range(m - 1):
            logs[value] = exponent
            value = value * root % m
        middle = (m - 2) / 2.0
        for value in range(m):
            if value == 0:
                table[value] = [1.0, 0.0]
            elif middle == 0.0:
                table[value] = [0.0, 0.0]
            else:
                table[value] = [0.0, np.float32((logs[value] - middle) / middle)]
    return table


def encode(config: SimpleConfig, equations):
    """``[a | b]`` feature rows of the configured encoding and answer
    classes (``:1039-1055``)."""
    m = config.modulus
    table = encoding_table(config)
    rows = len(equations)
    features = np.zeros((rows, 2 * table.shape[1]), dtype=np.float32)
    targets = np.zeros(rows, dtype=np.uint32)
    for r, (a, b, answer) in enumerate(equations):
        if a >= m or b >= m or answer >= m:
            raise ValueError("equation residue is outside the model's modulus")
        features[r] = np.concatenate([table[a], table[b]])
        targets[r] = answer
    return features, targets


# ----------------------------------------------------------------- operators
def _act(config, x):
    return np.maximum(x, 0.0) if config.activation == "relu" else x * x


def _act_grad(config, x):
    return (x > 0.0).astype(np.float64) if config.activation == "relu" else 2.0 * x


def _rmsnorm(x):
    inv = 1.0 / np.sqrt((x * x).mean(axis=1) + EPS)
    return x * inv[:, None], inv


def _rmsnorm_backward(y, inv, dy):
    dot = (dy * y).sum(axis=1, keepdims=True)
    return inv[:, None] * (dy - y * dot / y.shape[1])


def _rotation(width):
    """Rotate90 roles: channel c takes b's channel c^1, negated for even c."""
    perm = np.arange(width) ^ 1
    sign = np.where(np.arange(width) % 2 == 0, -1.0, 1.0)
    return perm, sign


def _split(config, parameters):
    p = np.asarray(parameters, dtype=np.float64)
    groups, out, offset = config.groups(), [], 0
    for size in groups:
        out.append(p[offset:offset + size])
        offset += size
    return out


# ------------------------------------------------------------------ model
class ReferenceSimpleModel:
    """f64 forward / loss / gradient of ``src/simple/reference.rs:143-448``."""

    def __init__(self, config: SimpleConfig, parameters=None, seed: int = 11, fp32_kink: bool = False):
        """``fp32_kink``: decide ReLU's kink (slope 1 above 0, else 0, as
        ``simple_slope`` at src/simple/gpu.rs:62-72 and the tape's relu at
        src/gpt/reference.rs:318-324) on the pre-activation rounded to f32,
        as any FP32 implementation of the model does.  It matters only where
        the f64 pre-activation is below f32's range: the shared-Neighbor
        model's near-identity chain makes values such as 1e-50 (products of
        its small mixing weights) that FP32 holds as exactly 0."""
        self.fp32_kink = fp32_kink
        self.kink_band = None  # (band, slope): ReLU slope for nonzero |pre-activation| <= band
        self.config = config.validate()
        self.parameters = (initial_parameters(config, seed) if parameters is None
                           else np.asarray(parameters, dtype=np.float32).copy())
        if self.parameters.size != config.parameter_count():
            raise ValueError("parameter count does not match the model")

    def _slope(self, x):
        if self.kink_band is not None and self.config.activation == "relu":
            band, value = self.kink_band
            x = np.asarray(x)
            return np.where((np.abs(x) <= band) & (x != 0.0), value, (x > 0.0).astype(np.float64))
        if self.fp32_kink and self.config.activation == "relu":
            return (np.asarray(x).astype(np.float32) > 0.0).astype(np.float64)
        return _act_grad(self.config, x)

    # forward returns logits [rows][modulus] and a cache for the backward
    def _forward(self, features):
        c = self.config
        x = np.asarray(features, dtype=np.float64)
        g = _split(c, self.parameters)
        m, w = c.modulus, c.width
        if c.architecture == "mlp":
            # src/simple/reference.rs:292-299
            zs = [x @ g[0].reshape(-1, w)]
            acts = []
            for layer in range(1, c.depth + 1):
                acts.append(_act(c, zs[-1]))
                out = c.layers()[layer][1]
                zs.append(acts[-1] @ g[layer].reshape(-1, out))
            return zs[-1], dict(x=x, zs=zs, acts=acts)
        if c.architecture == "residual-mlp":
            # src/simple/reference.rs:418-433
            hidden = w * c.expansion
            h = x @ g[0].reshape(-1, w)
            blocks = []
            for block in range(c.depth):
                n, inv = _rmsnorm(h)
                e = n @ g[1 + 2 * block].reshape(w, hidden)
                act = _act(c, e)
                blocks.append((n, inv, e, act))
                h = h + act @ g[2 + 2 * block].reshape(hidden, w)
            hf, invf = _rmsnorm(h)
            return hf @ g[1 + 2 * c.depth].reshape(w, m), dict(x=x, blocks=blocks, hf=hf, invf=invf)
        if c.architecture == "bilinear":
            # src/simple/reference.rs:434-444
            f = c.operand_features()
            left, right = x[:, :f] @ g[0].reshape(f, w), x[:, f:] @ g[1].reshape(f, w)
            prod = left * right
            return prod @ g[2].reshape(w, m), dict(x=x, left=left, right=right, prod=prod)
        if c.architecture == "mesh-mlp":
            w0 = g[0].reshape(-1, w)
            readout = g[1].reshape(w, m)
            h = [x @ w0]
            for layer in range(c.mesh_layers()):
                mw = g[2 + c.stored_mesh_layer(layer)].reshape(w, c.parents())
                act = _act(c, h[-1])
                y = act * mw[:, 0]
                if c.parents() == 2:
                    y = y + np.roll(act, -c.stride(layer), axis=1) * mw[:, 1]
                h.append(y)
            act = _act(c, h[-1])
            return act @ readout, dict(x=x, h=h, act=act)
        if c.architecture == "tied-concat-mesh-mlp":
            # src/simple/reference.rs:300-335 (tied)
            emb = g[0].reshape(m, w)
            j = np.concatenate([x[:, :m] @ emb, x[:, m:] @ emb], axis=1)
            h = [j @ g[1].reshape(2 * w, w)]
            for layer in range(c.mesh_layers()):
                mw = g[2 + c.stored_mesh_layer(layer)].reshape(w, c.parents())
                act = _act(c, h[-1])
                y = act * mw[:, 0]
                if c.parents() == 2:
                    y = y + np.roll(act, -c.stride(layer), axis=1) * mw[:, 1]
                h.append(y)
            act = _act(c, h[-1])
            return act @ emb.T, dict(x=x, j=j, h=h, act=act, emb=emb)
        if c.architecture in RESIDUAL_MESH:
            return self._residual_mesh_forward(x, g)
        if c.architecture == "full-mesh-mlp":
            # src/simple/reference.rs:271-290
            zs, h = [], x
            for index, (inputs, outputs, stride) in enumerate(c.two_parent_layers()):
                xin = h if index == 0 else _act(c, h)
                p = g[index].reshape(outputs, 3)
                a, b = two_parents(inputs, outputs, stride)
                h = xin[:, a] * p[:, 0] + xin[:, b] * p[:, 1] + p[:, 2]
                zs.append(h)
            return h, dict(x=x, zs=zs)
        perm, sign = _rotation(w)
        if c.architecture == "tied-rotary-residual-dense-mlp":
            emb = g[0].reshape(m, w)
            left, right = x[:, :m] @ emb, x[:, m:] @ emb
            h = left + right[:, perm] * sign
            blocks = []
            for block in range(c.depth):
                n, inv = _rmsnorm(h)
                z = n @ g[1 + block].reshape(w, w)
                blocks.append((h, n, inv, z))
                h = h + _act(c, z)
            hf, invf = _rmsnorm(h)
            return hf @ emb.T, dict(x=x, blocks=blocks, hf=hf, invf=invf, emb=emb)
        # shared-neighbor-mesh-mlp
        ed = c.embedding_mesh_depth
        chain = [g[i].reshape(w, 2) for i in range(ed)]
        core = [g[ed + i].reshape(w, 3) for i in range(c.depth)]
        rows = x.shape[0]

        def embed(v):
            v = np.concatenate([v, np.zeros((rows, w - m))], axis=1)
            states = [v]
            for layer in range(ed):
                v = v * chain[layer][:, 0] + np.roll(v, -1, axis=1) * chain[layer][:, 1]
                states.append(v)
            return states

        ls, rs = embed(x[:, :m]), embed(x[:, m:])
        h = ls[-1] + rs[-1][:, perm] * sign
        blocks = []
        for layer in range(c.depth):
            n, inv = _rmsnorm(h)
            p = core[layer]
            z = n * p[:, 0] + np.roll(n, -c.stride(layer), axis=1) * p[:, 1] + p[:, 2]
            blocks.append((h, n, inv, z))
            h = h + _act(c, z)
        hf, invf = _rmsnorm(h)
        # transposed chain, last embedding layer first
        reads = []
        y = hf
        for layer in reversed(range(ed)):
            reads.append(y)
            y = y * chain[layer][:, 0] + np.roll(y * chain[layer][:, 1], 1, axis=1)
        return y[:, :m], dict(x=x, ls=ls, rs=rs, blocks=blocks, hf=hf, invf=invf, reads=reads,
                              chain=chain, core=core)

    def _residual_mesh_forward(self, x, g):
        """``src/simple/reference.rs:337-407`` for the residual mesh family."""
        c = self.config
        m, w, md, nd = c.modulus, c.width, c.mesh_depth, len(c.layers())
        emb = j = None
        if c.architecture == "tied-rotary-residual-mesh-mlp":
            perm, sign = _rotation(w)
            emb = g[0].reshape(m, w)
            h = x[:, :m] @ emb + (x[:, m:] @ emb)[:, perm] * sign
        elif c.architecture == "tied-concat-residual-mesh-mlp":
            emb = g[0].reshape(m, w)
            j = np.concatenate([x[:, :m] @ emb, x[:, m:] @ emb], axis=1)
            h = j @ g[1].reshape(2 * w, w)
        else:
            h = x @ g[0].reshape(-1, w)
        blocks = []
        for block in range(c.depth):
            n, inv = _rmsnorm(h)
            branch, zs = n, []
            for layer in range(md):
                if layer > 0:
                    branch = _act(c, branch)
                mesh = block * md + layer
                mw = g[nd + mesh].reshape(w, c.parents())
                z = branch * mw[:, 0]
                if c.parents() == 2:
                    z = z + np.roll(branch, -c.stride(mesh), axis=1) * mw[:, 1]
                zs.append(z)
                branch = z
            if c.mesh_output_activation:
                branch = _act(c, branch)
            blocks.append((n, inv, zs))
            h = h + branch
        hf, invf = _rmsnorm(h)
        logits = hf @ emb.T if emb is not None else hf @ g[1].reshape(w, m)
        return logits, dict(x=x, j=j, emb=emb, blocks=blocks, hf=hf, invf=invf)

    def _residual_mesh_backward(self, s, g, grads, dlog):
        c = self.config
        m, w, md, nd = c.modulus, c.width, c.mesh_depth, len(c.layers())
        x, emb = s["x"], s["emb"]
        if emb is not None:
            demb = dlog.T @ s["hf"]
            dh = _rmsnorm_backward(s["hf"], s["invf"], dlog @ emb)
        else:
            grads[1] = (s["hf"].T @ dlog).reshape(-1)
            dh = _rmsnorm_backward(s["hf"], s["invf"], dlog @ g[1].reshape(w, m).T)
        for block in reversed(range(c.depth)):
            n, inv, zs = s["blocks"][block]
            dz = dh * self._slope(zs[-1]) if c.mesh_output_activation else dh
            for layer in reversed(range(md)):
                mesh = block * md + layer
                xin = n if layer == 0 else _act(c, zs[layer - 1])
                mw = g[nd + mesh].reshape(w, c.parents())
                gw = np.zeros((w, c.parents()))
                gw[:, 0] = (dz * xin).sum(axis=0)
                dx = dz * mw[:, 0]
                if c.parents() == 2:
                    st = c.stride(mesh)
                    gw[:, 1] = (dz * np.roll(xin, -st, axis=1)).sum(axis=0)
                    dx = dx + np.roll(dz * mw[:, 1], st, axis=1)
                grads[nd + mesh] = gw.reshape(-1)
                dz = dx * self._slope(zs[layer - 1]) if layer > 0 else dx
            dh = dh + _rmsnorm_backward(n, inv, dz)
        if c.architecture == "tied-rotary-residual-mesh-mlp":
            perm, sign = _rotation(w)
            dright = np.empty_like(dh)
            dright[:, perm] = dh * sign
            grads[0] = (demb + x[:, :m].T @ dh + x[:, m:].T @ dright).reshape(-1)
        elif c.architecture == "tied-concat-residual-mesh-mlp":
            grads[1] = (s["j"].T @ dh).reshape(-1)
            dj = dh @ g[1].reshape(2 * w, w).T
            grads[0] = (demb + x[:, :m].T @ dj[:, :w] + x[:, m:].T @ dj[:, w:]).reshape(-1)
        else:
            grads[0] = (x.T @ dh).reshape(-1)

    def logits(self, features) -> np.ndarray:
        return self._forward(features)[0]

    @staticmethod
    def row_losses(logits, targets):
        z = logits - logits.max(axis=1, keepdims=True)
        lse = np.log(np.exp(z).sum(axis=1))
        return lse - z[np.arange(len(targets)), targets]

    def loss_and_gradient(self, features, targets):
        """Mean answer cross-entropy and its f64 gradient (``:51-67,135-151``)."""
        c = self.config
        targets = np.asarray(targets, dtype=np.int64)
        logits, s = self._forward(features)
        rows = logits.shape[0]
        loss = float(self.row_losses(logits, targets).mean())
        p = np.exp(logits - logits.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        dlog = p
        dlog[np.arange(rows), targets] -= 1.0
        dlog /= rows
        g = _split(c, self.parameters)
        grads = [np.zeros_like(x) for x in g]
        m, w = c.modulus, c.width
        if c.architecture == "mlp":
            dz = dlog
            for layer in range(c.depth, 0, -1):
                out = c.layers()[layer][1]
                grads[layer] = (s["acts"][layer - 1].T @ dz).reshape(-1)
                dz = (dz @ g[layer].reshape(-1, out).T) * self._slope(s["zs"][layer - 1])
            grads[0] = (s["x"].T @ dz).reshape(-1)
            return loss, np.concatenate(grads)
        if c.architecture == "residual-mlp":
            hidden, d = w * c.expansion, c.depth
            readout = g[1 + 2 * d].reshape(w, m)
            grads[1 + 2 * d] = (s["hf"].T @ dlog).reshape(-1)
            dh = _rmsnorm_backward(s["hf"], s["invf"], dlog @ readout.T)
            for block in reversed(range(d)):
                n, inv, e, act = s["blocks"][block]
                down = g[2 + 2 * block].reshape(hidden, w)
                up = g[1 + 2 * block].reshape(w, hidden)
                grads[2 + 2 * block] = (act.T @ dh).reshape(-1)
                de = (dh @ down.T) * self._slope(e)
                grads[1 + 2 * block] = (n.T @ de).reshape(-1)
                dh = dh + _rmsnorm_backward(n, inv, de @ up.T)
            grads[0] = (s["x"].T @ dh).reshape(-1)
            return loss, np.concatenate(grads)
        if c.architecture == "bilinear":
            f = c.operand_features()
            grads[2] = (s["prod"].T @ dlog).reshape(-1)
            dp = dlog @ g[2].reshape(w, m).T
            grads[0] = (s["x"][:, :f].T @ (dp * s["right"])).reshape(-1)
            grads[1] = (s["x"][:, f:].T @ (dp * s["left"])).reshape(-1)
            return loss, np.concatenate(grads)
        if c.architecture == "mesh-mlp":
            readout = g[1].reshape(w, m)
            grads[1] = (s["act"].T @ dlog).reshape(-1)
            dh = (dlog @ readout.T) * self._slope(s["h"][-1])
            for layer in reversed(range(c.mesh_layers())):
                mw = g[2 + c.stored_mesh_layer(layer)].reshape(w, c.parents())
                hin = s["h"][layer]
                act = _act(c, hin)
                gw = np.zeros((w, c.parents()))
                gw[:, 0] = (dh * act).sum(axis=0)
                dact = dh * mw[:, 0]
                if c.parents() == 2:
                    st = c.stride(layer)
                    gw[:, 1] = (dh * np.roll(act, -st, axis=1)).sum(axis=0)
                    dact = dact + np.roll(dh * mw[:, 1], st, axis=1)
                grads[2 + c.stored_mesh_layer(layer)] = grads[2 + c.stored_mesh_layer(layer)] + gw.reshape(-1)
                dh = dact * self._slope(hin)
            grads[0] = (s["x"].T @ dh).reshape(-1)
            return loss, np.concatenate(grads)
        if c.architecture == "tied-concat-mesh-mlp":
            emb = s["emb"]
            demb = dlog.T @ s["act"]
            dh = (dlog @ emb) * self._slope(s["h"][-1])
            for layer in reversed(range(c.mesh_layers())):
                mw = g[2 + c.stored_mesh_layer(layer)].reshape(w, c.parents())
                hin = s["h"][layer]
                act = _act(c, hin)
                gw = np.zeros((w, c.parents()))
                gw[:, 0] = (dh * act).sum(axis=0)
                dact = dh * mw[:, 0]
                if c.parents() == 2:
                    st = c.stride(layer)
                    gw[:, 1] = (dh * np.roll(act, -st, axis=1)).sum(axis=0)
                    dact = dact + np.roll(dh * mw[:, 1], st, axis=1)
                grads[2 + c.stored_mesh_layer(layer)] = grads[2 + c.stored_mesh_layer(layer)] + gw.reshape(-1)
                dh = dact * self._slope(hin)
            grads[1] = (s["j"].T @ dh).reshape(-1)
            dj = dh @ g[1].reshape(2 * w, w).T
            x = s["x"]
            grads[0] = (demb + x[:, :m].T @ dj[:, :w] + x[:, m:].T @ dj[:, w:]).reshape(-1)
            return loss, np.concatenate(grads)
        if c.architecture in RESIDUAL_MESH:
            self._residual_mesh_backward(s, g, grads, dlog)
            return loss, np.concatenate(grads)
        if c.architecture == "full-mesh-mlp":
            layers, dz = c.two_parent_layers(), dlog
            for index in reversed(range(len(layers))):
                inputs, outputs, stride = layers[index]
                xin = s["x"] if index == 0 else _act(c, s["zs"][index - 1])
                p = g[index].reshape(outputs, 3)
                a, b = two_parents(inputs, outputs, stride)
                grads[index] = np.stack([(dz * xin[:, a]).sum(axis=0), (dz * xin[:, b]).sum(axis=0),
                                         dz.sum(axis=0)], axis=1).reshape(-1)
                if index > 0:
                    dx = np.zeros_like(xin)
                    np.add.at(dx.T, a, (dz * p[:, 0]).T)
                    np.add.at(dx.T, b, (dz * p[:, 1]).T)
                    dz = dx * self._slope(s["zs"][index - 1])
            return loss, np.concatenate(grads)
        perm, sign = _rotation(w)
        x = s["x"]
        if c.architecture == "tied-rotary-residual-dense-mlp":
            emb = s["emb"]
            demb = dlog.T @ s["hf"]
            dh = _rmsnorm_backward(s["hf"], s["invf"], dlog @ emb)
            for block in reversed(range(c.depth)):
                hin, n, inv, z = s["blocks"][block]
                dz = dh * self._slope(z)
                d = g[1 + block].reshape(w, w)
                grads[1 + block] = (n.T @ dz).reshape(-1)
                dh = dh + _rmsnorm_backward(n, inv, dz @ d.T)
            dright = np.empty_like(dh)
            dright[:, perm] = dh * sign
            demb = demb + x[:, :m].T @ dh + x[:, m:].T @ dright
            grads[0] = demb.reshape(-1)
            return loss, np.concatenate(grads)
        ed = c.embedding_mesh_depth
        chain, core = s["chain"], s["core"]
        gchain = [np.zeros((w, 2)) for _ in range(ed)]
        dy = np.zeros((rows, w))
        dy[:, :m] = dlog
        # back through the transposed chain: layers 0, 1, ..., ed-1
        for layer in range(ed):
            hin = s["reads"][ed - 1 - layer]
            nxt = np.roll(dy, -1, axis=1)
            gchain[layer][:, 0] += (hin * dy).sum(axis=0)
            gchain[layer][:, 1] += (hin * nxt).sum(axis=0)
            dy = dy * chain[layer][:, 0] + nxt * chain[layer][:, 1]
        dh = _rmsnorm_backward(s["hf"], s["invf"], dy)
        for layer in reversed(range(c.depth)):
            hin, n, inv, z = s["blocks"][layer]
            p = core[layer]
            st = c.stride(layer)
            dz = dh * self._slope(z)
            gp = np.stack([(dz * n).sum(axis=0), (dz * np.roll(n, -st, axis=1)).sum(axis=0),
                           dz.sum(axis=0)], axis=1)
            grads[ed + layer] = gp.reshape(-1)
            dn = dz * p[:, 0] + np.roll(dz * p[:, 1], st, axis=1)
            dh = dh + _rmsnorm_backward(n, inv, dn)
        dright = np.empty_like(dh)
        dright[:, perm] = dh * sign
        for states, dv in ((s["ls"], dh), (s["rs"], dright)):
            for layer in reversed(range(ed)):
                v = states[layer]
                gchain[layer][:, 0] += (dv * v).sum(axis=0)
                gchain[layer][:, 1] += (dv * np.roll(v, -1, axis=1)).sum(axis=0)
                dv = dv * chain[layer][:, 0] + np.roll(dv * chain[layer][:, 1], 1, axis=1)
        for layer in range(ed):
            grads[layer] = gchain[layer].reshape(-1)
        return loss, np.concatenate(grads)


def channel_decays(config: SimpleConfig, parameters, learning_rate, weight_decay):
    """Per-parameter decay of a one-layer MLP with ``decay_factors`` n != 2
    (``src/simple/gpu.rs:814-881``, checked on the host at ``:3800-3820``):
    channel c's input column and readout row decay at
    min(wd s_c^(2/n - 1), 1 / lr) with s_c = (|E_c|^2 + |R_c|^2) / 2 over the
    weights before the step, all in f32."""
    f = np.float32
    w, m = config.width, config.modulus
    p = np.asarray(parameters, dtype=np.float32)
    n_in = config.layers()[0][0] * w
    inputs, readout = p[:n_in].reshape(-1, w), p[n_in:].reshape(w, m)
    squares = np.zeros(w, dtype=np.float32)
    for row in inputs:
        squares = squares + row * row
    for k in range(m):
        squares = squares + readout[:, k] * readout[:, k]
    exponent = f(2.0 / config.decay_factors - 1.0)
    scale = np.power(np.maximum(f(0.5) * squares, f(np.finfo(np.float32).tiny)), exponent).astype(np.float32)
    channel = np.minimum(f(weight_decay) * scale, f(1.0) / f(learning_rate)).astype(np.float32)
    return np.concatenate([np.tile(channel, inputs.shape[0]), np.repeat(channel, m)]).astype(np.float32)


# ------------------------------------------------------------------ records
def row_metrics(logits, targets):
    """Per-row f64 cross-entropy from (f32) logits and the first maximum
    (``src/bin/mesh-gpt/grokking.rs:544-557``)."""
    lg = np.asarray(logits, dtype=np.float64)
    pred = lg.argmax(axis=1)
    mx = lg[np.arange(lg.shape[0]), pred]
    ce = np.log(np.exp(lg - mx[:, None]).sum(axis=1)) + mx - lg[np.arange(lg.shape[0]), targets]
    return ce, pred


def record(model: ReferenceSimpleModel, splits):
    """(train CE, validation CE, train accuracy, validation accuracy, weight L2)
    of one ``loss.csv`` line (``src/bin/mesh-gpt/simple.rs:807-860``)."""
    out = []
    accs = []
    for features, targets in splits:
        ce, pred = row_metrics(model.logits(features), targets)
        out.append(float(ce.sum() / len(targets)))
        accs.append(float((pred == targets).sum()) / len(targets))
    norm = math.sqrt(float((model.parameters.astype(np.float64) ** 2).sum()))
    return out[0], out[1], accs[0], accs[1], norm


def train_records(config: SimpleConfig, operation: str = "div", train_fraction: float = 0.5,
                  seed: int = 11, steps: int = 10, batch: int = 512, learning_rate: float = 1e-3,
                  weight_decay: float = 1.0, beta1: float = 0.9, beta2: float = 0.98,
                  epsilon: float = 1e-8):
    """The step-0 and step-``steps`` records of ``grok-simple``: a seeded
    split, ``EquationSampler`` minibatches drawn one epoch at a time with a
    short tail, a 10-step linear warmup and AdamW in f32
    (``src/bin/mesh-gpt/simple.rs:242-330,540-620``)."""
    dataset = EquationDataset(config.modulus, operation, train_fraction, seed)
    splits = [encode(config, dataset.split(v)) for v in (False, True)]
    model = ReferenceSimpleModel(config, seed=seed)
    records = [record(model, splits)]
    n_train = len(dataset.split(False))
    sampler = EquationSampler(n_train, seed)
    steps_per_epoch = -(-n_train // batch)
    m = np.zeros(config.parameter_count(), dtype=np.float32)
    v = np.zeros(config.parameter_count(), dtype=np.float32)
    b1p, b2p = np.float32(1.0), np.float32(1.0)
    scales = np.repeat(np.array(config.group_learning_rate_scale(), dtype=np.float32),
                       config.groups())
    features, targets = splits[0]
    step, epoch = 0, []
    while step < steps:
        if not epoch:
            epoch = [sampler.sample(batch) for _ in range(min(steps_per_epoch, steps - step))]
        rows = epoch.pop(0)
        step += 1
        lr = warmed_learning_rate(learning_rate, step)
        _, grad = model.loss_and_gradient(features[rows], targets[rows])
        b1p, b2p = np.float32(b1p * np.float32(beta1)), np.float32(b2p * np.float32(beta2))
        p = model.parameters
        if config.decay_factors != 2:
            decays = channel_decays(config, p, lr, weight_decay)
            adamw_step(p, m, v, grad, step, lr, decays, beta1, beta2, epsilon, (b1p, b2p))
        elif np.all(scales == 1):
            adamw_step(p, m, v, grad, step, lr, weight_decay, beta1, beta2, epsilon, (b1p, b2p))
        else:
            for scale in np.unique(scales):
                sel = scales == scale
                ps, ms, vs = p[sel], m[sel], v[sel]
                adamw_step(ps, ms, vs, grad[sel], step, np.float32(lr * scale), weight_decay,
                           beta1, beta2, epsilon, (b1p, b2p))
                p[sel], m[sel], v[sel] = ps, ms, vs
    records.append(record(model, splits))
    return records
