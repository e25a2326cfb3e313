"""grok-simple models on the B200 through ``libmeshb200.so``.

Python mirror of the reference's ``SimpleConfig`` (src/simple/mod.rs:500-1055)
and ``GpuSimpleModel`` (src/simple/gpu.rs:1757-2073): same names, argument
meaning and error behaviour (a nonzero library status raises
``MeshError``).  Eleven architectures run on this path: ``mesh-mlp``,
``tied-rotary-residual-dense-mlp``, ``shared-neighbor-mesh-mlp``, ``mlp``,
``bilinear``, ``residual-mlp``, ``residual-mesh-mlp``,
``tied-concat-residual-mesh-mlp``, ``tied-rotary-residual-mesh-mlp`` and
``tied-concat-mesh-mlp`` and ``full-mesh-mlp``, with one-hot or encoded operands.  There is no CPU
fallback.
"""

import ctypes
import math
import weakref
from dataclasses import dataclass, replace

import numpy as np

from . import _lib
from ._lib import AdamWC, SimpleConfigC, check, ptr
from .data import EquationDataset, EquationSampler
from .gpt import AdamWOptions

ARCHITECTURES = ("mesh-mlp", "tied-rotary-residual-dense-mlp", "shared-neighbor-mesh-mlp", "mlp", "bilinear",
                 "residual-mlp", "residual-mesh-mlp", "tied-concat-residual-mesh-mlp",
                 "tied-rotary-residual-mesh-mlp", "tied-concat-mesh-mlp", "full-mesh-mlp")
ACTIVATIONS = ("relu", "square")
ENCODINGS = ("one-hot", "binary", "scalar", "discrete-log")
CONNECTIVITIES = ("own", "neighbor", "butterfly")
INITIALIZATIONS = ("kaiming", "identity-hidden")


@dataclass(frozen=True)
class SimpleConfig:
    """``SimpleConfig`` fields read by the eleven architectures (reference
    defaults)."""
    architecture: str = "mesh-mlp"
    activation: str = "relu"
    modulus: int = 97
    width: int = 128
    depth: int = 1
    connectivity: str = "neighbor"
    embedding_mesh_depth: int = 4
    full_mesh_initialization: str = "kaiming"
    mesh_learning_rate_multiplier: int = 1
    expansion: int = 4
    mesh_depth: int = 4
    mesh_output_activation: bool = False
    tied_mesh: bool = False
    encoding: str = "one-hot"
    decay_factors: int = 2

    def with_(self, **kw):
        return replace(self, **kw)

    def operand_features(self) -> int:
        """Features per operand of the encoding (``Encoding::features``)."""
        if self.encoding == "one-hot":
            return self.modulus
        if self.encoding == "binary":
            return max((self.modulus - 1).bit_length(), 1)
        return 1 if self.encoding == "scalar" else 2

    def to_c(self) -> SimpleConfigC:
        def index(names, value, what):
            if value not in names:
                raise ValueError(f"unknown {what}: {value}")
            return names.index(value)
        return SimpleConfigC(index(ARCHITECTURES, self.architecture, "model"),
                             index(ACTIVATIONS, self.activation, "activation"), self.modulus, self.width,
                             self.depth, index(CONNECTIVITIES, self.connectivity, "mesh connectivity"),
                             self.embedding_mesh_depth,
                             index(INITIALIZATIONS, self.full_mesh_initialization, "full-mesh initialization"),
                             self.mesh_learning_rate_multiplier, self.expansion, self.mesh_depth,
                             int(self.mesh_output_activation), int(self.tied_mesh),
                             index(ENCODINGS, self.encoding, "encoding"), self.decay_factors)

    def validate(self):
        c = self.to_c()
        check(_lib.load().mb_simple_validate(ctypes.byref(c)))
        return self

    def parameter_count(self) -> int:
        c, n = self.to_c(), ctypes.c_size_t()
        check(_lib.load().mb_simple_parameter_count(ctypes.byref(c), ctypes.byref(n)))
        return n.value

    def groups(self):
        lib, c, n = _lib.load(), self.to_c(), ctypes.c_size_t()
        check(lib.mb_simple_groups(ctypes.byref(c), None, ctypes.byref(n)))
        out = np.empty(n.value, dtype=np.uint32)
        check(lib.mb_simple_groups(ctypes.byref(c), ptr(out, ctypes.c_uint32), ctypes.byref(n)))
        return [int(g) for g in out]

    def initial_parameters(self, seed: int) -> np.ndarray:
        c = self.to_c()
        out = np.empty(self.parameter_count(), dtype=np.float32)
        check(_lib.load().mb_simple_initial_parameters(ctypes.byref(c), seed, ptr(out, ctypes.c_float), out.size))
        return out

    def encode(self, equations):
        """One-hot ``[a | b]`` rows and answer classes of (a, b, answer) triples."""
        eq = np.ascontiguousarray(np.asarray(equations, dtype=np.uint32).reshape(-1, 3))
        c = self.to_c()
        features = np.empty((len(eq), 2 * self.operand_features()), dtype=np.float32)
        targets = np.empty(len(eq), dtype=np.uint32)
        check(_lib.load().mb_simple_encode(ctypes.byref(c), ptr(eq, ctypes.c_uint32), len(eq),
                                           ptr(features, ctypes.c_float), ptr(targets, ctypes.c_uint32)))
        return features, targets


def pinned_empty(count: int, dtype=np.float32) -> np.ndarray:
    """A numpy array of ``count`` elements in page-locked host memory
    (``PinnedHostBuffer``), freed when the last view of it is gone."""
    lib = _lib.load()
    nbytes = max(1, int(count) * np.dtype(dtype).itemsize)
    p = ctypes.c_void_p()
    check(lib.mb_host_alloc(nbytes, ctypes.byref(p)))
    raw = (ctypes.c_byte * nbytes).from_address(p.value)
    weakref.finalize(raw, lib.mb_host_free, ctypes.c_void_p(p.value))
    return np.frombuffer(raw, dtype=dtype, count=int(count))


class DeviceTable:
    """Encoded rows resident on the device (``DeviceTable``)."""

    def __init__(self, model, handle, rows, targets):
        self._model, self._handle, self.rows, self.targets = model, handle, rows, targets

    def __del__(self):
        if getattr(self, "_handle", None):
            try:
                _lib.load().mb_simple_table_destroy(self._handle)
            except TypeError:  # interpreter shutdown: the library is already gone
                pass
            self._handle = None


class DeviceBatches:
    """Minibatch row indices resident on the device (``DeviceBatches``)."""

    def __init__(self, model, handle, count):
        self._model, self._handle, self.count = model, handle, count

    def __len__(self):
        return self.count

    def __del__(self):
        if getattr(self, "_handle", None):
            try:
                _lib.load().mb_simple_batches_destroy(self._handle)
            except TypeError:  # interpreter shutdown: the library is already gone
                pass
            self._handle = None


class GpuSimpleModel:
    """``GpuSimpleModel``: parameters, AdamW state and workspaces on one GPU."""

    def __init__(self, device: int, config: SimpleConfig, seed: int):
        self.config = config
        self._lib = _lib.load()
        c = config.to_c()
        h = ctypes.c_void_p()
        check(self._lib.mb_simple_create(device, ctypes.byref(c), seed, ctypes.byref(h)))
        self._h = h
        self._count = config.parameter_count()
        self._host_buffers = []  # page-locked float32 buffers returned by reuse()

    def close(self):
        if getattr(self, "_h", None):
            self._lib.mb_simple_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def parameters(self) -> np.ndarray:
        out = np.empty(self._count, dtype=np.float32)
        check(self._lib.mb_simple_get_parameters(self._h, ptr(out, ctypes.c_float), out.size))
        return out

    def _take_pinned(self, count: int) -> np.ndarray:
        for i, b in enumerate(self._host_buffers):
            if b.size >= count:
                return self._host_buffers.pop(i)[:count]
        return pinned_empty(count)

    def pinned_parameters(self) -> np.ndarray:
        """``parameters`` in page-locked memory that ``reuse`` takes back
        (src/simple/gpu.rs:1827-1836)."""
        out = self._take_pinned(self._count)
        check(self._lib.mb_simple_get_parameters(self._h, ptr(out, ctypes.c_float), out.size))
        return out

    def reuse(self, buffer: np.ndarray) -> None:
        """Takes back the page-locked logits or parameters of earlier results
        so that later copies skip allocating them (src/simple/gpu.rs:1838-1842)."""
        if buffer.dtype == np.float32 and buffer.flags.c_contiguous:
            self._host_buffers.append(buffer.reshape(-1))

    def set_parameters(self, values):
        """Sets the weights and resets AdamW's moments and step count."""
        v = np.ascontiguousarray(values, dtype=np.float32)
        check(self._lib.mb_simple_set_parameters(self._h, ptr(v, ctypes.c_float), v.size))

    def upload_table(self, features, targets) -> DeviceTable:
        f = np.ascontiguousarray(features, dtype=np.float32)
        t = np.ascontiguousarray(targets, dtype=np.uint32)
        if f.size != t.size * 2 * self.config.operand_features():
            raise ValueError("each table row needs the model's input features")
        h = ctypes.c_void_p()
        check(self._lib.mb_simple_upload_table(self._h, ptr(f, ctypes.c_float), ptr(t, ctypes.c_uint32), t.size,
                                               ctypes.byref(h)))
        return DeviceTable(self, h, t.size, t)

    def upload_batches(self, table: DeviceTable, indices) -> DeviceBatches:
        idx = np.ascontiguousarray(indices, dtype=np.uint32)
        h = ctypes.c_void_p()
        check(self._lib.mb_simple_upload_batches(self._h, table._handle, ptr(idx, ctypes.c_uint32), idx.size,
                                                 ctypes.byref(h)))
        return DeviceBatches(self, h, idx.size)

    def evaluate(self, *tables):
        """(logits [rows][modulus], first-maximum predictions [rows]) per table."""
        out = []
        for table in tables:
            logits = self._take_pinned(table.rows * self.config.modulus).reshape(table.rows, self.config.modulus)
            preds = np.empty(table.rows, dtype=np.uint32)
            check(self._lib.mb_simple_evaluate(self._h, table._handle, ptr(logits, ctypes.c_float),
                                               ptr(preds, ctypes.c_uint32)))
            out.append((logits, preds))
        return out

    def logits(self, table: DeviceTable) -> np.ndarray:
        return self.evaluate(table)[0][0]

    def loss_and_gradient(self, table: DeviceTable, indices):
        """Mean answer cross-entropy (f64 from the f32 logits) and the f32 gradient."""
        idx = np.ascontiguousarray(indices, dtype=np.uint32)
        loss = ctypes.c_double()
        grad = np.empty(self._count, dtype=np.float32)
        check(self._lib.mb_simple_loss_and_gradient(self._h, table._handle, ptr(idx, ctypes.c_uint32), idx.size,
                                                    ctypes.byref(loss), ptr(grad, ctypes.c_float), grad.size))
        return loss.value, grad

    def train_batch(self, table: DeviceTable, batches: DeviceBatches, offset: int, rows: int,
                    optimizer: AdamWOptions):
        """One AdamW step on ``batches[offset:offset + rows]`` (asynchronous)."""
        o = optimizer.to_c() if isinstance(optimizer, AdamWOptions) else optimizer
        check(self._lib.mb_simple_train_step(self._h, table._handle, batches._handle, offset, rows,
                                             ctypes.byref(o)))

    def check(self):
        """Waits for queued work and raises on device-side errors."""
        check(self._lib.mb_simple_check(self._h))

    @property
    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(self._lib.mb_simple_stream(self._h, ctypes.byref(s)))
        return s.value or 0

    def step_launches(self) -> int:
        n = ctypes.c_uint32()
        check(self._lib.mb_simple_step_launches(self._h, ctypes.byref(n)))
        return n.value


def row_metrics(logits, targets):
    """f64 cross-entropy per row and first-maximum predictions from f32 logits
    (src/bin/mesh-gpt/grokking.rs:544-557)."""
    lg = np.asarray(logits, dtype=np.float64)
    pred = lg.argmax(axis=1)
    mx = lg[np.arange(len(lg)), pred]
    ce = np.log(np.exp(lg - mx[:, None]).sum(axis=1)) + mx - lg[np.arange(len(lg)), targets]
    return ce, pred


def record(model: GpuSimpleModel, tables):
    """One ``loss.csv`` record: train / validation CE, accuracies, weight L2
    (src/bin/mesh-gpt/simple.rs:757-860)."""
    ces, accs = [], []
    for (logits, preds), table in zip(model.evaluate(*tables), tables):
        ce, _ = row_metrics(logits, table.targets)
        ces.append(float(ce.sum() / table.rows))
        accs.append(float((preds == table.targets).sum()) / table.rows)
    norm = math.sqrt(float((model.parameters().astype(np.float64) ** 2).sum()))
    return ces[0], ces[1], accs[0], accs[1], norm


def warmed(optimizer: AdamWOptions, step: int) -> AdamWOptions:
    """10-step linear warmup in f32 (src/bin/mesh-gpt/grokking.rs:524-527)."""
    lr = np.float32(optimizer.learning_rate) * (np.float32(min(step, 10)) / np.float32(10.0))
    return replace(optimizer, learning_rate=float(lr))


def train_records(config: SimpleConfig, device: int = 0, operation: str = "div", train_fraction: float = 0.5,
                  seed: int = 11, steps: int = 10, batch: int = 512, optimizer: AdamWOptions = None):
    """The step-0 and step-``steps`` records of ``grok-simple``
    (src/bin/mesh-gpt/simple.rs:242-652): a seeded split, one epoch of
    ``EquationSampler`` minibatches at a time with a short tail, a 10-step
    warmup and AdamW."""
    optimizer = optimizer or AdamWOptions(learning_rate=1e-3, weight_decay=1.0, beta1=0.9, beta2=0.98)
    dataset = EquationDataset(config.modulus, operation, train_fraction, seed)
    model = GpuSimpleModel(device, config, seed)
    tables = [model.upload_table(*config.encode(dataset.split(v))) for v in (False, True)]
    records = [record(model, tables)]
    n_train = tables[0].rows
    sampler = EquationSampler(n_train, seed)
    steps_per_epoch = -(-n_train // batch)
    step = 0
    while step < steps:
        epoch = sampler.take(batch, min(steps_per_epoch, steps - step))
        batches = model.upload_batches(tables[0], np.concatenate(epoch))
        offset = 0
        for rows in epoch:
            step += 1
            model.train_batch(tables[0], batches, offset, len(rows), warmed(optimizer, step))
            offset += len(rows)
    model.check()
    records.append(record(model, tables))
    return records
