"""Mesh GPT model API over the sm_100a C ABI.

Mirrors the reference's ``GptConfig`` / ``AdamWOptions`` (src/gpt/config.rs:
22-56, 258-295) and ``SpecializedMeshGpt`` (src/gpt/gpu.rs:1701-2092): same
method names, argument meaning and error behaviour (invalid batches and
configurations raise before any launch; nonfinite results raise).
"""

import ctypes
from dataclasses import dataclass, replace

import numpy as np

from . import _lib
from ._lib import MB_ERR_INVALID, AdamWC, GptConfigC, IGNORE_TARGET, MeshError, check, ptr

__all__ = ["GptConfig", "AdamWOptions", "MeshGpt", "IGNORE_TARGET", "parameter_count",
           "initial_parameters", "token_codes"]


@dataclass(frozen=True)
class GptConfig:
    """``GptConfig`` (src/gpt/config.rs:22-56); connectivity "neighbor" or
    "butterfly"; embedding "mesh" or "table" (src/gpt/config.rs:60-67)."""
    vocab_size: int = 32
    context: int = 32
    width: int = 32
    heads: int = 4
    layers: int = 2
    attention_mesh_depth: int = 4
    ffn_mesh_depth: int = 6
    connectivity: str = "neighbor"
    embedding: str = "mesh"

    def to_c(self) -> GptConfigC:
        if self.connectivity not in ("neighbor", "butterfly"):
            raise ValueError(f"unknown mesh connectivity: {self.connectivity}")
        if self.embedding not in ("mesh", "table"):
            raise ValueError(f"unknown token embedding: {self.embedding}")
        return GptConfigC(self.vocab_size, self.context, self.width, self.heads, self.layers,
                          self.attention_mesh_depth, self.ffn_mesh_depth,
                          0 if self.connectivity == "neighbor" else 1, 0 if self.embedding == "mesh" else 1)

    def with_(self, **kw):
        return replace(self, **kw)

    def parameter_count(self) -> int:
        return parameter_count(self)


@dataclass(frozen=True)
class AdamWOptions:
    """``AdamWOptions`` (src/gpt/config.rs:258-276) with its defaults."""
    learning_rate: float = 0.003
    weight_decay: float = 0.01
    beta1: float = 0.9
    beta2: float = 0.999
    epsilon: float = 1e-8

    def to_c(self) -> AdamWC:
        return AdamWC(self.learning_rate, self.weight_decay, self.beta1, self.beta2, self.epsilon)


def parameter_count(config: GptConfig) -> int:
    lib = _lib.load()
    c = config.to_c()
    n = ctypes.c_size_t()
    check(lib.mb_gpt_parameter_count(ctypes.byref(c), ctypes.byref(n)))
    return n.value


def initial_parameters(config: GptConfig, seed: int) -> np.ndarray:
    """Seeded initial weights, ``GptConfig::initial_parameters`` (src/gpt/config.rs:187-190)."""
    lib = _lib.load()
    n = parameter_count(config)
    out = np.empty(n, dtype=np.float32)
    c = config.to_c()
    check(lib.mb_gpt_initial_parameters(ctypes.byref(c), seed, ptr(out, ctypes.c_float), n))
    return out


def token_codes(config: GptConfig) -> np.ndarray:
    lib = _lib.load()
    out = np.empty((config.vocab_size, config.width), dtype=np.float32)
    c = config.to_c()
    check(lib.mb_gpt_token_codes(ctypes.byref(c), ptr(out, ctypes.c_float), out.size))
    return out


def _u32(a) -> np.ndarray:
    if isinstance(a, np.ndarray) and a.dtype == np.uint32 and a.ndim == 1 and a.flags.c_contiguous:
        return a  # no copy: pinned host buffers stay pinned
    arr = np.ascontiguousarray(np.asarray(a, dtype=np.int64))
    if arr.ndim != 1:
        raise ValueError("token batches are flat arrays")
    if (arr < 0).any() or (arr > 0xFFFFFFFF).any():
        raise ValueError("token ID is outside the vocabulary")
    return arr.astype(np.uint32)


class Context:
    """A CUDA device and one stream that the models built in it share (the
    reference's ``Arc<CudaContext>``).  Close the models before the context."""

    def __init__(self, device: int):
        self._lib = _lib.load()
        h = ctypes.c_void_p()
        check(self._lib.mb_ctx_create(device, ctypes.byref(h)))
        self._h = h
        self.device = device

    @property
    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(self._lib.mb_ctx_stream(self._h, ctypes.byref(s)))
        return s.value or 0

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.mb_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MeshGpt:
    """``SpecializedMeshGpt``: a Mesh GPT on one CUDA device.

    Every learned parameter is a mesh edge; training runs forward, backward
    and AdamW on the GPU.  Repeated ``train_batch`` calls continue the same
    AdamW state; ``set_parameters`` resets it."""

    def __init__(self, device, config: GptConfig, seed: int):
        """``device``: a CUDA device index, or a ``Context`` whose device and
        stream the model then uses."""
        self._lib = _lib.load()
        self.config = config
        self._c = config.to_c()
        handle = ctypes.c_void_p()
        if isinstance(device, Context):
            self._context = device  # kept alive while the model uses its stream
            check(self._lib.mb_gpt_create_in(device._h, ctypes.byref(self._c), seed, ctypes.byref(handle)))
        else:
            check(self._lib.mb_gpt_create(device, ctypes.byref(self._c), seed, ctypes.byref(handle)))
        self._h = handle
        self._count = parameter_count(config)

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.mb_gpt_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---------------------------------------------------------- parameters
    def parameter_count(self) -> int:
        return self._count

    def parameters(self) -> np.ndarray:
        out = np.empty(self._count, dtype=np.float32)
        check(self._lib.mb_gpt_get_parameters(self._h, ptr(out, ctypes.c_float), out.size))
        return out

    def set_parameters(self, values) -> None:
        v = np.ascontiguousarray(values, dtype=np.float32)
        check(self._lib.mb_gpt_set_parameters(self._h, ptr(v, ctypes.c_float), v.size))

    # ------------------------------------------------------------- forward
    def logits(self, tokens, sequence: int) -> np.ndarray:
        t = _u32(tokens)
        out = np.empty((t.size, self.config.vocab_size), dtype=np.float32)
        check(self._lib.mb_gpt_logits(self._h, ptr(t, ctypes.c_uint32), t.size, sequence,
                                      ptr(out, ctypes.c_float)))
        return out

    def hidden_states(self, tokens, sequence: int) -> np.ndarray:
        t = _u32(tokens)
        out = np.empty((t.size, self.config.width), dtype=np.float32)
        check(self._lib.mb_gpt_hidden_states(self._h, ptr(t, ctypes.c_uint32), t.size, sequence,
                                             ptr(out, ctypes.c_float)))
        return out

    def token_embeddings(self) -> np.ndarray:
        out = np.empty((self.config.vocab_size, self.config.width), dtype=np.float32)
        check(self._lib.mb_gpt_token_embeddings(self._h, ptr(out, ctypes.c_float), out.size))
        return out

    def cross_entropy(self, inputs, targets, sequence: int) -> float:
        x, y = _u32(inputs), _u32(targets)
        if x.size != y.size:
            raise ValueError("inputs and targets must have equal lengths")
        loss = ctypes.c_double()
        check(self._lib.mb_gpt_cross_entropy(self._h, ptr(x, ctypes.c_uint32), ptr(y, ctypes.c_uint32), x.size,
                                             sequence, ctypes.byref(loss)))
        return loss.value

    # ------------------------------------------------------------ training
    def loss_and_gradient(self, inputs, targets, sequence: int):
        """(mean supervised cross-entropy, gradient as f64 array)."""
        x, y = _u32(inputs), _u32(targets)
        if x.size != y.size:
            raise ValueError("inputs and targets must have equal lengths")
        grad = np.empty(self._count, dtype=np.float32)
        loss = ctypes.c_double()
        check(self._lib.mb_gpt_loss_and_gradient(self._h, ptr(x, ctypes.c_uint32), ptr(y, ctypes.c_uint32), x.size,
                                                 sequence, ctypes.byref(loss), ptr(grad, ctypes.c_float),
                                                 grad.size))
        return loss.value, grad.astype(np.float64)

    def train_batch(self, inputs, targets, sequence: int, learning_rate: float, weight_decay: float) -> float:
        return self.train_batch_with_optimizer(
            inputs, targets, sequence, AdamWOptions(learning_rate=learning_rate, weight_decay=weight_decay))

    def train_batch_with_optimizer(self, inputs, targets, sequence: int, optimizer: AdamWOptions) -> float:
        x, y = _u32(inputs), _u32(targets)
        if x.size != y.size:
            raise ValueError("inputs and targets must have equal lengths")
        opt = optimizer.to_c()
        loss = ctypes.c_double()
        check(self._lib.mb_gpt_train_step(self._h, ptr(x, ctypes.c_uint32), ptr(y, ctypes.c_uint32), x.size,
                                          sequence, ctypes.byref(opt), ctypes.byref(loss)))
        return loss.value

    def train_batch_device(self, inputs_ptr: int, targets_ptr: int, rows: int, sequence: int,
                           optimizer: AdamWOptions, loss_ptr: int = 0) -> None:
        """One step on device-resident u32 batches (raw device pointers), enqueued
        on the model's stream without a host synchronisation."""
        opt = optimizer.to_c()
        check(self._lib.mb_gpt_train_step_device(self._h, ctypes.c_void_p(inputs_ptr), ctypes.c_void_p(targets_ptr),
                                                 rows, sequence, ctypes.byref(opt),
                                                 ctypes.c_void_p(loss_ptr or None)))

    def check(self) -> None:
        check(self._lib.mb_gpt_check(self._h))

    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(self._lib.mb_gpt_stream(self._h, ctypes.byref(s)))
        return s.value or 0

    def allocated_device_bytes(self) -> int:
        n = ctypes.c_size_t()
        check(self._lib.mb_gpt_allocated_device_bytes(self._h, ctypes.byref(n)))
        return n.value

    def step_launches(self, rows: int, sequence: int) -> int:
        n = ctypes.c_size_t()
        check(self._lib.mb_gpt_step_launches(self._h, rows, sequence, ctypes.byref(n)))
        return n.value

    def set_workspace_capacity(self, capacity: int) -> None:
        """How many batch-shape workspaces stay cached, 1..3 (src/gpt/gpu.rs:1779-1787)."""
        if capacity < 0:
            raise MeshError(MB_ERR_INVALID, "workspace capacity must be in 1..3")
        check(self._lib.mb_gpt_set_workspace_capacity(self._h, capacity))

    def workspace_capacity(self) -> int:
        """src/gpt/gpu.rs:1789-1791."""
        n = ctypes.c_size_t()
        check(self._lib.mb_gpt_workspace_capacity(self._h, ctypes.byref(n)))
        return n.value

    # ------------------------------------------------------------- timing
    def set_timing(self, enable: bool) -> None:
        check(self._lib.mb_gpt_set_timing(self._h, 1 if enable else 0))

    def kernel_times(self):
        """[(launch name, ms)] of the most recent training step (timing mode)."""
        n = ctypes.c_size_t(512)
        ms = np.zeros(512, dtype=np.float32)
        names = ctypes.create_string_buffer(1 << 16)
        check(self._lib.mb_gpt_kernel_times(self._h, names, len(names), ptr(ms, ctypes.c_float), ctypes.byref(n)))
        labels = names.value.decode().split(",")
        return list(zip(labels, ms[:n.value].tolist()))

    # ----------------------------------------------------- data parallelism
    def attach_nccl(self, unique_id: bytes, rank: int, world_size: int) -> None:
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        check(self._lib.mb_gpt_attach_nccl(self._h, buf, rank, world_size))

    def attach_nccl_comm(self, comm: int, world_size: int) -> None:
        """Uses a caller-owned NCCL communicator (an ``ncclComm_t`` as an
        integer address) created on this model's device."""
        check(self._lib.mb_gpt_attach_nccl_comm(self._h, ctypes.c_void_p(comm), world_size))

    def detach_nccl(self) -> None:
        check(self._lib.mb_gpt_detach_nccl(self._h))


def nccl_unique_id() -> bytes:
    lib = _lib.load()
    buf = (ctypes.c_uint8 * 128)()
    check(lib.mb_nccl_unique_id(buf))
    return bytes(buf)
