"""Weight checkpoints in the reference's formats.

``Checkpoint`` mirrors ``src/gpt/checkpoint.rs`` (MSHGPT07 for the default
architecture, MSHGPT08 for a table embedding or butterfly connectivity): the configuration, the
character tokenizer and the FP32 parameters, read and written by the C ABI
(``mb_gpt_checkpoint_write`` / ``mb_gpt_checkpoint_read``).  Loading into a
model goes through ``set_parameters``, which resets AdamW as the reference's
loader does.  ``save_raw`` / ``load_raw`` are grok-simple's ``model.bin``
(``src/bin/mesh-gpt/simple.rs:843-850``): the parameters as little-endian f32
and nothing else.
"""

import ctypes
import os
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import GptConfigC, check, ptr
from .gpt import GptConfig, MeshGpt


def _codes(characters) -> np.ndarray:
    if isinstance(characters, str):
        return np.array([ord(c) for c in characters], dtype=np.uint32)
    return np.ascontiguousarray(characters, dtype=np.uint32)


@dataclass
class Checkpoint:
    config: GptConfig
    characters: str
    parameters: np.ndarray

    def save(self, path):
        c = self.config.to_c()
        codes = _codes(self.characters)
        p = np.ascontiguousarray(self.parameters, dtype=np.float32)
        check(_lib.load().mb_gpt_checkpoint_write(os.fsencode(path), ctypes.byref(c), ptr(codes, ctypes.c_uint32),
                                                  codes.size, ptr(p, ctypes.c_float), p.size))

    @classmethod
    def load(cls, path) -> "Checkpoint":
        lib = _lib.load()
        c = GptConfigC()
        nc, npar = ctypes.c_size_t(), ctypes.c_size_t()
        check(lib.mb_gpt_checkpoint_read(os.fsencode(path), ctypes.byref(c), None, ctypes.byref(nc), None,
                                         ctypes.byref(npar)))
        codes = np.empty(nc.value, dtype=np.uint32)
        params = np.empty(npar.value, dtype=np.float32)
        check(lib.mb_gpt_checkpoint_read(os.fsencode(path), ctypes.byref(c), ptr(codes, ctypes.c_uint32),
                                         ctypes.byref(nc), ptr(params, ctypes.c_float), ctypes.byref(npar)))
        config = GptConfig(c.vocab_size, c.context, c.width, c.heads, c.layers, c.attention_mesh_depth,
                           c.ffn_mesh_depth, "butterfly" if c.connectivity else "neighbor",
                           "table" if c.embedding else "mesh")
        return cls(config, "".join(chr(int(x)) for x in codes), params)

    @classmethod
    def from_model(cls, model: MeshGpt, characters) -> "Checkpoint":
        return cls(model.config, characters if isinstance(characters, str) else
                   "".join(chr(int(x)) for x in characters), model.parameters())

    def model(self, device: int = 0, seed: int = 0) -> MeshGpt:
        """A model holding these weights with a fresh AdamW state."""
        m = MeshGpt(device, self.config, seed)
        m.set_parameters(self.parameters)
        return m


def save_raw(path, parameters):
    """grok-simple ``model.bin``: little-endian f32 parameters."""
    np.ascontiguousarray(parameters, dtype="<f4").tofile(path)


def load_raw(path, count: int) -> np.ndarray:
    data = np.fromfile(path, dtype="<f4")
    if data.size != count:
        raise ValueError("parameter count does not match the model")
    if not np.isfinite(data).all():
        raise ValueError("parameters must be finite")
    return data.astype(np.float32)
