"""B200-native (sm_100a) training hot path of fxeqxmulfx/grokking_abmod.

``MeshGpt`` runs Mesh GPT forward, backward and AdamW through the C ABI of
``libmeshb200.so`` (``include/meshb200.h``); ``data`` generates the
reference's seeded equation datasets and the benchmark token streams.
"""

from .gpt import AdamWOptions, Context, GptConfig, IGNORE_TARGET, MeshGpt, initial_parameters, nccl_unique_id, \
    parameter_count, token_codes
from ._lib import MeshError, UnsupportedShape

__all__ = ["AdamWOptions", "Context", "GptConfig", "IGNORE_TARGET", "MeshGpt", "MeshError", "UnsupportedShape",
           "initial_parameters", "nccl_unique_id", "parameter_count", "token_codes"]
