"""ctypes binding of ``libmeshb200.so`` (the C ABI in ``include/meshb200.h``).

The library is built in-tree by ``grokking_abmod_b200.build``; loading fails
loudly when it is missing - there is no CPU fallback.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmeshb200.so")

MB_OK = 0
MB_ERR_INVALID = -1
MB_ERR_CUDA = -2
MB_ERR_NONFINITE = -3
MB_ERR_NCCL = -4
MB_ERR_UNSUPPORTED = -5
IGNORE_TARGET = 0xFFFFFFFF

c_size_p = ctypes.POINTER(ctypes.c_size_t)
c_float_p = ctypes.POINTER(ctypes.c_float)
c_double_p = ctypes.POINTER(ctypes.c_double)
c_u32_p = ctypes.POINTER(ctypes.c_uint32)
c_u8_p = ctypes.POINTER(ctypes.c_uint8)


class GptConfigC(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "vocab_size", "context", "width", "heads", "layers",
        "attention_mesh_depth", "ffn_mesh_depth", "connectivity", "embedding")]


class SimpleConfigC(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "architecture", "activation", "modulus", "width", "depth", "connectivity",
        "embedding_mesh_depth", "full_mesh_initialization", "mesh_learning_rate_multiplier", "expansion",
        "mesh_depth", "mesh_output_activation", "tied_mesh", "encoding", "decay_factors")]


class AdamWC(ctypes.Structure):
    _fields_ = [(n, ctypes.c_float) for n in (
        "learning_rate", "weight_decay", "beta1", "beta2", "epsilon")]


class MeshError(RuntimeError):
    """A nonzero status from the library, with its code and message."""

    def __init__(self, code, message):
        super().__init__(f"[{code}] {message}")
        self.code = code


class UnsupportedShape(MeshError):
    pass


# name -> (restype, argtypes)
SIGNATURES = {
    "mb_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
    "mb_version": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "mb_device_count": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "mb_gpt_validate": (ctypes.c_int, [ctypes.POINTER(GptConfigC)]),
    "mb_gpt_parameter_count": (ctypes.c_int, [ctypes.POINTER(GptConfigC), c_size_p]),
    "mb_gpt_initial_parameters": (ctypes.c_int, [ctypes.POINTER(GptConfigC), ctypes.c_uint64, c_float_p,
                                                 ctypes.c_size_t]),
    "mb_gpt_token_codes": (ctypes.c_int, [ctypes.POINTER(GptConfigC), c_float_p, ctypes.c_size_t]),
    "mb_gpt_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(GptConfigC), ctypes.c_uint64,
                                     ctypes.POINTER(ctypes.c_void_p)]),
    "mb_gpt_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "mb_gpt_get_config": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(GptConfigC)]),
    "mb_gpt_get_parameters": (ctypes.c_int, [ctypes.c_void_p, c_float_p, ctypes.c_size_t]),
    "mb_gpt_set_parameters": (ctypes.c_int, [ctypes.c_void_p, c_float_p, ctypes.c_size_t]),
    "mb_gpt_logits": (ctypes.c_int, [ctypes.c_void_p, c_u32_p, ctypes.c_size_t, ctypes.c_size_t, c_float_p]),
    "mb_gpt_hidden_states": (ctypes.c_int, [ctypes.c_void_p, c_u32_p, ctypes.c_size_t, ctypes.c_size_t,
                                            c_float_p]),
    "mb_gpt_token_embeddings": (ctypes.c_int, [ctypes.c_void_p, c_float_p, ctypes.c_size_t]),
    "mb_gpt_cross_entropy": (ctypes.c_int, [ctypes.c_void_p, c_u32_p, c_u32_p, ctypes.c_size_t, ctypes.c_size_t,
                                            c_double_p]),
    "mb_gpt_loss_and_gradient": (ctypes.c_int, [ctypes.c_void_p, c_u32_p, c_u32_p, ctypes.c_size_t,
                                                ctypes.c_size_t, c_double_p, c_float_p, ctypes.c_size_t]),
    "mb_gpt_train_step": (ctypes.c_int, [ctypes.c_void_p, c_u32_p, c_u32_p, ctypes.c_size_t, ctypes.c_size_t,
                                         ctypes.POINTER(AdamWC), c_double_p]),
    "mb_gpt_train_step_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_size_t, ctypes.c_size_t, ctypes.POINTER(AdamWC),
                                                ctypes.c_void_p]),
    "mb_gpt_check": (ctypes.c_int, [ctypes.c_void_p]),
    "mb_gpt_stream": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "mb_gpt_allocated_device_bytes": (ctypes.c_int, [ctypes.c_void_p, c_size_p]),
    "mb_gpt_step_launches": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, c_size_p]),
    "mb_gpt_set_timing": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "mb_gpt_set_workspace_capacity": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t]),
    "mb_gpt_workspace_capacity": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_size_t)]),
    "mb_gpt_kernel_times": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, c_float_p, c_size_p]),
    "mb_nccl_unique_id": (ctypes.c_int, [c_u8_p]),
    "mb_gpt_attach_nccl": (ctypes.c_int, [ctypes.c_void_p, c_u8_p, ctypes.c_int, ctypes.c_int]),
    "mb_gpt_attach_nccl_comm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]),
    "mb_gpt_detach_nccl": (ctypes.c_int, [ctypes.c_void_p]),
    "mb_op_mesh_forward": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32,
                                          ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p]),
    "mb_op_mesh_backward": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                           ctypes.c_void_p, ctypes.c_void_p]),
    "mb_op_gemm_tf32x3": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                                         ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                                         ctypes.c_void_p]),
    "mb_test_gemm_lost_arrival": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                 ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                                 ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p]),
    "mb_op_mesh_backward_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                   ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32,
                                                   ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                                                   ctypes.c_void_p]),
    "mb_ctx_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "mb_ctx_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "mb_ctx_stream": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "mb_gpt_create_in": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(GptConfigC), ctypes.c_uint64,
                                        ctypes.POINTER(ctypes.c_void_p)]),
    "mb_op_rmsnorm_forward": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_size_t, ctypes.c_uint32,
                                                                     ctypes.c_uint32, ctypes.c_void_p]),
    "mb_op_rmsnorm_backward": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_size_t, ctypes.c_uint32,
                                                                      ctypes.c_uint32, ctypes.c_void_p]),
    "mb_op_rope": (ctypes.c_int, [ctypes.c_void_p] * 2 + [ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32,
                                                         ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p]),
    "mb_op_attn_forward": (ctypes.c_int, [ctypes.c_void_p] * 5 + [ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32,
                                                                 ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p]),
    "mb_op_attn_backward": (ctypes.c_int, [ctypes.c_void_p] * 9 + [ctypes.c_size_t, ctypes.c_uint32,
                                                                  ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                                                                  ctypes.c_void_p]),
    "mb_op_xsa_forward": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32,
                                                                 ctypes.c_void_p]),
    "mb_op_xsa_backward": (ctypes.c_int, [ctypes.c_void_p] * 5 + [ctypes.c_size_t, ctypes.c_uint32,
                                                                  ctypes.c_uint32, ctypes.c_void_p]),
    "mb_op_head_ce": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32] +
                      [ctypes.c_void_p] * 6),
    "mb_op_adamw": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_size_t, ctypes.POINTER(AdamWC),
                                                           ctypes.c_uint32, ctypes.c_void_p]),
    "mb_gpt_checkpoint_write": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(GptConfigC), c_u32_p, ctypes.c_size_t,
                                               c_float_p, ctypes.c_size_t]),
    "mb_gpt_checkpoint_read": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(GptConfigC), c_u32_p, c_size_p,
                                              c_float_p, c_size_p]),
    "mb_random_units": (ctypes.c_int, [ctypes.c_uint64, c_float_p, ctypes.c_size_t]),
    "mb_equation_dataset": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_double, ctypes.c_uint64,
                                           c_u32_p, c_u32_p, c_size_p, c_u32_p, c_size_p]),
    "mb_equation_sampler": (ctypes.c_int, [ctypes.c_size_t, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_size_t,
                                           c_u32_p, c_u32_p]),
    "mb_zipf_batch": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t,
                                     ctypes.c_size_t, ctypes.c_uint32, ctypes.c_double, c_u32_p, c_u32_p]),
    "mb_simple_validate": (ctypes.c_int, [ctypes.POINTER(SimpleConfigC)]),
    "mb_simple_parameter_count": (ctypes.c_int, [ctypes.POINTER(SimpleConfigC), c_size_p]),
    "mb_simple_groups": (ctypes.c_int, [ctypes.POINTER(SimpleConfigC), c_u32_p, c_size_p]),
    "mb_simple_initial_parameters": (ctypes.c_int, [ctypes.POINTER(SimpleConfigC), ctypes.c_uint64, c_float_p,
                                                    ctypes.c_size_t]),
    "mb_simple_encode": (ctypes.c_int, [ctypes.POINTER(SimpleConfigC), c_u32_p, ctypes.c_size_t, c_float_p,
                                        c_u32_p]),
    "mb_simple_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(SimpleConfigC), ctypes.c_uint64,
                                        ctypes.POINTER(ctypes.c_void_p)]),
    "mb_simple_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "mb_simple_get_parameters": (ctypes.c_int, [ctypes.c_void_p, c_float_p, ctypes.c_size_t]),
    "mb_simple_set_parameters": (ctypes.c_int, [ctypes.c_void_p, c_float_p, ctypes.c_size_t]),
    "mb_simple_upload_table": (ctypes.c_int, [ctypes.c_void_p, c_float_p, c_u32_p, ctypes.c_size_t,
                                              ctypes.POINTER(ctypes.c_void_p)]),
    "mb_simple_table_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "mb_simple_upload_batches": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, c_u32_p, ctypes.c_size_t,
                                                ctypes.POINTER(ctypes.c_void_p)]),
    "mb_simple_batches_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "mb_simple_train_step": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                            ctypes.c_size_t, ctypes.POINTER(AdamWC)]),
    "mb_simple_evaluate": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, c_float_p, c_u32_p]),
    "mb_simple_loss_and_gradient": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, c_u32_p, ctypes.c_size_t,
                                                   c_double_p, c_float_p, ctypes.c_size_t]),
    "mb_host_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "mb_host_free": (ctypes.c_int, [ctypes.c_void_p]),
    "mb_simple_stream": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "mb_simple_check": (ctypes.c_int, [ctypes.c_void_p]),
    "mb_simple_step_launches": (ctypes.c_int, [ctypes.c_void_p, c_u32_p]),
}

_lib = None


def load(build_if_missing: bool = True):
    """Loads the shared library (building it first when absent or stale and
    nvcc is available)."""
    global _lib
    if _lib is not None:
        return _lib
    if build_if_missing:
        try:
            from .build import build
            build()
        except Exception:
            if not os.path.exists(LIB_PATH):
                raise
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing; run python -m grokking_abmod_b200.build")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int):
    if status != MB_OK:
        buf = ctypes.create_string_buffer(1024)
        load().mb_last_error(buf, len(buf))
        message = buf.value.decode(errors="replace")
        if status == MB_ERR_UNSUPPORTED:
            raise UnsupportedShape(status, message)
        raise MeshError(status, message)
    return status


def ptr(array, ctype):
    """ctypes pointer to a C-contiguous numpy array's data."""
    return array.ctypes.data_as(ctypes.POINTER(ctype))
