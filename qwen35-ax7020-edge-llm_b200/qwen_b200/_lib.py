"""ctypes binding of libqwen_kernels_b200.so (the C ABI in include/qwen_b200.h).

The library is built in-tree by ``build.py``.  Importing this module never
falls back to anything else: if the library is missing or fails to load, the
import raises, so a run without the CUDA path fails loudly.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwen_kernels_b200.so")
TORCH_LIB_PATH = os.path.join(HERE, "libqwen_b200_torch.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float

# name -> (restype, argtypes); mirrors include/qwen_b200.h
# void(int layer_idx, float* h, void* py_context): forward_token_c's
# full-attention callback, the engine's CALLBACK_TYPE (qwen_real_engine.py:982)
FULL_ATTN_CALLBACK = ctypes.CFUNCTYPE(None, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p)

SIGNATURES = {
    "init_kernels": (None, []),
    "bfp8_gemv": (None, [_P, _P, _P, _P, _I, _I]),
    "lm_head_argmax": (_I, [_P, _P, _I, _I]),
    "lm_head_topk": (_I, [_P, _P, _I, _I, _I, _P, _P]),
    "sample_from_topk": (_I, [_P, _P, _I, _F, _I, _F, _P]),
    "forward_mlp": (None, [_P, _P]),
    "forward_linear_layer": (None, [_P, _P]),
    "forward_token_c": (_I, [_I, _P, _P, _P, _P, _P, _P, FULL_ATTN_CALLBACK, _P]),
    "qwen_b200_gdn_state_mode": (_I, [_I]),
    "qwen_b200_gdn_state_sync": (_I, []),
    "qwen_b200_gdn_state_drop": (None, []),
    "qwen_prof_enable": (None, [_I]),
    "qwen_prof_reset": (None, []),
    "qwen_prof_count": (_I, []),
    "qwen_prof_get": (ctypes.c_double, [_I]),
    "qwen_prof_name": (ctypes.c_char_p, [_I]),
    "qwen_b200_register_weights": (_I, [_P, ctypes.c_size_t]),
    "qwen_b200_forget_weights": (_I, [_P]),
    "qwen_b200_reset_weights": (None, []),
    "qwen_b200_gemv_dev": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "qwen_b200_gemv_noalloc_dev": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "qwen_b200_gemv_fast_dev": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "qwen_b200_gemv_q_dev": (_I, [_P, _P, _P, _P, _P, _I, _I, _P]),
    "qwen_b200_swiglu_gemv_dev": (_I, [_P, _P, _P, _P, _P, _I, _I, _P]),
    "qwen_b200_gemv_rtl20_dev": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _P, _P]),
    "qwen_b200_rmsnorm_gemv_dev": (_I, [_P, _P, _P, _F, _P, _P, _I, _I, _P]),
    "qwen_b200_residual_rmsnorm_gemv_dev": (_I, [_P, _P, _P, _P, _P, _F, _P, _P, _I, _I, _P]),
    "qwen_b200_rmsnorm_gemv2_dev": (_I, [_P, _P, _P, _P, _P, _P, _F, _P, _P, _I, _P, _P, _I, _I, _P]),
    "qwen_b200_quant_dev": (_I, [_P, _I, _I, _P, _P, _P]),
    "qwen_b200_stack_create": (_I, [_I, _P, _P, _P, _P, _P, _P]),
    "qwen_b200_stack_create_ex": (_I, [_I, _P, _P, _P, _P, _P, _P, _I]),
    "qwen_b200_stack_run": (_I, [_I, _P]),
    "qwen_b200_stack_destroy": (_I, [_I]),
    "qwen_b200_stack_create_sharded": (_I, [_I, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P]),
    "qwen_b200_stack_run_sync": (_I, [_I, _P, _P, ctypes.c_uint, _P, ctypes.c_uint, _I, _I]),
    "qwen_b200_swiglu_quant_sharded_dev": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I, _P, _P, ctypes.c_uint,
                                                 _P, _I, _I, _P]),
    "qwen_b200_dev_alloc": (_I, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "qwen_b200_dev_free": (_I, [_P]),
    "qwen_b200_ipc_handle": (_I, [_P, _P]),
    "qwen_b200_ipc_open": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "qwen_b200_ipc_close": (_I, [_P]),
    "qwen_b200_quant_planes_dev": (_I, [_P, _I, _I, _P, _P, _I, _P]),
    "qwen_b200_gemm_tc_dev": (_I, [_P, _P, _P, _I, _P, _P, _I, _I, _I, _P, _P]),
    "qwen_b200_tc_stack_create": (_I, [_I, _P, _P, _P, _P, _P, _P, _P, _I, _I]),
    "qwen_b200_tc_stack_run": (_I, [_I, _P]),
    "qwen_b200_tc_stack_destroy": (_I, [_I]),
    "qwen_b200_tc_stack_create_sharded": (_I, [_I, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _P]),
    "qwen_b200_tc_stack_run_sync": (_I, [_I, _P, _P, ctypes.c_uint, _I, _I]),
    "qwen_b200_quant_planes_wait_dev": (_I, [_P, _I, _I, _P, _P, _I, _P, ctypes.c_uint, _I, _P]),
    "qwen_b200_sync_epoch_base": (_I, [_P]),
    "qwen_b200_sync_epoch_advance": (_I, [_P, ctypes.c_uint, _P]),
    "qwen_b200_lm_head_bf16_dev": (_I, [_P, _P, _I, _I, _I, _P, _P, _P, _P, _P]),
    "qwen_b200_lm_head_bfp8_dev": (_I, [_P, _P, _P, _I, _I, _I, _P, _P, _P, _P, _P]),
    "qwen_b200_sample_topk_dev": (_I, [_P, _P, _P, _I, _F, _I, _F, _P, _P, _P]),
    "qwen_b200_pack_bfp8_dev": (_I, [_P, _I, _I, _P, _P, _P]),
    "qwen_b200_device_error": (_I, [_I]),
    "qwen_b200_last_error": (ctypes.c_char_p, []),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load the kernel library (raises OSError if it is absent)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: run qwen35-ax7020-edge-llm_b200/build.py")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


_torch_ops = None


def torch_ops():
    """torch.ops.qwen_b200 (the PyTorch operator library, built in-tree by
    ``build.py``); raises if the library is absent."""
    global _torch_ops
    if _torch_ops is None:
        import torch

        if not os.path.exists(TORCH_LIB_PATH):
            raise OSError(f"{TORCH_LIB_PATH} is missing: run qwen35-ax7020-edge-llm_b200/build.py")
        load()   # the operator library resolves the kernel library through its rpath
        torch.ops.load_library(TORCH_LIB_PATH)
        _torch_ops = torch.ops.qwen_b200
    return _torch_ops


class KernelError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().qwen_b200_last_error().decode(errors="replace")
        raise KernelError(f"{what} failed ({rc}): {msg}")
