"""B200 (sm_100a) BFP8 GEMV / lm_head decode hot path of qwen35-ax7020-edge-llm.

Submodules:
  _lib      ctypes binding of libqwen_kernels_b200.so (the C ABI)
  ops       device-tensor API (quantizer, exact GEMV, grouped stack, lm_heads, packer)
  model     Qwen3.5-0.8B linear-stack shapes and synthetic weight stacks
"""
from ._lib import KernelError, load  # noqa: F401

__all__ = ["KernelError", "load"]
