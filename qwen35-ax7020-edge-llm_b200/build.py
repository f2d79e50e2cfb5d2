"""Build the native parts of the package.

    python qwen35-ax7020-edge-llm_b200/build.py

produces, in-tree:
  qwen_b200/libqwen_kernels_b200.so   CUDA kernels + C ABI (nvcc, sm_100a)
  qwen_b200/libqwen_b200_torch.so     PyTorch operator library (torch.ops.qwen_b200)
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_ROOT = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
OUT_DIR = os.path.join(PKG_ROOT, "qwen_b200")
INCLUDE = os.path.join(REPO, "include")
LIB_NAME = "libqwen_kernels_b200.so"
TORCH_LIB_NAME = "libqwen_b200_torch.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["bfp8_gemv.cu", "bfp8_gemm_tc.cu", "lm_head.cu", "pack.cu", "sample.cu", "tma.cu", "capi.cu",
              "noalloc.cu", "gdn.cu"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_core(force: bool = False, verbose: bool = False) -> str:
    target = os.path.join(OUT_DIR, LIB_NAME)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, "qwen_b200.h")]
    if not force and not _stale(target, deps):
        return target
    cmd = [_nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-shared", f"-I{INCLUDE}", f"-I{CSRC}",
           "-o", target + ".tmp", *[os.path.join(CSRC, f) for f in CU_SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(target + ".tmp", target)
    return target


def build_torch_ext(force: bool = False) -> str:
    """Compile the torch.ops.qwen_b200 operator library (C++ only; every
    operator calls the C ABI of the core library) into qwen_b200/ beside the
    core library, which it finds through an $ORIGIN rpath."""
    import torch
    import torch.utils.cpp_extension as ce

    src = os.path.join(CSRC, "torch_ops.cpp")
    core = os.path.join(OUT_DIR, LIB_NAME)
    target = os.path.join(OUT_DIR, TORCH_LIB_NAME)
    if not force and not _stale(target, [src, core, os.path.join(INCLUDE, "qwen_b200.h")]):
        return target
    cuda_home = ce.CUDA_HOME or "/usr/local/cuda"
    cmd = [shutil.which("g++") or "g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{p}" for p in ce.include_paths()], f"-I{os.path.join(cuda_home, 'include')}", f"-I{INCLUDE}",
           src, "-o", target + ".tmp",
           *[f"-L{p}" for p in ce.library_paths()], f"-L{OUT_DIR}",
           "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch", "-lqwen_kernels_b200",
           "-Wl,-rpath,$ORIGIN"]
    subprocess.run(cmd, check=True)
    os.replace(target + ".tmp", target)
    return target


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_core(force=force, verbose=verbose)
    build_torch_ext(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print("built", os.path.join(OUT_DIR, LIB_NAME))
