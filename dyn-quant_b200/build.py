"""Build the dyn-quant B200 library in-tree.

  dyn_quant/libdq_b200.so    the sm_100a kernels + the C ABI (include/dq_abi.h),
                             nvcc -gencode arch=compute_100a,code=sm_100a, static cudart
  dyn_quant/_C.<abi>.so      the torch extension (csrc/torch_ext.cpp) over that ABI

usage: python dyn-quant_b200/build.py [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "dyn_quant")
INCLUDE = os.path.join(REPO, "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB_SOURCES = ["dq_gemv.cu", "dq_stream.cu", "dq_batched.cu", "dq_moe.cu", "dq_abi.cu"]
LIB_HEADERS = ["dq_common.cuh", "dq_internal.h", "dq_plan.cuh", "dq_gplan.cuh"]
LIB_PATH = os.path.join(PKG, "libdq_b200.so")
EXT_SUFFIX = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
EXT_PATH = os.path.join(PKG, "_C" + EXT_SUFFIX)


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.exists(d) and os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_lib(force: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in LIB_SOURCES if os.path.exists(os.path.join(CSRC, s))]
    deps = srcs + [os.path.join(CSRC, h) for h in LIB_HEADERS] + [os.path.join(INCLUDE, "dq_abi.h"), __file__]
    if force or _stale(LIB_PATH, deps):
        _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-Xptxas", "-v", "-shared", "-cudart", "static",
              f"-I{INCLUDE}", "-o", LIB_PATH, *srcs])
    return LIB_PATH


def build_ext(force: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension as ce

    src = os.path.join(CSRC, "torch_ext.cpp")
    if not (force or _stale(EXT_PATH, [src, LIB_PATH, os.path.join(INCLUDE, "dq_abi.h"), __file__])):
        return EXT_PATH
    inc = ce.include_paths(device_type="cuda") if "device_type" in ce.include_paths.__code__.co_varnames \
        else ce.include_paths(cuda=True)
    libdirs = ce.library_paths(device_type="cuda") if "device_type" in ce.library_paths.__code__.co_varnames \
        else ce.library_paths(cuda=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O3", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-I{sysconfig.get_paths()['include']}", f"-I{INCLUDE}"]
    cmd += [f"-I{p}" for p in inc]
    cmd += [src, "-o", EXT_PATH]
    cmd += [f"-L{p}" for p in libdirs]
    cmd += [f"-L{PKG}", "-ldq_b200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            "-ltorch_python", "-Wl,-rpath,$ORIGIN"]
    _run(cmd)
    return EXT_PATH


def build(force: bool = False) -> None:
    build_lib(force)
    build_ext(force)


if __name__ == "__main__":
    build("--force" in sys.argv[1:])
