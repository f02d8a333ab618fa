"""Build recipe for the oracle (test infrastructure only).

Outputs (all git-ignored, all travel with the working tree):
  oracle/liboracle.so          the C restatement, gcc -O3 -fopenmp -ffp-contract=off
  oracle/_ref/ref_quant        the reference's own host quantizer, built from the
                               unmodified src/quant_format.cuh where it lies
  oracle/_ref/libdqref_gpu.so  the reference's own kernels for sm_100a, built from a
                               scratch copy outside the repository with the three
                               minimal patches listed in oracle/ref_gpu_harness.cu

The two _ref targets need the read-only reference tree (default
/root/reference, or $DQ_REFERENCE_DIR); where it is absent they are skipped and
whatever was built before is kept.  Reference sources are never copied into
the repository.

usage: python oracle/build_oracle.py [--force]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.environ.get("DQ_REFERENCE_DIR", "/root/reference")
REF_OUT = os.path.join(HERE, "_ref")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources if os.path.exists(s))


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_liboracle(force: bool = False) -> str:
    src = os.path.join(HERE, "dq_oracle.c")
    out = os.path.join(HERE, "liboracle.so")
    if force or _stale(out, [src, __file__]):
        _run(["gcc", "-O3", "-std=c11", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
              "-fPIC", "-shared", "-Wall", "-o", out, src, "-lm"])
    return out


def build_ref_quant(force: bool = False) -> str | None:
    hdr = os.path.join(REF_DIR, "src", "quant_format.cuh")
    if not os.path.exists(hdr):
        return None
    os.makedirs(REF_OUT, exist_ok=True)
    src = os.path.join(HERE, "ref_quant_main.cpp")
    out = os.path.join(REF_OUT, "ref_quant")
    if force or _stale(out, [src, hdr, __file__]):
        # g++ as the reference's host build uses it (x86-64 default ISA: no FMA contraction)
        _run(["g++", "-O3", "-std=c++17", "-w", f"-I{CUDA_HOME}/include",
              f"-I{os.path.join(REF_DIR, 'src')}", "-o", out, src])
    return out


# (file, exact text, replacement) -- each must match exactly once
_PATCHES = [
    ("quant_format.cuh",
     "__device__ __forceinline__ uint8_t pack_int4(uint8_t lo, uint8_t hi) {",
     "__host__ __device__ __forceinline__ uint8_t pack_int4(uint8_t lo, uint8_t hi) {"),
    ("outlier_detect.cuh",
     "    int*   smem_warp_mean,    // float*, size = num_warps",
     "    float* smem_warp_mean,    // float*, size = num_warps"),
    ("split_gemv.cu",
     "    split_gemv_kernel<<<grid, block, smem_bytes, stream>>>(",
     "    cudaFuncSetAttribute(split_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,"
     " (int)smem_bytes);\n    split_gemv_kernel<<<grid, block, smem_bytes, stream>>>("),
]

_REF_FILES = ["quant_format.cuh", "outlier_detect.cuh", "split_gemv.cu", "split_gemv.cuh",
              "int4_gemv.cu", "int4_gemv.cuh", "reference_gemv.cu", "reference_gemv.cuh"]


def build_ref_gpu(force: bool = False) -> str | None:
    src_dir = os.path.join(REF_DIR, "src")
    if not all(os.path.exists(os.path.join(src_dir, f)) for f in _REF_FILES):
        return None
    if not os.path.exists(NVCC):
        return None
    os.makedirs(REF_OUT, exist_ok=True)
    harness = os.path.join(HERE, "ref_gpu_harness.cu")
    out = os.path.join(REF_OUT, "libdqref_gpu.so")
    deps = [harness, __file__] + [os.path.join(src_dir, f) for f in _REF_FILES]
    if not (force or _stale(out, deps)):
        return out
    tmp = tempfile.mkdtemp(prefix="dqref_src_")
    try:
        for f in _REF_FILES:
            shutil.copy(os.path.join(src_dir, f), os.path.join(tmp, f))
        for fname, old, new in _PATCHES:
            p = os.path.join(tmp, fname)
            text = open(p).read()
            if text.count(old) != 1:
                raise RuntimeError(f"patch anchor not found exactly once in {fname}: {old!r}")
            with open(p, "w") as fh:
                fh.write(text.replace(old, new))
        flags = ["-O3", "-std=c++17", "--expt-relaxed-constexpr", "-use_fast_math",
                 "-Xcompiler", "-fPIC", "-w"] + ARCH
        objs = []
        for f in ["split_gemv.cu", "int4_gemv.cu", "reference_gemv.cu"]:
            o = os.path.join(tmp, f + ".o")
            _run([NVCC, *flags, "-I", tmp, "-c", os.path.join(tmp, f), "-o", o])
            objs.append(o)
        o = os.path.join(tmp, "harness.o")
        _run([NVCC, *flags, "-I", tmp, "-c", harness, "-o", o])
        objs.append(o)
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", out, *objs])
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return out


def main(argv: list[str]) -> int:
    force = "--force" in argv
    print("liboracle:", build_liboracle(force))
    print("ref_quant:", build_ref_quant(force))
    print("libdqref_gpu:", build_ref_gpu(force))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
