"""Compile the reference CUDA extension (fast_fp4/wrapper.cpp + nvfp4sim.cu)
from its own sources into oracle/_ref/, as a GPU-side checker.

TEST INFRASTRUCTURE ONLY.  The sources are read where they lie in the
reference checkout (FP4_REFERENCE_DIR, default /root/reference); nothing is
copied into this repository.  The flags are the reference's own
(fast_fp4/setup.py:11-12: host -O0 -g, device -O0 -g -G) plus an explicit
sm_100a target, so the compiled numerics are the reference's.

The CUDA runtime is linked statically.  torch.utils.cpp_extension would
link libcudart.so.12 dynamically, and inside a torch process that name
resolves to torch's bundled (older) runtime; a fatbin built by this nvcc
then registers through a mismatched runtime, which crashed the first call.

The module is importable as ``nvfp4sim_ref`` from oracle/_ref/ and is only
ever called by tests, to check the C restatement of its numerics
(oracle/nvfp4_oracle.c) and this package's compatible kernels.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
SO = os.path.join(OUT, "nvfp4sim_ref.so")
REF = os.environ.get("FP4_REFERENCE_DIR", "/root/reference")


def build(verbose: bool = False) -> str | None:
    src = [os.path.join(REF, "fast_fp4", "wrapper.cpp"), os.path.join(REF, "fast_fp4", "nvfp4sim.cu")]
    if not all(os.path.exists(s) for s in src):
        return None
    os.makedirs(OUT, exist_ok=True)
    if os.path.exists(SO) and os.path.getmtime(SO) >= max(os.path.getmtime(s) for s in src) and \
            os.path.getmtime(SO) >= os.path.getmtime(__file__):
        return SO
    import torch
    tdir = os.path.dirname(torch.__file__)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    common = ["-DTORCH_EXTENSION_NAME=nvfp4sim_ref", "-DTORCH_API_INCLUDE_EXTENSION_H",
              f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-std=c++17",
              "-isystem", os.path.join(tdir, "include"),
              "-isystem", os.path.join(tdir, "include", "torch", "csrc", "api", "include"),
              "-isystem", sysconfig.get_paths()["include"]]
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    objs = []
    for s in src:
        o = os.path.join(OUT, os.path.basename(s) + ".o")
        if s.endswith(".cu"):
            cmd = [nvcc, "-O0", "-g", "-G", "-gencode", "arch=compute_100a,code=sm_100a",
                   "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                   "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
                   "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__", *common, "-c", s, "-o", o]
        else:
            cmd = [os.environ.get("CXX", "g++"), "-O0", "-g", "-fPIC", *common,
                   "-isystem", "/usr/local/cuda/include", "-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(o)
    link = [nvcc, "-shared", "-cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a", "-o", SO, *objs,
            "-L" + os.path.join(tdir, "lib"), "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            "-ltorch_python", "-Xlinker", "-rpath=" + os.path.join(tdir, "lib")]
    if verbose:
        print(" ".join(link), flush=True)
    subprocess.run(link, check=True)
    return SO


def load():
    """Import the prebuilt module from oracle/_ref (no compilation)."""
    import torch  # noqa: F401  (the module links against torch)
    sys.path.insert(0, OUT)
    try:
        import nvfp4sim_ref
    finally:
        sys.path.remove(OUT)
    return nvfp4sim_ref


if __name__ == "__main__":
    print(build(verbose=True))
