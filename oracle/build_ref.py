"""Compile the reference CUDA extension (fast_fp4/wrapper.cpp + nvfp4sim.cu)
from its own sources into oracle/_ref/, as a GPU-side checker.

TEST INFRASTRUCTURE ONLY.  The sources are read where they lie in the
reference checkout (FP4_REFERENCE_DIR, default /root/reference); nothing is
copied into this repository.  The flags are the reference's own
(fast_fp4/setup.py:11-12: -O0 -g, device -O0 -G) plus an explicit sm_100a
target, so the compiled numerics are the reference's.  The built module is
importable as ``nvfp4sim_ref`` from oracle/_ref/ and is only ever called by
tests, to check the C restatement of its numerics (oracle/nvfp4_oracle.c).
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
REF = os.environ.get("FP4_REFERENCE_DIR", "/root/reference")


def build(verbose: bool = False) -> str | None:
    src = [os.path.join(REF, "fast_fp4", "wrapper.cpp"), os.path.join(REF, "fast_fp4", "nvfp4sim.cu")]
    if not all(os.path.exists(s) for s in src):
        return None
    os.makedirs(OUT, exist_ok=True)
    so = os.path.join(OUT, "nvfp4sim_ref.so")
    if os.path.exists(so) and os.path.getmtime(so) >= max(os.path.getmtime(s) for s in src):
        return so
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils import cpp_extension
    mod = cpp_extension.load(
        name="nvfp4sim_ref", sources=src, build_directory=OUT, verbose=verbose,
        extra_cflags=["-O0", "-g"],
        extra_cuda_cflags=["-O0", "-g", "-G", "-gencode", "arch=compute_100a,code=sm_100a"],
        with_cuda=True, is_python_module=True)
    return mod.__file__


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
