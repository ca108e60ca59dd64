"""Build libfp4attn.so in-tree with nvcc for sm_100a.

``python -m fp4_attn_b200.build`` (or ``build()``) compiles every
``csrc/*.cu`` to an object and links them into ``fp4_attn_b200/libfp4attn.so``.
Objects are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libfp4attn.so")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
          "-I", CSRC, "-I", os.path.join(ROOT, "include")]
# Files whose arithmetic must round exactly like the reference: no FMA contraction.
EXACT = {"quant.cu", "quant_f32.cu", "quant_bf16.cu", "quant_f16.cu", "quant_fused.cu", "nvfp4sim_compat.cu",
         "qkv_quant.cu"}


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _newest(paths):
    return max(os.path.getmtime(p) for p in paths)


def build(verbose: bool = False, extra: list[str] | None = None) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    hdr_time = _newest(hdrs) if hdrs else 0.0
    nvcc = _nvcc()
    objs, jobs = [], []
    for s in srcs:
        o = os.path.join(OBJ, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), hdr_time):
            continue
        cmd = [nvcc, *ARCH, *COMMON, "--fmad=" + ("false" if os.path.basename(s) in EXACT else "true"),
               *(extra or []), "-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd), flush=True)
        jobs.append(cmd)
    with ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        for r in ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs):
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError("nvcc failed: " + " ".join(r.args[-3:]))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
