"""Builds libflashprefill_b200.so (sm_100a) in-tree with nvcc.

    python -m flashprefill_b200.build [--verbose-ptxas]

The library is one unity translation unit (csrc/fp_api.cu includes the kernels) linked
against the static CUDA runtime, so it only needs the NVIDIA driver at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libflashprefill_b200.so")
SOURCES = ["fp_api.cu"]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is needed to build flashprefill_b200")


def _deps():
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh"))]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "flashprefill_b200.h"))
    return deps


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(d) > t for d in _deps())


def build(force: bool = False, ptxas_verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    cmd = [nvcc_path(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
           "-cudart", "static", "-o", LIB + ".tmp"]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    # extra nvcc flags, e.g. -DFPB_SA_PROFILE=1 for an instrumented build
    cmd += os.environ.get("FLASHPREFILL_B200_NVCC_FLAGS", "").split()
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    if ptxas_verbose:
        sys.stderr.write(r.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, ptxas_verbose="--verbose-ptxas" in sys.argv))
