"""Build ``luma_b200/_lib/libluma_b200.so`` with nvcc for sm_100a.

    python -m luma_b200.build [--debug]

The library statically links the CUDA runtime, so it only needs the driver
(libcuda) at run time.  The build output stays in-tree next to the package.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SOURCES = [os.path.join(HERE, "csrc", "luma_step.cu"), os.path.join(HERE, "csrc", "luma_peer.cu")]
OUT = os.path.join(HERE, "_lib", "libluma_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-shared",
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(verbose: bool = False, extra: list[str] | None = None) -> str:
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = [nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), *(extra or []),
           "-o", OUT + ".tmp", *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


def is_stale() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = SOURCES + [os.path.join(ROOT, "include", "luma_b200.h"),
                      os.path.join(HERE, "csrc", "luma_internal.h")]
    return any(os.path.getmtime(s) > t for s in deps)


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
