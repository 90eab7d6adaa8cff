#!/usr/bin/env python3
"""Build the native pieces in-tree.

* ``emmyrt/libemmyrt.so`` -- the C-ABI launch runtime (csrc/emmyrt.c), compiled with
  gcc against the CUDA driver API headers; libcuda / libnccl are dlopen'd at run
  time, so the library has no link-time GPU dependency.
* every kernel template is exercised by compiling the golden IR fixtures and the
  BASELINE-sized configurations and assembling the PTX with ``ptxas -arch=sm_100a``
  (the cubins land in the content-addressed cache the runtime loads from).
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def build_runtime(verbose: bool = False) -> Path:
    out = PKG / "emmyrt" / "libemmyrt.so"
    src = PKG / "csrc" / "emmyrt.c"
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fvisibility=hidden", "-Wall", "-Wextra", "-Werror",
           f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}", str(src), "-o", str(out), "-ldl"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


def build_static_scratch(verbose: bool = False) -> Path:
    """``emmyrt/libemmyrt_static.so``: the whole-array reduction entry point that takes
    its scratch from a file-scope device array (csrc/emmyrt_static_scratch.cu), linked
    against libemmyrt.so for the launch and against the static CUDA runtime."""
    out = PKG / "emmyrt" / "libemmyrt_static.so"
    src = PKG / "csrc" / "emmyrt_static_scratch.cu"
    cmd = [str(CUDA / "bin" / "nvcc"), "-O2", "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-gencode", "arch=compute_100a,code=sm_100a",
           "-lineinfo", f"-I{ROOT / 'include'}", str(src), "-o", str(out),
           f"-L{PKG / 'emmyrt'}", "-lemmyrt", "-Xlinker", "-rpath,$ORIGIN", "-cudart", "static"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


def main() -> int:
    build_runtime(verbose=True)
    build_static_scratch(verbose=True)
    print("built", PKG / "emmyrt" / "libemmyrt.so")
    return 0


if __name__ == "__main__":
    sys.exit(main())
