"""Builds libchatcuda.so in-tree (chat_wgpu_b200/libchatcuda.so) with the
Makefile in csrc/: nvcc -gencode arch=compute_100a,code=sm_100a."""
from __future__ import annotations

import os
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(PKG, "libchatcuda.so")


def build_library(force: bool = False, jobs: int = 8) -> str:
    csrc = os.path.join(PKG, "csrc")
    if force:
        subprocess.run(["make", "-s", "-C", csrc, "clean"], check=True)
    subprocess.run(["make", "-s", "-C", csrc, f"-j{jobs}"], check=True)
    if not os.path.exists(LIB):
        raise RuntimeError(f"build did not produce {LIB}")
    return LIB


if __name__ == "__main__":
    print(build_library())
