"""Compile libnelisp_cuda (sm_100a), the protocol server and the CLIs in-tree
with nvcc (-gencode arch=compute_100a,code=sm_100a -lineinfo)."""
from __future__ import annotations

import os
import subprocess

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build(jobs: int = 8) -> None:
    subprocess.run(["make", "-s", "-C", PKG_DIR, f"-j{jobs}"], check=True)


if __name__ == "__main__":
    build()
