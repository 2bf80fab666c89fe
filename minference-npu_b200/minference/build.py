"""Builds libminference_b200.so in-tree with nvcc for sm_100a.

    python -m minference.build
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

_PKG = os.path.dirname(os.path.abspath(__file__))
_CSRC = os.path.join(os.path.dirname(_PKG), "csrc")
_OUT = os.path.join(_PKG, "libminference_b200.so")


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(
        os.path.join(_CSRC, f) for f in os.listdir(_CSRC) if f.endswith((".cu", ".cuh", ".h"))
    ) + [os.path.join(os.path.dirname(os.path.dirname(_PKG)), "include", "minference_b200.h")]


def needs_build() -> bool:
    if not os.path.exists(_OUT):
        return True
    t = os.path.getmtime(_OUT)
    return any(os.path.getmtime(s) > t for s in sources() if os.path.exists(s))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return _OUT
    cmd = [
        nvcc_path(),
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "-shared", "-Xcompiler", "-fPIC",
        "-o", _OUT + ".tmp",
        os.path.join(_CSRC, "mib200_all.cu"),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.check_call(cmd)
    os.replace(_OUT + ".tmp", _OUT)
    return _OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
