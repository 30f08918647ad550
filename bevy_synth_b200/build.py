"""Builds libsparseconv.so in-tree for sm_100a with nvcc.

    python -m bevy_synth_b200.build
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc", "sc_lib.cu")
OUT = os.path.join(HERE, "libsparseconv.so")
DEPS = [os.path.join(HERE, "csrc", f) for f in sorted(os.listdir(os.path.join(HERE, "csrc")))
        if f.endswith((".cu", ".cuh", ".h"))] + [
    os.path.join(ROOT, "include", "sparseconv.h")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-I" + os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


STAMP = OUT + ".srchash"


def source_hash() -> str:
    """SHA-256 over the compile command and every source the library is built from."""
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS).encode())
    for d in DEPS:
        h.update(os.path.basename(d).encode())
        with open(d, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def up_to_date() -> bool:
    """True when the in-tree library was built by this module from exactly the
    current sources (the hash written beside it at build time matches)."""
    if not (os.path.exists(OUT) and os.path.exists(STAMP)):
        return False
    with open(STAMP) as f:
        return f.read().strip() == source_hash()


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-o", OUT, SRC]
    subprocess.run(cmd, check=True)
    with open(STAMP, "w") as f:
        f.write(source_hash() + "\n")
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
