"""Build libaugur_kv.so in-tree for sm_100a.

    python -m augur_b200.csrc.build

nvcc cross-compiles without a GPU. The library is written next to the
package (augur_b200/libaugur_kv.so) so it travels with the source tree; the
CUDA runtime is linked statically, so the .so needs only the NVIDIA driver.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
SOURCES = [os.path.join(HERE, f) for f in ("augur_kv.cu", "augur_attn.cu", "augur_rope.cu", "augur_decode.cu", "augur_prefill.cu")]
HEADERS = [os.path.join(ROOT, "include", "augur_kv.h"), os.path.join(HERE, "common.cuh")]
OUTPUT = os.path.join(PKG, "libaugur_kv.so")

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-shared",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def needs_build() -> bool:
    if not os.path.exists(OUTPUT):
        return True
    out_mtime = os.path.getmtime(OUTPUT)
    return any(os.path.getmtime(p) > out_mtime for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if a source is newer than it; return its path."""
    if not force and not needs_build():
        return OUTPUT
    tmp = OUTPUT + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-o", tmp, *SOURCES]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
