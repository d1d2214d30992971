"""Build ``libfd_b200.so`` from ``csrc/*.cu`` for sm_100a with nvcc.

``python -m fused_decode_b200.build`` (or ``__graft_entry__.build()``).  The
library is written next to this file so it travels with the source tree.
Objects are rebuilt only when a source or header is newer than the library.
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT = os.path.join(HERE, "libfd_b200.so")
BUILD_DIR = os.path.join(HERE, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand) and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found")
    return cand


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    built = os.path.getmtime(OUT)
    return all(os.path.getmtime(p) <= built for p in _deps())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = []
    cmds = []
    for src in _sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src).replace(".cu", ".o"))
        objs.append(obj)
        cmds.append([nvcc, *ARCH, *FLAGS, "-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        return res.stderr

    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, len(cmds))) as pool:
        for err in pool.map(run, cmds):
            if verbose and err:
                print(err, file=sys.stderr)
    tmp = OUT + ".tmp"
    run([nvcc, *ARCH, "-shared", "-o", tmp, *objs])
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
