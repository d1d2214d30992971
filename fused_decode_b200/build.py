"""Build ``libfd_b200.so`` from ``csrc/*.cu`` for sm_100a with nvcc, then the
``_fastpath`` Python extension (``csrc/fd_fastpath.cpp``) that calls it.

``python -m fused_decode_b200.build`` (or ``__graft_entry__.build()``).  Both
are written next to this file so they travel with the source tree.  Each is
rebuilt only when one of its sources or headers is newer than it.
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys
import sysconfig

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


FASTPATH_SRC = os.path.join(CSRC, "fd_fastpath.cpp")
FASTPATH_OUT = os.path.join(HERE, "_fastpath" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    built = os.path.getmtime(OUT)
    return all(os.path.getmtime(p) <= built for p in _deps())


def _fastpath_up_to_date() -> bool:
    if not os.path.exists(FASTPATH_OUT):
        return False
    built = os.path.getmtime(FASTPATH_OUT)
    deps = [FASTPATH_SRC, OUT, *glob.glob(os.path.join(INCLUDE, "*.h"))]
    return all(os.path.getmtime(p) <= built for p in deps)


def build_fastpath(force: bool = False, verbose: bool = False) -> str:
    """Compile the pybind11 / ATen extension against the installed torch and
    link it to libfd_b200.so (found next to it at run time)."""
    if not force and _fastpath_up_to_date():
        return FASTPATH_OUT
    import torch

    torch_dir = os.path.dirname(torch.__file__)
    torch_lib = os.path.join(torch_dir, "lib")
    cuda_home = os.environ.get("CUDA_HOME") or os.path.dirname(os.path.dirname(os.path.realpath(_nvcc())))
    incs = [os.path.join(torch_dir, "include"), os.path.join(torch_dir, "include", "torch", "csrc", "api", "include"),
            os.path.join(cuda_home, "include"), sysconfig.get_paths()["include"]]
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}", "-I", INCLUDE]
    for inc in incs:
        cmd += ["-isystem", inc]
    tmp = FASTPATH_OUT + ".tmp"
    cmd += [FASTPATH_SRC, "-o", tmp, "-L", HERE, "-lfd_b200", "-Wl,-rpath,$ORIGIN",
            "-L", torch_lib, f"-Wl,-rpath,{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
            "-ltorch_python"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"fastpath build failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, FASTPATH_OUT)
    return FASTPATH_OUT


def build(force: bool = False, verbose: bool = False) -> str:
    _build_library(force, verbose)
    build_fastpath(force, verbose)
    return OUT


# The persistent stack kernel moves registers between its warpgroups with
# setmaxnreg; its split (csrc/fd_stack.cu) fits a launch allotment of at
# least this many registers per thread.  setmaxnreg.inc would wait forever
# for registers the launch never had, so a build whose allotment is smaller
# must not ship.
STACK_MIN_LAUNCH_REGS = 160


def _check_stack_registers(ptxas_log: str) -> None:
    """The persistent stack kernel launches with enough registers for its
    setmaxnreg split, and its one-tile (batch <= 8, NT = 1) instantiations do
    not spill: their prologue and stream share the consumer warps' budget."""
    entry = None
    seen = 0
    for line in ptxas_log.splitlines():
        if "Compiling entry function" in line:
            entry = line
        elif entry and "spill stores" in line and "mlp_stack_kernel" in entry and "Li1ELb" in entry:
            spilled = int(line.split("bytes spill stores")[0].split(",")[-1])
            if spilled:
                raise RuntimeError(f"mlp_stack_kernel (NT = 1) spills {spilled} bytes: {entry}")
        elif entry and "Used" in line and "registers" in line:
            if "mlp_stack_kernel" in entry:
                regs = int(line.split("Used")[1].split("registers")[0])
                if regs < STACK_MIN_LAUNCH_REGS:
                    raise RuntimeError(f"mlp_stack_kernel launches with {regs} registers per thread, below the "
                                       f"{STACK_MIN_LAUNCH_REGS} its setmaxnreg split needs: {entry}")
                seen += 1
            entry = None
    if seen == 0:
        raise RuntimeError("no ptxas register report for mlp_stack_kernel")


def _build_library(force: bool, verbose: bool) -> str:
    if not force and up_to_date():
        return OUT
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = []
    cmds = []
    for src in _sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src).replace(".cu", ".o"))
        objs.append(obj)
        extra = ["-Xptxas", "-v"] if src.endswith("fd_stack.cu") else []
        cmds.append([nvcc, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        return res.stderr

    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, len(cmds))) as pool:
        for cmd, err in zip(cmds, pool.map(run, cmds)):
            if verbose and err:
                print(err, file=sys.stderr)
            if cmd[-3].endswith("fd_stack.cu"):
                _check_stack_registers(err)
    tmp = OUT + ".tmp"
    run([nvcc, *ARCH, "-shared", "-o", tmp, *objs])
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
