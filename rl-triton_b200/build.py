"""Build librlscan.so (sm_100a) in-tree.

    python rl-triton_b200/build.py [--verbose]

Compiles csrc/*.cu with nvcc for sm_100a only and writes
rl_triton/_lib/librlscan.so next to the Python package, so the library
travels with the source tree.  The C ABI is declared in include/rlscan.h.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "rl_triton", "_lib")
LIB = os.path.join(LIBDIR, "librlscan.so")
TORCH_LIB = os.path.join(LIBDIR, "librlscan_torch.so")
SOURCES = ["rlscan.cu", "segment.cu", "ppo.cu"]
HEADERS = ["common.cuh", "algs.cuh", "scan_kernel.cuh", "rows_kernel.cuh", "rows2_kernel.cuh", "tile_kernel.cuh", "tile_policies.cuh", "host_shared.h"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; librlscan.so needs the CUDA toolkit to build")
    return cand


def nvcc_flags(verbose: bool = False) -> list[str]:
    flags = [
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
        "-I", os.path.join(ROOT, "include"),
        "-I", CSRC,
    ]
    if verbose:
        flags += ["-Xptxas", "-v"]
    return flags


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "rlscan.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def torch_flags() -> list[str]:
    import torch
    from torch.utils import cpp_extension as ce

    inc = [os.path.join(os.path.dirname(torch.__file__), "include"),
           os.path.join(os.path.dirname(torch.__file__), "include", "torch", "csrc", "api", "include"),
           os.path.join(os.path.dirname(os.path.dirname(nvcc_path())), "include")]
    libdir = ce.library_paths()[0]
    abi = "1" if torch.compiled_with_cxx11_abi() else "0"
    return ([f"-I{d}" for d in inc] + ["-I", os.path.join(ROOT, "include"), f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
                                       "-DTORCH_API_INCLUDE_EXTENSION_H=0"],
            [f"-L{libdir}", f"-Wl,-rpath,{libdir}", f"-L{LIBDIR}", "-Wl,-rpath,$ORIGIN", "-lrlscan", "-lc10",
             "-lc10_cuda", "-ltorch_cpu", "-ltorch"])


def build_torch_ops(force: bool = False) -> str:
    """librlscan_torch.so: the rl_triton::* PyTorch operators (torch_ops.cpp),
    linked against librlscan.so."""
    src = os.path.join(CSRC, "torch_ops.cpp")
    if (not force and os.path.exists(TORCH_LIB) and os.path.getmtime(TORCH_LIB) > os.path.getmtime(src)
            and os.path.getmtime(TORCH_LIB) > os.path.getmtime(LIB)):
        return TORCH_LIB
    cflags, ldflags = torch_flags()
    tmp = TORCH_LIB + ".tmp"
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", *cflags, src, "-o", tmp, *ldflags]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("g++ failed building librlscan_torch.so")
    os.replace(tmp, TORCH_LIB)
    return TORCH_LIB


OBJDIR = os.path.join(HERE, "_build")


def _deps(src: str) -> list[str]:
    # every source includes some of the headers; rebuild on any of them
    return [os.path.join(CSRC, src)] + [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include",
                                                                                               "rlscan.h")]


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile each csrc/*.cu to an object (in parallel, skipping objects newer
    than their sources and headers), link librlscan.so, then the operator
    library."""
    if not force and not _stale():
        build_torch_ops()
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(OBJDIR, exist_ok=True)
    procs = []
    objs = []
    for src in SOURCES:
        obj = os.path.join(OBJDIR, src.replace(".cu", ".o"))
        objs.append(obj)
        if (not verbose and os.path.exists(obj)
                and all(os.path.getmtime(obj) > os.path.getmtime(d) for d in _deps(src))):
            continue
        cmd = [nvcc_path(), *nvcc_flags(verbose), "-c", os.path.join(CSRC, src), "-o", obj + ".tmp"]
        procs.append((obj, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
    failed = False
    for obj, pr in procs:
        out, err = pr.communicate()
        if pr.returncode != 0:
            sys.stderr.write(out + err)
            failed = True
        else:
            if verbose:
                sys.stderr.write(err)
            os.replace(obj + ".tmp", obj)
    if failed:
        raise RuntimeError("nvcc failed building librlscan.so")
    tmp = LIB + ".tmp"
    cmd = [nvcc_path(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xlinker", "-soname=librlscan.so",
           "-o", tmp, *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed linking librlscan.so")
    os.replace(tmp, LIB)
    build_torch_ops(force=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill report")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--torch-only", action="store_true", help="rebuild only librlscan_torch.so")
    a = ap.parse_args()
    if a.torch_only:
        print(build_torch_ops(force=True))
    else:
        print(build(force=a.force or a.verbose, verbose=a.verbose))
