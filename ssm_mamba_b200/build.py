"""In-tree build of the native parts of ssm_mamba_b200.

  lib/libssm_b200.so  -- the sm_100a kernels behind the C ABI of include/ssm_b200.h
                         (nvcc, -gencode arch=compute_100a,code=sm_100a, static cudart)
  _C.<abi>.so         -- the torch binding (g++ against torch's headers), linked to the
                         library above through an $ORIGIN rpath

Run `python ssm_mamba_b200/build.py` (or __graft_entry__.build()) -- by path: importing
the package needs the extension this builds.  Objects go to _build/.
Both outputs are written next to the sources so they travel with the tree.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libssm_b200.so")
EXT = os.path.join(HERE, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))
INCLUDE = os.path.join(ROOT, "include")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")

CU_SOURCES = ["scan_fwd.cu", "scan_bwd.cu", "scan_bwd_pair.cu", "scan_bwd_split.cu", "scan_chunk.cu", "conv1d.cu", "state_update.cu", "capi.cu", "noalloc.cu"]
HEADERS = ["common.cuh", "params.h", "scan_layout.h", "warp_reduce.cuh", "bwd_prologue.cuh"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden"]


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r


def build_lib(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "ssm_b200.h")]
    jobs = []
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src + ".o")
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            jobs.append([NVCC] + NVCC_FLAGS + ["-c", s, "-o", o])
    if jobs:
        with ThreadPoolExecutor(max_workers=len(jobs)) as ex:
            for r in ex.map(_run, jobs):
                if verbose and r.stderr:
                    print(r.stderr, file=sys.stderr)
    if force or _newer(LIB, objs):
        # exported symbols: the extern "C" entry points (default visibility in capi.cu)
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB + ".tmp"] + objs +
             ["-Xlinker", "--exclude-libs=ALL"])
        os.replace(LIB + ".tmp", LIB)
    return LIB


def build_ext(force: bool = False) -> str:
    src = os.path.join(CSRC, "torch_ext.cpp")
    if not force and not _newer(EXT, [src, LIB, os.path.join(INCLUDE, "ssm_b200.h")]):
        return EXT
    import torch
    from torch.utils import cpp_extension as ce
    inc = ce.include_paths() + [sysconfig.get_paths()["include"], os.path.join(CUDA, "include")]
    libdirs = ce.library_paths()
    cmd = ["g++", "-O2", "-shared", "-fPIC", "-std=c++17", src, "-o", EXT + ".tmp",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"]
    cmd += sum((["-I", p] for p in inc), [])
    cmd += ["-L", LIBDIR, "-lssm_b200", "-Wl,-rpath,$ORIGIN/lib"]
    cmd += sum((["-L", d, "-Wl,-rpath," + d] for d in libdirs), [])
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
    _run(cmd)
    os.replace(EXT + ".tmp", EXT)
    return EXT


def build(force: bool = False, verbose: bool = False) -> None:
    build_lib(force=force, verbose=verbose)
    build_ext(force=force)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
    print(EXT)
