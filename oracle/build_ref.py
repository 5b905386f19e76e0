"""Compile the REFERENCE's own CUDA extension sources into oracle/_ref/ -- test infrastructure.

The reference (nmquan1503/ssm-mamba) ships two PyTorch CUDA extensions built by its
setup.py (setup.py:8-47).  This recipe does not run that build system: it calls nvcc and
g++ directly on the reference's source files where they lie (read-only), with the
reference's own flags (-O3 --use_fast_math, setup.py:10-16) and an explicit sm_100 target.
The only changes are the extension names, set through the TORCH_EXTENSION_NAME macro to
`ref_selective_scan` / `ref_selective_update`, so that the reference kernels can be loaded
in the same process as this repository's drop-in modules named `selective_scan` /
`selective_update`.

It also stages the reference's Python package (its __init__.py and ops/, modules/,
models/, utils/) unchanged into oracle/_ref/ssm_mamba_ref/, so that GPU tests can run the
reference's own modules (Mamba, CausalLM) once on its kernels and once on this library's
drop-in extension modules (tests/test_reference_modules_gpu.py).

Outputs go only to oracle/_ref/ (git-ignored; it travels to the GPU box with the tree).
The reference kernels run on the GPU only (the reference has no CPU path), so they are
used by GPU tests and by tests/golden/make_golden.py to pin the CPU oracle.

The reference checkout is found through the environment variable SSM_REFERENCE_ROOT, or
as a directory named `reference` beside this repository; without either, nothing is built.
"""
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
REF = os.environ.get("SSM_REFERENCE_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
# the reference's Python package, staged under this name (its own name has a hyphen)
PKG = "ssm_mamba_ref"
PKG_PARTS = ["__init__.py", "ops", "modules", "models", "utils"]

EXTS = {
    "ref_selective_scan": ["selective_scan/bindings.cpp", "selective_scan/selective_scan.cpp",
                           "selective_scan/forward_kernel.cu", "selective_scan/backward_kernel.cu"],
    "ref_selective_update": ["selective_update/bindings.cpp",
                             "selective_update/selective_update.cpp",
                             "selective_update/kernel.cu"],
}


def _torch_flags():
    import torch
    from torch.utils import cpp_extension as ce
    inc = ce.include_paths() + [sysconfig.get_paths()["include"]]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    libdirs = ce.library_paths()
    return inc, abi, libdirs


def lib_path(name: str) -> str:
    return os.path.join(OUT, name + sysconfig.get_config_var("EXT_SUFFIX"))


def available() -> bool:
    return all(os.path.exists(lib_path(n)) for n in EXTS)


def package_available() -> bool:
    return os.path.exists(os.path.join(OUT, PKG, "__init__.py"))


def stage_package() -> bool:
    """Copy the reference's Python package (unchanged) to oracle/_ref/ssm_mamba_ref/."""
    import shutil
    if not os.path.isfile(os.path.join(REF, "__init__.py")):
        return False
    dst = os.path.join(OUT, PKG)
    tmp = dst + ".tmp"
    shutil.rmtree(tmp, ignore_errors=True)
    os.makedirs(tmp)
    for part in PKG_PARTS:
        src = os.path.join(REF, part)
        if os.path.isdir(src):
            shutil.copytree(src, os.path.join(tmp, part), ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
        elif os.path.isfile(src):
            shutil.copy2(src, os.path.join(tmp, part))
    shutil.rmtree(dst, ignore_errors=True)
    os.replace(tmp, dst)
    return True


def build(force: bool = False) -> bool:
    """Build both reference extensions and stage the reference's Python package.  Returns
    False when the reference tree is absent."""
    csrc = os.path.join(REF, "csrc")
    if not os.path.isdir(csrc):
        return False
    os.makedirs(OUT, exist_ok=True)
    if force or not package_available():
        stage_package()
    if available() and not force:
        return True
    os.makedirs(OUT, exist_ok=True)
    inc, abi, libdirs = _torch_flags()
    incf = sum((["-I", p] for p in inc + [csrc]), [])
    jobs = []
    for name, srcs in EXTS.items():
        defs = [f"-DTORCH_EXTENSION_NAME={name}", "-DTORCH_API_INCLUDE_EXTENSION_H",
                f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
        for s in srcs:
            src = os.path.join(csrc, s)
            obj = os.path.join(OUT, name + "__" + os.path.basename(s) + ".o")
            if s.endswith(".cu"):
                cmd = [os.path.join(CUDA, "bin", "nvcc"), "-c", src, "-o", obj, "-O3", "-std=c++17",
                       "--use_fast_math", "--expt-relaxed-constexpr", "--expt-extended-lambda",
                       "-gencode", "arch=compute_100,code=sm_100", "-Xcompiler", "-fPIC",
                       "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
                       "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__",
                       ] + defs + incf
            else:
                cmd = ["g++", "-c", src, "-o", obj, "-O3", "-std=c++17", "-fPIC",
                       "-I", os.path.join(CUDA, "include")] + defs + incf
            jobs.append((name, obj, cmd))
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for (_, _, cmd), rc in zip(jobs, ex.map(lambda j: subprocess.call(j[2]), jobs)):
            if rc != 0:
                raise RuntimeError("reference compile failed: " + " ".join(cmd))
    for name in EXTS:
        objs = [o for (n, o, _) in jobs if n == name]
        ldirs = sum((["-L", d, "-Wl,-rpath," + d] for d in libdirs), [])
        cmd = ["g++", "-shared", "-o", lib_path(name)] + objs + ldirs + [
            "-L", os.path.join(CUDA, "lib64"), "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
            "-ltorch_cuda", "-ltorch_python", "-lcudart"]
        subprocess.check_call(cmd)
    for (_, o, _) in jobs:
        os.remove(o)
    return True


def load(name: str):
    """Import one of the compiled reference extensions under its ref_* name."""
    import importlib.util
    import torch  # noqa: F401  (the extension links libtorch)
    spec = importlib.util.spec_from_file_location(name, lib_path(name))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ok = build(force="--force" in sys.argv)
    print("built" if ok else "reference tree absent", OUT)
