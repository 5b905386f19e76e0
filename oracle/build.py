"""Build recipe for the CPU oracle (test infrastructure only).

Compiles oracle/scan_ref.c -- the C restatement of the reference scan math -- into
oracle/_build/libscan_ref.so with gcc and OpenMP.  Nothing in the product links it.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libscan_ref.so")
SRCS = [os.path.join(HERE, "scan_ref.c"), os.path.join(HERE, "scan_ref_impl.h")]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in SRCS)


def build(force: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    # -O2 without -ffast-math keeps IEEE semantics for the double-precision oracle.
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-std=c11",
           SRCS[0], "-o", LIB + ".tmp", "-lm"]
    subprocess.check_call(cmd)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
