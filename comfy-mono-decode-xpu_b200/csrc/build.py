"""Build libmono_b200.so (the C ABI of include/mono_b200.h) for sm_100a with nvcc.

Objects go to csrc/_build/, the library next to the Python package (mono_b200/libmono_b200.so), so it
travels with the source tree. Rebuilds only what changed (sources or headers newer than the object).
Usage: python build.py [--force] [--verbose]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(ROOT, "mono_b200", "libmono_b200.so")
INCLUDE = os.path.join(os.path.dirname(ROOT), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", INCLUDE]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def sources():
    return sorted(f for f in os.listdir(HERE) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(HERE, f) for f in os.listdir(HERE) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(INCLUDE, "mono_b200.h"))
    return hs


def _stale(obj, src, newest_header):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def build(force=False, verbose=False, extra=None):
    os.makedirs(BUILD, exist_ok=True)
    newest_header = max(os.path.getmtime(h) for h in headers())
    cmds, objs = [], []
    for s in sources():
        src = os.path.join(HERE, s)
        obj = os.path.join(BUILD, s[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, src, newest_header):
            cmds.append([nvcc(), *ARCH, *FLAGS, *(extra or []), "-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, sep="\n", flush=True)

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(run, cmds))
    if cmds or force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-lrt", "-lpthread", "-ldl"])
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
