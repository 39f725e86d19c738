"""Build libattnb.so (sm_100a kernels + C ABI + C++ shims) and the `_attn_cpu`
pybind11 module in-tree, next to the Python package.

    python attn-cpu_b200/build.py [--force] [--verbose]

nvcc cross-compiles for sm_100a, so this runs on machines without a GPU.
Objects go to attn-cpu_b200/_build/; the two shared objects to
attn-cpu_b200/attn_cpu/.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
PKG = os.path.join(HERE, "attn_cpu")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = "/usr/bin/g++"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-ccbin", CXX,
    "-I", CSRC, "-I", INCLUDE,
]

LIB = os.path.join(PKG, "libattnb.so")


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    return r.stdout + r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    objs = []
    jobs = []
    log = []
    for src in cu:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _newer(obj, [src] + headers + [__file__]):
            cmd = [NVCC] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_info else []) + \
                ["-c", src, "-o", obj]
            jobs.append(cmd)
    shim_src = os.path.join(CSRC, "shims.cpp")
    shim_obj = os.path.join(BUILD, "shims.cpp.o")
    objs.append(shim_obj)
    if force or _newer(shim_obj, [shim_src] + headers):
        jobs.append([CXX, "-O2", "-fPIC", "-std=c++17", "-fvisibility=default", "-I", INCLUDE,
                     "-c", shim_src, "-o", shim_obj])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for out in ex.map(lambda c: _run(c, verbose), jobs):
            log.append(out)
    if force or _newer(LIB, objs):
        _run([NVCC, "-shared", "-ccbin", CXX, "-o", LIB] + objs +
             ["-Xlinker", "--version-script=" + os.path.join(CSRC, "exports.map")], verbose)
    # pybind11 module linked against libattnb.so (rpath $ORIGIN).
    import pybind11

    ext = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    mod = os.path.join(PKG, "_attn_cpu" + ext)
    mod_src = os.path.join(CSRC, "pymodule.cpp")
    if force or _newer(mod, [mod_src, LIB] + headers):
        py_inc = sysconfig.get_paths()["include"]
        _run([CXX, "-O2", "-shared", "-fPIC", "-std=c++17", "-fvisibility=hidden",
              "-I", pybind11.get_include(), "-I", py_inc, "-I", INCLUDE, mod_src,
              "-L", PKG, "-lattnb", "-Wl,-rpath,$ORIGIN", "-o", mod], verbose)
    return "".join(log)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills (-Xptxas -v)")
    a = ap.parse_args()
    out = build(a.force, a.verbose, a.ptxas_info)
    if a.ptxas_info:
        print(out)
    print("built", LIB)
