"""Builds libbmo.so in-tree (bmo_jetson_b200/lib/libbmo.so) for sm_100a.

CUDA sources are compiled by nvcc with ``-gencode arch=compute_100a,code=sm_100a``,
host sources by g++; the shared library links the CUDA runtime statically so it
does not depend on whichever libcudart a host process already loaded.
Rebuilds only objects whose source or headers changed.

    python -m bmo_jetson_b200.build [--force] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "lib", "obj")
LIB = os.path.join(HERE, "lib", "libbmo.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = "/usr/bin/g++"
CUDA_INC = "/usr/local/cuda/include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-ccbin", CXX, "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "-DBMO_BUILDING_SHARED", f"-I{ROOT}/include"]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-ffp-contract=off", "-Wall",
             "-DBMO_BUILDING_SHARED", f"-I{CUDA_INC}", f"-I{ROOT}/include"]


def _sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True))
    cpp = sorted(glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True))
    return cu, cpp


def _headers():
    hs = glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True)
    hs += glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True)
    hs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return hs


def _obj_path(src: str) -> str:
    rel = os.path.relpath(src, CSRC).replace(os.sep, "__")
    return os.path.join(OBJ, rel + ".o")


def _stale(src: str, obj: str, newest_header: float) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def _compile(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    cu, cpp = _sources()
    live = {_obj_path(s) for s in cu + cpp}
    for o in glob.glob(os.path.join(OBJ, "*.o")):  # objects of sources that no longer exist
        if o not in live:
            os.remove(o)
    newest = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    cmds = []
    objs = []
    for s in cu:
        o = _obj_path(s)
        objs.append(o)
        if force or _stale(s, o, newest):
            cmds.append([NVCC] + NVCC_FLAGS + ["-c", s, "-o", o])
    for s in cpp:
        o = _obj_path(s)
        objs.append(o)
        if force or _stale(s, o, newest):
            cmds.append([CXX] + CXX_FLAGS + ["-c", s, "-o", o])
    if cmds:
        jobs = jobs or min(len(cmds), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(jobs) as ex:
            for err in ex.map(_compile, cmds):
                if verbose and err:
                    sys.stderr.write(err)
    lib_time = os.path.getmtime(LIB) if os.path.exists(LIB) else -1.0
    if cmds or force or lib_time < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        _compile([NVCC] + ARCH + ["-shared", "-ccbin", CXX, "-o", tmp] + objs +
                 ["-cudart", "static", "-lpthread", "-ldl", "-Xlinker", "--no-undefined"])
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.j, a.v))


if __name__ == "__main__":
    main()
