"""Build libbolt_b200.so in-tree with nvcc for sm_100a (B200).

    python -m nemotron_ops_b200.build [--force] [-j N]

Every csrc/*.cu is compiled to an object under csrc/_build/ (relocatable device code, so the
translation units share the device status word), then nvcc links them into
nemotron_ops_b200/libbolt_b200.so.  Objects are rebuilt when any source or header is newer.
With ORT_INCLUDE_DIR set (ONNX Runtime's headers), ort/bolt_ort.cc is also built into
libbolt_b200_ort.so, the library an ORT session registers (register_custom_ops_library).
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(CSRC, "_build")
LIB = os.path.join(PKG, "libbolt_b200.so")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-rdc=true", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "-diag-suppress", "177", "-I", INCLUDE]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = _headers()
    cc = nvcc()

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if force or _stale(obj, [src] + hdrs):
            cmd = [cc, *ARCH, *FLAGS, "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources))
    if force or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [cc, *ARCH, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", *objs, "-o", tmp]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def build_ort_adapter(force: bool = False) -> str:
    """libbolt_b200_ort.so: the ONNX Runtime adapter (ort/bolt_ort.cc, exports RegisterCustomOps),
    compiled only when ORT_INCLUDE_DIR names a directory holding onnxruntime_cxx_api.h (as the
    reference's CMakeLists.txt requires); returns its path, or "" when the headers are absent."""
    inc = os.environ.get("ORT_INCLUDE_DIR", "")
    if not inc or not os.path.exists(os.path.join(inc, "onnxruntime_cxx_api.h")):
        return ""
    lib = build(force)
    out = os.path.join(PKG, "libbolt_b200_ort.so")
    src = os.path.join(PKG, "ort", "bolt_ort.cc")
    if force or _stale(out, [src, lib, os.path.join(INCLUDE, "bolt_b200.h")]):
        cmd = [shutil.which("g++") or "g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-I", inc, "-I", INCLUDE, src,
               "-L", PKG, "-l:libbolt_b200.so", "-Wl,-rpath,$ORIGIN", "-o", out]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"ORT adapter build failed:\n{r.stdout}\n{r.stderr}")
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args(argv)
    print(build(a.force, a.j, a.v))
    ort = build_ort_adapter(a.force)
    if ort:
        print(ort)


if __name__ == "__main__":
    sys.exit(main())
