"""Builds the ONNX Runtime stand-in and the libraries the tests load through it -- TEST
INFRASTRUCTURE, outputs only under oracle/_ref/ (git-ignored; travels with the tree):

  libort_shim_host.so      the session side (ort_host.cc)
  libbolt_ort_shim.so      nemotron_ops_b200/ort/bolt_ort.cc (the product's ORT adapter) compiled
                           against the stand-in header, linked to nemotron_ops_b200/libbolt_b200.so
  libbolt_ref.so           the reference's own src/bolt_ops.cu compiled from its checkout for
                           sm_100a against the stand-in header -- only where the checkout exists
                           (BOLT_REFERENCE_DIR, else the build container's read-only checkout);
                           elsewhere the prebuilt file is used if present

    python oracle/ort_shim/build.py [--force]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(ROOT, "oracle", "_ref")
PKG = os.path.join(ROOT, "nemotron_ops_b200")
HOST = os.path.join(OUT, "libort_shim_host.so")
ADAPTER = os.path.join(OUT, "libbolt_ort_shim.so")
REF = os.path.join(OUT, "libbolt_ref.so")


def _stale(target, deps):
    return not os.path.exists(target) or any(os.path.getmtime(d) > os.path.getmtime(target) for d in deps if
                                             os.path.exists(d))


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def reference_dir():
    d = os.environ.get("BOLT_REFERENCE_DIR", "/root/reference")
    return d if os.path.exists(os.path.join(d, "src", "bolt_ops.cu")) else None


def build(force: bool = False, reference: bool = True) -> dict:
    os.makedirs(OUT, exist_ok=True)
    hdr = os.path.join(HERE, "onnxruntime_cxx_api.h")
    cxx = shutil.which("g++") or "g++"
    src = os.path.join(HERE, "ort_host.cc")
    if force or _stale(HOST, [src, hdr]):
        _run([cxx, "-std=c++17", "-O2", "-fPIC", "-shared", "-fvisibility=hidden", "-I", HERE, src, "-ldl", "-o", HOST])
    lib = os.path.join(PKG, "libbolt_b200.so")
    adapter_src = os.path.join(PKG, "ort", "bolt_ort.cc")
    if force or _stale(ADAPTER, [adapter_src, hdr, lib, os.path.join(ROOT, "include", "bolt_b200.h")]):
        _run([cxx, "-std=c++17", "-O2", "-fPIC", "-shared", "-fvisibility=hidden", "-I", HERE, "-I",
              os.path.join(ROOT, "include"), adapter_src, "-L", PKG, "-l:libbolt_b200.so",
              "-Wl,-rpath,$ORIGIN/../../nemotron_ops_b200", "-o", ADAPTER])
    out = {"host": HOST, "adapter": ADAPTER, "reference": REF if os.path.exists(REF) else None}
    rdir = reference_dir() if reference else None
    if rdir:
        rsrc = os.path.join(rdir, "src", "bolt_ops.cu")
        if force or _stale(REF, [rsrc, hdr]):
            nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
            # the reference's own source, unmodified, recompiled for B200 (its CMakeLists uses -arch=sm_90)
            _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo", "-shared",
                  "-Xcompiler", "-fPIC", "-I", HERE, "-I", os.path.join(rdir, "src"), rsrc, "-o", REF])
        out["reference"] = REF
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    print(build(a.force))


if __name__ == "__main__":
    sys.exit(main())
