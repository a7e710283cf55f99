"""Build recipe for the two native libraries of the `ocl` backend.

* ``lib/libpvb2.so``  -- the CUDA kernel library behind the C-ABI in
  ``include/pvb2.h``; compiled by nvcc for sm_100a only, links NCCL.
* ``_C.so``           -- the PyTorch host extension (PrivateUse1 allocator,
  device guard, hooks, generator and the ATen op registrations); plain C++
  against the torch headers, calls into libpvb2 through the C-ABI.

Both land in-tree so they travel with the source tree.  Objects go to
``<repo>/_build``.  Rebuilds are incremental on source/header mtimes.

Usage:  python pytorch_vulkan_b200/_build.py [--force] [-j N]
(run it as a script: importing the package first would need the libraries)
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
BUILD = os.path.join(REPO, "_build")
KDIR = os.path.join(PKG, "csrc", "kernels")
HDIR = os.path.join(PKG, "csrc", "host")
INCLUDE = os.path.join(REPO, "include")
LIBDIR = os.path.join(PKG, "lib")
KLIB = os.path.join(LIBDIR, "libpvb2.so")
EXT = os.path.join(PKG, "_C.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_INC = os.path.join(os.path.dirname(os.path.dirname(NVCC)), "include")
CXX = os.environ.get("PVB2_CXX", "/usr/bin/g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUTLASS_INC = None  # kernels are hand-written; CuTe headers are not needed


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths if os.path.exists(p)), default=0.0)


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed:\n" + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


def _compile_cu(src, force, extra_flags):
    obj = os.path.join(BUILD, "kernels", os.path.basename(src) + ".o")
    deps = [src] + glob.glob(os.path.join(KDIR, "*.cuh")) + [os.path.join(INCLUDE, "pvb2.h")]
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= _newest(deps):
        return obj, ""
    os.makedirs(os.path.dirname(obj), exist_ok=True)
    cmd = [NVCC, "-ccbin", CXX, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "--expt-relaxed-constexpr", "-I", INCLUDE, "-c", src, "-o", obj, *extra_flags]
    out = _run(cmd)
    return obj, out


def _torch_flags():
    import torch
    from torch.utils import cpp_extension as ce

    incs = ce.include_paths()
    libdirs = ce.library_paths()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    py_inc = sysconfig.get_paths()["include"]
    cflags = ["-O2", "-std=c++17", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
              "-DTORCH_API_INCLUDE_EXTENSION_H", "-Wno-unused-parameter", "-Wno-sign-compare"]
    # the CUDA include tree only for the header-only NVTX v3 ranges of the op guard
    for i in incs + [py_inc, CUDA_INC, INCLUDE]:
        cflags += ["-isystem" if i != INCLUDE else "-I", i]
    ldflags = []
    for d in libdirs:
        ldflags += ["-L", d, f"-Wl,-rpath,{d}"]
    ldflags += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-ldl"]
    return cflags, ldflags


def _compile_cpp(src, force, cflags):
    obj = os.path.join(BUILD, "host", os.path.basename(src) + ".o")
    deps = [src] + glob.glob(os.path.join(HDIR, "*.h")) + [os.path.join(INCLUDE, "pvb2.h")]
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= _newest(deps):
        return obj, ""
    os.makedirs(os.path.dirname(obj), exist_ok=True)
    out = _run([CXX, *cflags, "-c", src, "-o", obj])
    return obj, out


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> None:
    jobs = jobs or max(1, os.cpu_count() or 1)
    os.makedirs(LIBDIR, exist_ok=True)
    cus = sorted(glob.glob(os.path.join(KDIR, "*.cu")))
    cpps = sorted(glob.glob(os.path.join(HDIR, "*.cpp")))
    cflags, ldflags = _torch_flags()
    with cf.ThreadPoolExecutor(jobs) as ex:
        kfuts = [ex.submit(_compile_cu, s, force, []) for s in cus]
        hfuts = [ex.submit(_compile_cpp, s, force, cflags) for s in cpps]
        kobjs = []
        for f in kfuts:
            o, out = f.result()
            kobjs.append(o)
            if verbose and out:
                print(out)
        hobjs = []
        for f in hfuts:
            o, out = f.result()
            hobjs.append(o)
            if verbose and out:
                print(out)
    if force or not os.path.exists(KLIB) or os.path.getmtime(KLIB) < _newest(kobjs):
        _run([NVCC, "-ccbin", CXX, *ARCH, "-shared", "-o", KLIB, *kobjs, "-L/usr/lib/x86_64-linux-gnu", "-lnccl",
              "-Xlinker", "-soname=libpvb2.so"])
    if force or not os.path.exists(EXT) or os.path.getmtime(EXT) < max(_newest(hobjs), os.path.getmtime(KLIB)):
        _run([CXX, "-shared", "-o", EXT, *hobjs, "-L", LIBDIR, "-lpvb2", "-Wl,-rpath,$ORIGIN/lib", *ldflags])


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args(argv)
    build(force=a.force, jobs=a.j, verbose=a.v)
    print("built", KLIB, "and", EXT)


if __name__ == "__main__":
    sys.exit(main())
