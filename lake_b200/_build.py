"""In-tree native build for lake_b200.

Compiles
  * ``csrc/kernels/*.cu``   -> sm_100a objects (nvcc, no torch headers)
  * ``csrc/bindings/ops.cpp`` -> torch/pybind11 binding
  * links both into ``lake_b200/_C.so`` (CUDA runtime linked statically)
  * ``csrc/host/**/*.cpp``  -> ``lake_b200/_host.so`` (pybind11 + static CUDA runtime, no torch)

``--debug`` builds the bounds-checked variant of the kernels and bindings instead
(``-DLAKEB_DEBUG_CHECKS``) into ``lake_b200/_C_debug.so``: index checks record an
error code in the status word and skip the access. ``LAKEB_DEBUG_CHECKS=1`` makes
``lake_b200.ops`` load it in place of ``_C``.

The build is driven by a generated ninja file under ``_build/`` so repeated
builds are incremental. Nothing is JIT-compiled at import time: the ``.so``
files live next to the Python sources and travel with the tree.

Usage: ``python -m lake_b200._build [-j N] [--debug]``.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys
import sysconfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(ROOT, "_build")
PKG = os.path.join(ROOT, "lake_b200")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _torch_paths():
    import torch

    tdir = os.path.dirname(torch.__file__)
    inc = [os.path.join(tdir, "include"), os.path.join(tdir, "include", "torch", "csrc", "api", "include")]
    lib = os.path.join(tdir, "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return inc, lib, abi


def _pybind_inc():
    import pybind11

    return pybind11.get_include()


def _q(xs):
    return " ".join(xs)


def write_ninja(debug: bool = False) -> str:
    tinc, tlib, abi = _torch_paths()
    pyinc = sysconfig.get_paths()["include"]
    nvcc = os.path.join(CUDA_HOME, "bin", "nvcc")
    cuda_inc = os.path.join(CUDA_HOME, "include")
    cuda_lib = os.path.join(CUDA_HOME, "lib64")
    kdir = os.path.join(ROOT, "csrc", "kernels")

    mod = "_C_debug" if debug else "_C"
    build_dir = BUILD + ("_debug" if debug else "")
    nv_flags = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                       f"-I{kdir}", "-DNDEBUG"] + (["-DLAKEB_DEBUG_CHECKS"] if debug else [])
    ext_flags = ["-O2", "-fPIC", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
                 f"-DTORCH_EXTENSION_NAME={mod}", f"-DLAKEB_MODULE={mod}", f"-I{pyinc}", f"-I{cuda_inc}",
                 f"-I{kdir}"] + [f"-I{i}" for i in tinc] + (["-DLAKEB_DEBUG_CHECKS"] if debug else [])
    host_flags = ["-O2", "-fPIC", "-std=c++17", f"-I{pyinc}", f"-I{_pybind_inc()}",
                  f"-I{os.path.join(ROOT, 'csrc', 'host')}", f"-I{cuda_inc}", "-fvisibility=hidden", "-Wall", "-Wno-unused-function"]

    lines = [
        "ninja_required_version = 1.3",
        f"nvcc = {nvcc}",
        "cxx = g++",
        f"nvflags = {_q(nv_flags)}",
        f"extflags = {_q(ext_flags)}",
        f"hostflags = {_q(host_flags)}",
        "rule nvcc",
        "  command = $nvcc $nvflags -MD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = NVCC $in",
        "rule cxx_ext",
        "  command = $cxx $extflags -MMD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CXX $in",
        "rule cxx_host",
        "  command = $cxx $hostflags -MMD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CXX $in",
        "rule link_ext",
        f"  command = $cxx -shared $in -o $out -L{tlib} -lc10 -lc10_cuda -ltorch -ltorch_cpu -ltorch_cuda "
        f"-ltorch_python -L{cuda_lib} -lcudart_static -ldl -lrt -lpthread -Wl,-rpath,{tlib}",
        "  description = LINK $out",
        "rule link_host",
        f"  command = $cxx -shared $in -o $out -L{cuda_lib} -lcudart_static -ldl -lrt -lpthread",
        "  description = LINK $out",
    ]
    kobjs = []
    for src in sorted(glob.glob(os.path.join(kdir, "*.cu"))):
        obj = os.path.join(build_dir, "kernels", os.path.basename(src) + ".o")
        lines.append(f"build {obj}: nvcc {src}")
        kobjs.append(obj)
    bind_src = os.path.join(ROOT, "csrc", "bindings", "ops.cpp")
    bind_obj = os.path.join(build_dir, "bindings", "ops.o")
    lines.append(f"build {bind_obj}: cxx_ext {bind_src}")
    lines.append(f"build {os.path.join(PKG, mod + '.so')}: link_ext {_q(kobjs + [bind_obj])}")

    hobjs = []
    for src in sorted(glob.glob(os.path.join(ROOT, "csrc", "host", "**", "*.cpp"), recursive=True)):
        rel = os.path.relpath(src, os.path.join(ROOT, "csrc", "host")).replace(os.sep, "_")
        obj = os.path.join(BUILD, "host", rel + ".o")
        lines.append(f"build {obj}: cxx_host {src}")
        hobjs.append(obj)
    if hobjs and not debug:
        lines.append(f"build {os.path.join(PKG, '_host.so')}: link_host {_q(hobjs)}")
    os.makedirs(build_dir, exist_ok=True)
    path = os.path.join(build_dir, "build.ninja")
    text = "\n".join(lines) + "\n"
    old = open(path).read() if os.path.exists(path) else None
    if old != text:
        with open(path, "w") as f:
            f.write(text)
    return path


def build(jobs: int | None = None, verbose: bool = False, debug: bool = False) -> None:
    write_ninja(debug)
    cmd = ["ninja", "-C", BUILD + ("_debug" if debug else "")]
    if jobs:
        cmd += ["-j", str(jobs)]
    if verbose:
        cmd.append("-v")
    subprocess.run(cmd, check=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--debug", action="store_true", help="bounds-checked build -> lake_b200/_C_debug.so")
    args = ap.parse_args(argv)
    build(args.j, args.v, args.debug)


if __name__ == "__main__":
    sys.exit(main())
