"""In-tree build of the two native artefacts of this package.

  liblsek.so       the sm_100a kernels and the C ABI of include/lsek.h,
                   compiled by nvcc (-gencode arch=compute_100a,code=sm_100a),
                   cudart linked statically, no torch dependency
  _C<ext-suffix>   the torch binding (pybind11), compiled by g++; it calls
                   liblsek.so through the C ABI and is found next to it via
                   an $ORIGIN rpath

Both land in this package directory so they travel with the source tree.
A target is rebuilt only when one of its inputs is newer.

    python layerstormexpertkernels_b200/build.py [--force] [--jobs N]

This file imports nothing from its package, so it runs in a checkout that
has no native extension yet.  Run it as a script (or load it by path, as
__graft_entry__.build() does): `python -m layerstormexpertkernels_b200.build`
executes the package __init__ first, and that refuses to load without the
extension.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

CU_SOURCES = ["common.cu", "gating.cu", "permute.cu", "swiglu.cu", "grouped_gemm.cu",
              "layer.cu", "ep.cu"]
HEADERS = ["common.cuh", "swiglu.cuh"]
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = GENCODE + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                        "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
                        "-I" + INCLUDE, "-I" + CSRC]

LIB = os.path.join(PKG, "liblsek.so")
EXT = os.path.join(PKG, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))
EXT_SOURCE = os.path.join(CSRC, "torch_binding.cpp")


def _newer(target: str, inputs: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(i) > t for i in inputs)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {os.path.basename(cmd[0])} (exit {r.returncode})")


def build_lib(force: bool = False, jobs: int = 8, extra_flags: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "lsek.h")]
    objs, todo = [], []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _newer(o, [s] + headers):
            todo.append([NVCC] + NVCC_FLAGS + (extra_flags or []) + ["-c", s, "-o", o])
    with ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        list(ex.map(_run, todo))
    if force or todo or _newer(LIB, objs):
        _run([NVCC] + GENCODE + ["-shared", "-o", LIB] + objs + ["-Xlinker", "--no-undefined",
                                                                  "-lpthread", "-ldl", "-lrt"])
    return LIB


def build_ext(force: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension as ce

    if not (force or _newer(EXT, [EXT_SOURCE, LIB, os.path.join(INCLUDE, "lsek.h")])):
        return EXT
    incs = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], INCLUDE]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = (["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-w", EXT_SOURCE, "-o", EXT,
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
            "-DTORCH_API_INCLUDE_EXTENSION_H"]
           + ["-I" + i for i in incs] + ["-L" + d for d in libdirs]
           + ["-L" + PKG, "-llsek", "-Wl,-rpath,$ORIGIN"]
           + ["-Wl,-rpath," + d for d in libdirs]
           + ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
              "-lcudart"])
    _run(cmd)
    return EXT


def build(force: bool = False, jobs: int = 8) -> None:
    build_lib(force=force, jobs=jobs)
    build_ext(force=force)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--lib-only", action="store_true")
    args = ap.parse_args()
    build_lib(force=args.force, jobs=args.jobs)
    if not args.lib_only:
        build_ext(force=args.force)
    print(LIB)
    if not args.lib_only:
        print(EXT)


if __name__ == "__main__":
    main()
