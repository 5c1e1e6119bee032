"""In-tree build of the native parts for sm_100a.

Produces, next to this file:
  libfcci_decode.so                          the C-ABI library (nvcc, static cudart, cuBLAS)
  attn_varlen<ext-suffix>                    pybind module `attn_varlen`
  capture_decode_step<ext-suffix>            pybind module `capture_decode_step`

Usage: python fully_custom_cuda_inference_lamma2_b200/build.py [--force]
(by path: importing the package requires the modules this script builds)
Nothing is compiled when every output is newer than its sources.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
import tempfile

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB = os.path.join(PKG, "libfcci_decode.so")
LIB_SOURCES = ["decode_attn.cu", "capi.cu", "compat.cu", "noalloc.cu", "prefill_attn.cu", "gemv.cu", "step.cu", "exchange.cu"]
LIB_HEADERS = ["ptx.cuh", "tcgen05.cuh", "fcci_internal.h"]
MODULES = {
    "attn_varlen": "attn_varlen_module.cpp",
    "capture_decode_step": "capture_decode_step_module.cpp",
}


def ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def module_path(name: str) -> str:
    return os.path.join(PKG, name + ext_suffix())


def _newer(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(d) <= t for d in deps)


def _run(cmd: list[str], cwd: str | None = None) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=cwd)


def _common_headers() -> list[str]:
    return [os.path.join(INCLUDE, h) for h in ("fcci_decode.h", "fcci_compat.h", "fcci_prefill.h", "fcci_exchange.h")]


def build_library(force: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in LIB_SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in LIB_HEADERS] + _common_headers()
    if not force and _newer(LIB, deps):
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    with tempfile.TemporaryDirectory() as tmp:
        objs = [os.path.join(tmp, os.path.basename(s) + ".o") for s in srcs]
        cmds = [[NVCC, *GENCODE, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC,
                 "-c", s, "-o", o] for s, o in zip(srcs, objs)]
        with ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 1)) as pool:
            list(pool.map(_run, cmds))
        tmp_lib = os.path.join(tmp, "libfcci_decode.so")
        _run([NVCC, *GENCODE, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp_lib, "-lcublas"])
        shutil.move(tmp_lib, LIB)
    return LIB


def build_module(name: str, force: bool = False) -> str:
    src = os.path.join(CSRC, MODULES[name])
    out = module_path(name)
    deps = [src, os.path.join(CSRC, "binding_common.h"), LIB] + _common_headers()
    if not force and _newer(out, deps):
        return out
    import torch
    from torch.utils import cpp_extension as ce

    py_inc = sysconfig.get_paths()["include"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = [
        "-O3", "-std=c++17", "-fPIC", "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        f"-DTORCH_EXTENSION_NAME={name}",
        '-DPYBIND11_COMPILER_TYPE="_gcc"', '-DPYBIND11_STDLIB="_libstdcpp"', '-DPYBIND11_BUILD_ABI="_cxxabi1018"',
        "-I", INCLUDE, "-I", CSRC, "-I", py_inc, "-I", os.path.join(CUDA_HOME, "include"),
    ]
    for inc in ce.include_paths():
        cflags += ["-isystem", inc]
    ldflags = []
    for libdir in ce.library_paths():
        ldflags += ["-L", libdir]
    ldflags += ["-L", PKG, "-lfcci_decode", "-Wl,-rpath,$ORIGIN",
                "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python"]
    with tempfile.TemporaryDirectory() as tmp:
        tmp_out = os.path.join(tmp, os.path.basename(out))
        _run(["g++", *cflags, src, "-o", tmp_out, *ldflags])
        shutil.move(tmp_out, out)
    return out


def build_all(force: bool = False) -> list[str]:
    outs = [build_library(force)]
    for name in MODULES:
        outs.append(build_module(name, force))
    return outs


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
