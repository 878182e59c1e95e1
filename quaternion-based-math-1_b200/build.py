"""Build the in-tree shared library ``lib/libqlin_b200.so`` for sm_100a.

The library exports the C ABI declared in ``include/qlin_b200.h``.  It links
the CUDA runtime statically and resolves the one driver entry point it needs
(``cuTensorMapEncodeTiled``) at run time, so it depends on nothing but the
driver.  Run ``python quaternion-based-math-1_b200/build.py`` (or
``__graft_entry__.build()``); nvcc cross-compiles without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_DIR = os.path.join(PKG, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libqlin_b200.so")
SOURCES = [os.path.join(CSRC, "qlin_abi.cu")]
DEPENDS = SOURCES + [os.path.join(CSRC, f) for f in ("qlin_common.cuh", "qlin_gemv.cuh", "qlin_pair.cuh",
                                                      "qlin_simt.cuh", "qlin_tc.cuh")] + [
    os.path.join(REPO, "include", "qlin_b200.h")
]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-Xlinker", "-soname=libqlin_b200.so",
    "-Xptxas", "-v",
    "-I", os.path.join(REPO, "include"),
]


def find_nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


# CPython binding of qlin_forward_ex (the per-call path; ctypes otherwise)
PYCALL_SRC = os.path.join(CSRC, "qlin_pycall.c")
PYCALL_PATH = os.path.join(LIB_DIR, "_qlin_call" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


# torch extension: the modules' inference forward in C++
TORCH_EXT_SRC = os.path.join(CSRC, "qlin_torch_ext.cpp")
TORCH_EXT_PATH = os.path.join(LIB_DIR, "_qlin_torch" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def needs_build() -> bool:
    outs = (LIB_PATH, PYCALL_PATH, TORCH_EXT_PATH)
    if not all(os.path.exists(p) for p in outs):
        return True
    t = min(os.path.getmtime(p) for p in outs)
    return any(os.path.getmtime(p) > t for p in DEPENDS + [PYCALL_SRC, TORCH_EXT_SRC])


def build_torch_ext() -> None:
    import torch
    import torch.utils.cpp_extension as ce

    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cuda_home = ce.CUDA_HOME or "/usr/local/cuda"
    cxx = os.environ.get("QLIN_CXX") or shutil.which("g++") or "c++"
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-DTORCH_EXTENSION_NAME=_qlin_torch", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-I", os.path.join(os.path.dirname(torch.__file__), "include"),
           "-I", os.path.join(os.path.dirname(torch.__file__), "include", "torch", "csrc", "api", "include"),
           "-I", os.path.join(cuda_home, "include"), "-I", sysconfig.get_paths()["include"],
           "-I", os.path.join(REPO, "include"),
           "-o", TORCH_EXT_PATH + ".tmp", TORCH_EXT_SRC,
           "-L", torch_lib, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
           "-L", LIB_DIR, "-lqlin_b200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"building the torch extension failed:\n{res.stderr[-3000:]}")
    os.replace(TORCH_EXT_PATH + ".tmp", TORCH_EXT_PATH)


def build_pycall() -> None:
    cc = os.environ.get("QLIN_CC") or shutil.which("gcc") or "cc"
    cmd = [cc, "-O2", "-shared", "-fPIC", "-I", sysconfig.get_paths()["include"], "-I",
           os.path.join(REPO, "include"), "-o", PYCALL_PATH + ".tmp", PYCALL_SRC, "-L", LIB_DIR,
           "-lqlin_b200", "-Wl,-rpath,$ORIGIN"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"building the CPython binding failed:\n{res.stderr[-2000:]}")
    os.replace(PYCALL_PATH + ".tmp", PYCALL_PATH)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [find_nvcc(), *NVCC_FLAGS, "-o", tmp, *SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    log = os.path.join(LIB_DIR, "build.log")
    with open(log, "w") as f:
        f.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}); see {log}\n{res.stderr[-4000:]}")
    os.replace(tmp, LIB_PATH)
    build_pycall()
    build_torch_ext()
    if verbose:
        print(res.stderr)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
