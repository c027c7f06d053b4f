"""Build the in-tree binaries of the package (run from anywhere):

  libtdc_sm100.so                 nvcc, -gencode arch=compute_100a,code=sm_100a:
                                  the kernels + the C ABI of include/tdc_dwconv.h
                                  (static cudart, no libcuda link: the TMA encoder
                                  is fetched with cudaGetDriverEntryPoint)
  _tma_dwconv_C<EXT_SUFFIX>       g++: the PyTorch extension (csrc/bindings.cpp),
                                  linked to libtdc_sm100.so through rpath $ORIGIN

Both land next to this file, so the directory is importable as-is
(``import tma_dwconv`` with this directory on ``sys.path``).  Rebuilds only
what is older than its sources.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB = os.path.join(HERE, "libtdc_sm100.so")
EXT = os.path.join(HERE, "_tma_dwconv_C" + sysconfig.get_config_var("EXT_SUFFIX"))

# (No --split-compile: it builds ~4x faster but, with every instantiation in
# one translation unit, made the 7x7 direct-scheme kernels spill ~800 B.)
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
              "-Xcompiler", "-fPIC,-fvisibility=hidden", "-Xptxas", "-v"]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> str:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout[-6000:] + r.stderr[-6000:])
        raise RuntimeError(f"build step failed: {cmd[0]}")
    return r.stdout + r.stderr


def _deps(*names: str) -> list[str]:
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return [os.path.join(CSRC, n) for n in names] + hdrs + [os.path.join(INCLUDE, "tdc_dwconv.h")]


def _tmp(path: str) -> str:
    """A temporary name beside `path`: a binary is written there and renamed
    into place, so no reader ever sees a partly written file."""
    d, f = os.path.split(path)
    return os.path.join(d, f".{f}.{os.getpid()}.tmp")


def build_lib(force: bool = False) -> str:
    deps = _deps("tdc_capi.cu")
    if force or _stale(LIB, deps):
        nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
        tmp = _tmp(LIB)
        out = _run([nvcc, *NVCC_FLAGS, "-shared", f"-I{INCLUDE}", f"-I{CSRC}",
                    os.path.join(CSRC, "tdc_capi.cu"), "-o", tmp])
        os.replace(tmp, LIB)
        with open(os.path.join(HERE, "libtdc_sm100.ptxas.txt"), "w") as f:
            f.write("\n".join(l for l in out.splitlines() if "ptxas" in l or "spill" in l) + "\n")
    return LIB


def build_ext(force: bool = False) -> str:
    deps = _deps("bindings.cpp") + [LIB]
    if force or _stale(EXT, deps):
        import torch
        import torch.utils.cpp_extension as ce
        incs = ce.include_paths("cuda") + [sysconfig.get_paths()["include"], INCLUDE]
        libdirs = ce.library_paths("cuda")
        cmd = ["g++", "-shared", "-fPIC", "-O2", "-std=c++17",
               "-DTORCH_EXTENSION_NAME=_tma_dwconv_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
               f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
               *[f"-I{i}" for i in incs], os.path.join(CSRC, "bindings.cpp"), "-o", _tmp(EXT),
               f"-L{HERE}", "-ltdc_sm100", "-Wl,-rpath,$ORIGIN",
               *[f"-L{d}" for d in libdirs],
               "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
               "-lcudart"]
        _run(cmd)
        os.replace(_tmp(EXT), EXT)
    return EXT


def build_all(force: bool = False) -> None:
    build_lib(force)
    build_ext(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(LIB)
    print(EXT)
