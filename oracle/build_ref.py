"""Compile the reference's own CUDA extension into oracle/_ref/ (test infrastructure).

Recipe for the parity checker, not part of the product: it compiles the three
source files of haowen-han/tma-depthwise-conv where they lie
(``/root/reference/csrc/{bindings.cpp,kernel_v0_naive_float4.cu,kernel_tma_ws.cu}``)
with the compiler flags of the reference's ``setup.py:33-43``, without running
the reference's own build system and without copying its sources.  The output
``oracle/_ref/_tma_dwconv_ref_C*.so`` exposes the reference's ``dwconv_v0``,
``dwconv_ws`` and ``dwconv_ws_probe`` under the module name
``_tma_dwconv_ref_C`` (set through ``-DTORCH_EXTENSION_NAME``, the macro the
reference's ``PYBIND11_MODULE`` uses) so it can be imported beside this
repository's ``_tma_dwconv_C``.

Third-party dependency: the reference's CuTe/CUTLASS submodule
(``.gitmodules:1-3``) is empty in the reference checkout and its pinned commit
is not recorded.  The CUTLASS 4.5.0 header tree shipped inside the installed
flashinfer wheel is used instead; the reference uses CuTe only for the TMA
descriptor and mbarrier wrappers, not for arithmetic.

Besides the extension it stages, unchanged, the reference's own test files
``tests/test_dwconv.py``, ``tests/test_ws_time.py`` and ``tests/__init__.py``
into ``oracle/_ref/tests/`` (git-ignored, like the extension), so that a GPU
test can run them against this repository's ``tma_dwconv`` on a machine that
has no reference checkout; and it copies the built extension to
``baseline/_ref/``, where ``bench.py`` loads it to time the reference's own ws
kernel beside this repository's (the same binary; ``oracle/_ref`` serves the
parity tests).

Usage:  TDC_REFERENCE_DIR=<reference checkout> python3 oracle/build_ref.py [--cutlass DIR] [-j N]
        (or --reference DIR).  Without either, nothing is built.
Writes only into oracle/_ref/ and baseline/_ref/.  nvcc cross-compiles for
sm_100a, so no GPU is needed; the result is loaded by the GPU tests on a B200.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
BASELINE_OUT = os.path.join(os.path.dirname(HERE), "baseline", "_ref")
MODULE = "_tma_dwconv_ref_C"
REF_TESTS = ["tests/__init__.py", "tests/test_dwconv.py", "tests/test_ws_time.py"]


def _default_cutlass() -> str | None:
    try:
        import flashinfer  # noqa: F401  (only its data directory is used)
        import importlib.util
        spec = importlib.util.find_spec("flashinfer")
        root = os.path.dirname(spec.origin)
        cand = os.path.join(root, "data", "cutlass")
        return cand if os.path.isdir(os.path.join(cand, "include", "cute")) else None
    except Exception:
        return None


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TDC_REFERENCE_DIR"))
    ap.add_argument("--cutlass", default=os.environ.get("CUTLASS_DIR") or _default_cutlass())
    ap.add_argument("-j", type=int, default=3)
    args = ap.parse_args()
    ref = args.reference
    if not ref:
        print("no reference checkout given (TDC_REFERENCE_DIR or --reference); nothing built",
              file=sys.stderr)
        return 0
    srcs = ["csrc/bindings.cpp", "csrc/kernel_v0_naive_float4.cu", "csrc/kernel_tma_ws.cu"]
    if not all(os.path.exists(os.path.join(ref, s)) for s in srcs):
        print(f"reference sources not found under {ref}; nothing built", file=sys.stderr)
        return 0
    _stage_tests(ref)
    if not args.cutlass:
        print("no CUTLASS header tree found; reference not built", file=sys.stderr)
        return 1
    import torch
    import torch.utils.cpp_extension as ce

    os.makedirs(OUT, exist_ok=True)
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    target = os.path.join(OUT, MODULE + suffix)
    newest_src = max(os.path.getmtime(os.path.join(ref, s)) for s in srcs)
    if os.path.exists(target) and os.path.getmtime(target) >= newest_src:
        _copy_to_baseline(target)
        print(f"up to date: {target}")
        return 0

    cuda_home = ce.CUDA_HOME or "/usr/local/cuda"
    incs = ce.include_paths("cuda") + [sysconfig.get_paths()["include"],
                                       os.path.join(args.cutlass, "include"),
                                       os.path.join(args.cutlass, "tools", "util", "include")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = [f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    inc_flags = [f"-I{i}" for i in incs]
    # reference setup.py:33-43
    nvcc_flags = ["-O3", "-std=c++17", "--generate-code=arch=compute_100a,code=sm_100a",
                  "--expt-relaxed-constexpr", "--expt-extended-lambda",
                  "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
                  "-U__CUDA_NO_HALF2_OPERATORS__", "-Xcompiler", "-fPIC"]
    objs, jobs = [], []
    for s in srcs:
        src = os.path.join(ref, s)
        obj = os.path.join(OUT, os.path.basename(s) + ".o")
        objs.append(obj)
        if s.endswith(".cu"):
            cmd = [os.path.join(cuda_home, "bin", "nvcc"), "-c", src, "-o", obj] + nvcc_flags + defs + inc_flags
        else:
            cmd = ["g++", "-c", src, "-o", obj, "-O3", "-std=c++17", "-fPIC"] + defs + inc_flags
        jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=max(1, args.j)) as ex:
        results = list(ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs))
    for cmd, r in zip(jobs, results):
        if r.returncode != 0:
            print(" ".join(cmd), file=sys.stderr)
            print(r.stdout[-4000:], r.stderr[-4000:], file=sys.stderr)
            return 1
    lib_dirs = ce.library_paths("cuda") + [os.path.join(cuda_home, "lib64", "stubs")]
    link = ["g++", "-shared", "-o", target] + objs + [f"-L{d}" for d in lib_dirs] + [
        "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
        "-lcudart", "-lcuda"]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        print(" ".join(link), file=sys.stderr)
        print(r.stdout[-4000:], r.stderr[-4000:], file=sys.stderr)
        return 1
    for o in objs:
        os.remove(o)
    _copy_to_baseline(target)
    print(f"built {target}")
    return 0


def _stage_tests(ref: str) -> None:
    """Copy the reference's own test files, unchanged, into oracle/_ref/tests/."""
    dst_dir = os.path.join(OUT, "tests")
    os.makedirs(dst_dir, exist_ok=True)
    for rel in REF_TESTS:
        src = os.path.join(ref, rel)
        if os.path.exists(src):
            shutil.copyfile(src, os.path.join(dst_dir, os.path.basename(rel)))


def _copy_to_baseline(target: str) -> None:
    os.makedirs(BASELINE_OUT, exist_ok=True)
    dst = os.path.join(BASELINE_OUT, os.path.basename(target))
    if not os.path.exists(dst) or os.path.getmtime(dst) < os.path.getmtime(target):
        shutil.copyfile(target, dst)


if __name__ == "__main__":
    sys.exit(main())
