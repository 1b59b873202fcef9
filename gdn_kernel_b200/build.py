"""Build the in-tree shared libraries of the package (sm_100a only).

* ``libgdn_b200.so``           — CUDA kernels + the C ABI of ``include/gdn_b200.h``
* ``libgdn_b200_tvm_decode.so``  — TVM-FFI ``kernel`` export for decode
* ``libgdn_b200_tvm_prefill.so`` — TVM-FFI ``kernel`` export for prefill

Run ``python -m gdn_kernel_b200.build`` from the repository root.  nvcc
cross-compiles without a GPU; the outputs sit next to this file so that they
travel with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
              "--expt-relaxed-constexpr"]

LIB = os.path.join(PKG, "libgdn_b200.so")
TVM_DECODE = os.path.join(PKG, "libgdn_b200_tvm_decode.so")
TVM_PREFILL = os.path.join(PKG, "libgdn_b200_tvm_prefill.so")


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stdout}")
    return res.stdout


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _sources(*names):
    return [os.path.join(CSRC, n) for n in names]


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> list:
    """Compile every shared library of the package; returns their paths."""
    core_deps = _sources("gdn_b200.cu", "gdn_ptx.cuh", "decode_kernel.cuh", "prefill_kernel.cuh",
                         "prefill_split.cuh", "state_affine_kernel.cuh")
    core_deps.append(os.path.join(INCLUDE, "gdn_b200.h"))
    if force or _stale(LIB, core_deps):
        cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", "-o", LIB,
               os.path.join(CSRC, "gdn_b200.cu")]
        if ptxas_verbose:
            cmd.insert(1, "-Xptxas=-v")
        out = _run(cmd, verbose)
        if ptxas_verbose:
            print(out)
    built = [LIB]
    try:
        import tvm_ffi  # noqa: F401
        from tvm_ffi import libinfo
    except ImportError:  # the C ABI library alone is the product; TVM-FFI exports are optional
        return built
    tvm_inc = libinfo.find_include_path()
    dl_inc = libinfo.find_dlpack_include_path()
    tvm_lib = os.path.dirname(libinfo.find_libtvm_ffi())
    for target, src in ((TVM_DECODE, "tvm_ffi_decode.cc"), (TVM_PREFILL, "tvm_ffi_prefill.cc")):
        deps = _sources(src, "tvm_ffi_common.h") + [os.path.join(INCLUDE, "gdn_b200.h"), LIB]
        if force or _stale(target, deps):
            cuda = os.path.dirname(os.path.dirname(_nvcc()))
            cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-I{INCLUDE}", f"-I{tvm_inc}",
                   f"-I{dl_inc}", f"-I{cuda}/include", "-o", target, os.path.join(CSRC, src),
                   f"-L{PKG}", "-lgdn_b200", f"-L{tvm_lib}", "-ltvm_ffi", f"-L{cuda}/lib64",
                   "-lcudart", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{tvm_lib}"]
            _run(cmd, verbose)
        built.append(target)
    return built


if __name__ == "__main__":
    force = "--force" in sys.argv
    for path in build(verbose=True, force=force, ptxas_verbose="--ptxas-v" in sys.argv):
        print("built", path)
