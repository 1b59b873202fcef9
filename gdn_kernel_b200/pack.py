"""Pack the GDN kernels into contest Solution JSONs (flashinfer-bench format).

The reference packs its `kernel` entry points with `scripts/pack_solution.py`
(ref scripts/pack_solution.py:36-106, configured by ref config.toml:1-25) into
a Solution JSON: name, definition, author, a build ``spec`` and the ``sources``
(schema in ref README.md:225-279).  The contest's CUDA builders take no custom
compile flags (ref FAQ.md:59-61), and these kernels need ``sm_100a``
(tcgen05, TMA), so this packer emits a *Python* solution whose entry module
compiles the shipped CUDA sources for sm_100a itself with ``tvm_ffi.cpp.load``
on first use and forwards every call to the TVM-FFI ``kernel`` export - the
workaround the contest FAQ names.

    python -m gdn_kernel_b200.pack [--out DIR] [--kind decode|prefill|both]
                                   [--layout qk4_v8|qk16_v32] [--author NAME]

writes ``solution_gdn_<kind>.json`` files.  Each lists, as {"path", "content"}
entries, the entry module ``gdn_solution.py`` and every source and header the
build reads, flat in one directory.  ``unpack(solution, dest)`` writes the
sources back out (what a harness does before importing the entry point).
"""

from __future__ import annotations

import argparse
import json
import os
import re
from typing import Dict, List

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")

ENTRY = "gdn_solution.py"
ENTRY_POINT = f"{ENTRY}::kernel"

# Definitions of the contest track (ref config.toml:6, 19); heads are runtime
# values in these kernels, so any layout name of the family can be packed.
DEFINITIONS = {
    "decode": "gdn_decode_{layout}_d128_k_last",
    "prefill": "gdn_prefill_{layout}_d128_k_last",
}
TVM_EXPORT = {"decode": "tvm_ffi_decode.cc", "prefill": "tvm_ffi_prefill.cc"}
CUDA_SOURCE = "gdn_b200.cu"
NVCC_FLAGS = ["-O3", "-lineinfo", "--expt-relaxed-constexpr"]   # target: sm_100a (entry module)

_ENTRY_TEMPLATE = '''"""Entry point of the packed B200 GDN {kind} solution (language "python").

On first use it compiles this solution's sources (beside this file) for sm_100a
with tvm_ffi.cpp.load - the contest's CUDA builders take no compile flags - and
then forwards each call, in destination-passing style with the reference's
argument order, to the TVM-FFI `kernel` export it built.
"""

import functools
import os

HERE = os.path.dirname(os.path.abspath(__file__))
KIND = {kind!r}
CUDA_FILES = {cuda_files!r}
CPP_FILES = {cpp_files!r}
NVCC_FLAGS = {nvcc_flags!r}


def _cuda_include():
    import shutil

    home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if not home:
        nvcc = shutil.which("nvcc")
        home = os.path.dirname(os.path.dirname(nvcc)) if nvcc else "/usr/local/cuda"
    return os.path.join(home, "include")


@functools.cache
def _kernel():
    import tvm_ffi.cpp

    build_dir = os.environ.get("GDN_SOLUTION_BUILD_DIR") or os.path.join(HERE, "_build_" + KIND)
    os.makedirs(build_dir, exist_ok=True)
    # The kernels use sm_100a-only instructions (tcgen05, TMA): the target is
    # fixed here rather than detected (a detected "10.0" would also build for
    # plain sm_100, which cannot assemble them).
    prev = os.environ.get("TVM_FFI_CUDA_ARCH_LIST")
    os.environ["TVM_FFI_CUDA_ARCH_LIST"] = "10.0a"
    try:
        mod = tvm_ffi.cpp.load(
            "gdn_b200_solution_" + KIND,
            cpp_files=[os.path.join(HERE, f) for f in CPP_FILES],
            cuda_files=[os.path.join(HERE, f) for f in CUDA_FILES],
            extra_cflags=["-O2", "-I" + _cuda_include()],   # the exports include cuda_runtime.h
            extra_cuda_cflags=NVCC_FLAGS,
            extra_include_paths=[HERE],
            extra_ldflags=["-lcudart"],
            build_directory=build_dir,
        )
    finally:
        if prev is None:
            os.environ.pop("TVM_FFI_CUDA_ARCH_LIST", None)
        else:
            os.environ["TVM_FFI_CUDA_ARCH_LIST"] = prev
    return mod["kernel"]


def kernel(*args):
    """The reference's `kernel` ({kind}): all inputs, then the outputs."""
    _kernel()(*args)
'''

_INCLUDE_RE = re.compile(r'^\s*#\s*include\s+"([^"]+)"', re.M)


def _find(name: str) -> str:
    for d in (CSRC, INCLUDE):
        path = os.path.join(d, name)
        if os.path.exists(path):
            return path
    raise FileNotFoundError(f"source {name} not found in {CSRC} or {INCLUDE}")


def _closure(roots: List[str]) -> List[str]:
    """The roots and every file they include with quotes, transitively."""
    seen: List[str] = []
    todo = list(roots)
    while todo:
        name = todo.pop(0)
        if name in seen:
            continue
        seen.append(name)
        with open(_find(name)) as f:
            todo.extend(_INCLUDE_RE.findall(f.read()))
    return seen


def solution(kind: str, layout: str = "qk4_v8", author: str = "gdn-b200") -> Dict:
    """The Solution dict for `kind` in {"decode", "prefill"}."""
    if kind not in DEFINITIONS:
        raise ValueError(f"kind must be one of {sorted(DEFINITIONS)}")
    roots = [CUDA_SOURCE, TVM_EXPORT[kind]]
    files = _closure(roots)
    entry = _ENTRY_TEMPLATE.format(kind=kind, cuda_files=[CUDA_SOURCE],
                                   cpp_files=[TVM_EXPORT[kind]], nvcc_flags=NVCC_FLAGS)
    sources = [{"path": ENTRY, "content": entry}]
    for name in files:
        with open(_find(name)) as f:
            sources.append({"path": name, "content": f.read()})
    return {
        "name": f"gdn-b200-{kind}",
        "definition": DEFINITIONS[kind].format(layout=layout),
        "author": author,
        "description": ("B200 (sm_100a) Gated DeltaNet " + kind + ": tcgen05/TMA kernels "
                        "behind the reference's TVM-FFI kernel signature; the entry module "
                        "compiles the sources for sm_100a on first use."),
        "spec": {
            "language": "python",
            "target_hardware": ["cuda"],
            "entry_point": ENTRY_POINT,
            "dependencies": [],
            "destination_passing_style": True,
            "binding": "tvm-ffi",
        },
        "sources": sources,
    }


def unpack(sol: Dict, dest: str) -> str:
    """Write a Solution's sources into `dest`; returns the entry module's path."""
    os.makedirs(dest, exist_ok=True)
    for src in sol["sources"]:
        path = os.path.join(dest, src["path"])
        if os.path.dirname(src["path"]):
            os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "w") as f:
            f.write(src["content"])
    return os.path.join(dest, sol["spec"]["entry_point"].split("::")[0])


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--out", default=".", help="directory for the solution JSON files")
    ap.add_argument("--kind", choices=["decode", "prefill", "both"], default="both")
    ap.add_argument("--layout", default="qk4_v8",
                    help="head layout of the definition name (qk4_v8: the contest track)")
    ap.add_argument("--author", default="gdn-b200")
    args = ap.parse_args(argv)
    kinds = ["decode", "prefill"] if args.kind == "both" else [args.kind]
    os.makedirs(args.out, exist_ok=True)
    for kind in kinds:
        sol = solution(kind, args.layout, args.author)
        path = os.path.join(args.out, f"solution_gdn_{kind}.json")
        with open(path, "w") as f:
            json.dump(sol, f, indent=2)
        print(f"packed {path}: {sol['definition']}, {len(sol['sources'])} sources")


if __name__ == "__main__":
    main()
