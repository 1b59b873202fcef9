"""The contest Solution JSONs (python -m gdn_kernel_b200.pack): schema fields
as the reference's packer writes them (ref scripts/pack_solution.py:36-106,
README.md:225-279), a self-contained source list, and an entry module that
builds from those sources alone."""

import importlib.util
import json
import re

import pytest

from gdn_kernel_b200 import pack


@pytest.mark.parametrize("kind", ["decode", "prefill"])
def test_solution_fields(kind, tmp_path):
    pack.main(["--out", str(tmp_path), "--kind", kind])
    sol = json.loads((tmp_path / f"solution_gdn_{kind}.json").read_text())
    assert set(sol) >= {"name", "definition", "author", "spec", "sources"}
    assert sol["definition"] == f"gdn_{kind}_qk4_v8_d128_k_last"   # ref config.toml:6, 19
    spec = sol["spec"]
    assert spec["language"] == "python"
    assert spec["target_hardware"] == ["cuda"]
    assert spec["destination_passing_style"] is True
    assert spec["binding"] == "tvm-ffi"
    assert spec["dependencies"] == []
    entry_file, entry_fn = spec["entry_point"].split("::")
    assert entry_fn == "kernel"
    paths = [s["path"] for s in sol["sources"]]
    assert entry_file in paths and len(paths) == len(set(paths))
    assert all(set(s) == {"path", "content"} and s["content"] for s in sol["sources"])


@pytest.mark.parametrize("kind", ["decode", "prefill"])
def test_solution_sources_are_complete(kind):
    sol = pack.solution(kind)
    files = {s["path"]: s["content"] for s in sol["sources"]}
    for name, text in files.items():
        for inc in re.findall(r'^\s*#\s*include\s+"([^"]+)"', text, re.M):
            assert inc in files, f"{name} includes {inc}, which the solution does not ship"
    entry = files[sol["spec"]["entry_point"].split("::")[0]]
    for listed in re.findall(r"^(?:CUDA|CPP)_FILES = (\[.*\])$", entry, re.M):
        for f in json.loads(listed.replace("'", '"')):
            assert f in files
    assert {"gdn_b200.cu", "gdn_b200.h", pack.TVM_EXPORT[kind]} <= set(files)


def test_unpacked_solution_builds(tmp_path):
    """The prefill solution builds for sm_100a from its own sources (nvcc
    cross-compiles without a GPU) and exposes the TVM-FFI kernel."""
    sol = pack.solution("prefill")
    entry = pack.unpack(sol, str(tmp_path / "sol"))
    spec = importlib.util.spec_from_file_location("gdn_solution_cpu_test", entry)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert callable(mod._kernel())
