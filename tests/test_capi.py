"""The C-ABI library loads and exports every symbol include/gdn_b200.h declares;
host-side validation rejects bad arguments before any CUDA call (no GPU needed)."""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from gdn_kernel_b200 import _lib

HEADER = os.path.join(ROOT, "include", "gdn_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(gdn_b200_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("gdn_b200_decode", "gdn_b200_prefill", "gdn_b200_device_status",
              "gdn_b200_last_error", "gdn_b200_abi_version"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_declared()) == set(_lib._SIGNATURES), "ctypes table out of sync with the header"
    assert lib.gdn_b200_abi_version() == 103


def _decode_call(lib, **kw):
    z = ctypes.c_void_p(0)
    args = dict(batch=1, h_qk=16, h_v=32, d=128)
    args.update(kw)
    return lib.gdn_b200_decode(z, z, z, z, z, z, z, z, 0.0, z, z, args["batch"], args["h_qk"],
                               args["h_v"], args["d"], z)


def test_decode_rejects_bad_head_layout():
    lib = _lib.load()
    assert _decode_call(lib, d=64) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert b"head_dim" in lib.gdn_b200_last_error()
    assert _decode_call(lib, h_qk=3, h_v=32) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert b"multiple" in lib.gdn_b200_last_error()
    assert _decode_call(lib, batch=-1) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    # a non-empty batch with null pointers is rejected before touching the GPU
    assert _decode_call(lib, batch=2) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert b"null" in lib.gdn_b200_last_error()
    # an empty batch is a no-op
    assert _decode_call(lib, batch=0) == _lib.GDN_B200_OK
    assert lib.gdn_b200_last_error() == b""


def test_prefill_rejects_bad_arguments():
    lib = _lib.load()
    z = ctypes.c_void_p(0)

    def call(n, t, h_qk=16, h_v=32, d=128):
        return lib.gdn_b200_prefill(z, z, z, z, z, z, z, z, z, 0, 0.0, z, z, n, t, h_qk, h_v, d, z)

    assert call(1, 10, d=256) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert call(-1, 10) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert call(70000, 10) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert call(2, 10) == _lib.GDN_B200_ERR_INVALID_ARGUMENT    # null pointers
    assert call(0, 0) == _lib.GDN_B200_OK                       # nothing to do


def test_python_check_maps_error_codes():
    with pytest.raises(ValueError):
        lib = _lib.load()
        _decode_call(lib, d=64)
        _lib.check(_lib.GDN_B200_ERR_INVALID_ARGUMENT)


def test_tvm_ffi_modules_export_kernel():
    tvm_ffi = pytest.importorskip("tvm_ffi")
    for path in (_lib.TVM_DECODE_PATH, _lib.TVM_PREFILL_PATH):
        assert os.path.exists(path), path
        mod = tvm_ffi.load_module(path)
        assert mod["kernel"] is not None


def test_python_api_rejects_cpu_tensors():
    import torch

    from gdn_kernel_b200 import kernel as K
    q = torch.zeros(1, 1, 16, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        K.gdn_decode(q, q, q, None, None, None, None, None, 0.0, None, None)


def test_decode_pool_rejects_bad_arguments():
    lib = _lib.load()
    z = ctypes.c_void_p(0)

    def call(batch=2, seq_len=3, pool=4, h_qk=16, h_v=32, d=128):
        return lib.gdn_b200_decode_pool(z, z, z, z, z, 0, z, z, 0, z, z, z, z, z, 0.0, z,
                                        batch, seq_len, pool, h_qk, h_v, d, z)

    assert call(d=64) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert call(seq_len=0) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert b"seq_len" in lib.gdn_b200_last_error()
    assert call(pool=0) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert call() == _lib.GDN_B200_ERR_INVALID_ARGUMENT            # null pointers
    assert b"null" in lib.gdn_b200_last_error()
    assert call(batch=0) == _lib.GDN_B200_OK                         # nothing to do


def test_selftest_wait_rejects_bad_limits():
    lib = _lib.load()
    z = ctypes.c_void_p(0)
    assert lib.gdn_b200_selftest_wait_timeout(0, z) == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert lib.gdn_b200_selftest_wait_timeout(5_000_000_000, z) == \
        _lib.GDN_B200_ERR_INVALID_ARGUMENT
