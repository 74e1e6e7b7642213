# SPDX-License-Identifier: Apache-2.0
"""The C-ABI library loads and exports every symbol include/kotflash_b200.h
declares; host-side argument checks work without a GPU (no kernel launches)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from kotflash_b200 import _ext

HEADER = Path(__file__).resolve().parents[1] / "include" / "kotflash_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(kf_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for n in ("kf_append", "kf_attn_fwd", "kf_attn_bwd", "kf_decode", "kf_merge_partials",
              "kf_last_error", "kf_version"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _ext.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} missing from {_ext.LIB_PATH}"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_ext.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (kf_[a-z0-9_]+)", out))
    assert set(declared_functions()) <= exported
    assert set(_ext.SIGNATURES) == set(declared_functions())


def test_version_and_workspace_queries():
    lib = _ext.load()
    assert lib.kf_version() >= 10000
    assert lib.kf_decode_workspace_bytes(2, 8, 1, 64, 1) == 0
    assert lib.kf_decode_workspace_bytes(2, 8, 1, 64, 4) >= 4 * 16 * 65 * 4
    assert lib.kf_attn_bwd_workspace_bytes(4, 32, 4096, 128) >= 4 * 32 * 4096 * 130 * 4


def _t(shape, ptr=0x1000):
    d = _ext.KFTensor4()
    d.ptr = ptr
    strides = [shape[1] * shape[2] * shape[3], shape[2] * shape[3], shape[3], 1]
    for i in range(4):
        d.size[i] = shape[i]
        d.stride[i] = strides[i]
    return d


def test_argument_errors_are_reported_before_any_launch():
    lib = _ext.load()
    kc, vc = _t((1, 2, 8, 16)), _t((1, 2, 8, 16))
    nk, nv = _t((1, 2, 3, 16)), _t((1, 2, 3, 16))
    rc = lib.kf_append(ctypes.byref(kc), ctypes.byref(vc), ctypes.byref(nk), ctypes.byref(nv), 6, 0, None)
    assert rc == _ext.KF_ERR_INVALID and "capacity" in _ext.last_error()
    rc = lib.kf_append(ctypes.byref(kc), ctypes.byref(vc), ctypes.byref(nk), ctypes.byref(nv), 0, 7, None)
    assert rc == _ext.KF_ERR_INVALID and "dtype" in _ext.last_error()
    q, k = _t((1, 3, 1, 16)), _t((1, 2, 8, 16))
    rc = lib.kf_decode(ctypes.byref(q), ctypes.byref(k), ctypes.byref(k), None, None, 0,
                       ctypes.byref(q), None, 0, 0.25, 0, None, 0, None)
    assert rc == _ext.KF_ERR_INVALID and "divisible" in _ext.last_error()
    q = _t((1, 4, 17, 16))
    o = _t((1, 4, 17, 16))
    rc = lib.kf_decode(ctypes.byref(q), ctypes.byref(k), ctypes.byref(k), None, None, 0,
                       ctypes.byref(o), None, 0, 0.25, 0, None, 0, None)
    assert rc == _ext.KF_ERR_UNSUPPORTED
    q = _t((1, 4, 5, 20))
    k = _t((1, 2, 8, 20))
    rc = lib.kf_attn_fwd(ctypes.byref(q), ctypes.byref(k), ctypes.byref(k), ctypes.byref(q),
                         ctypes.c_void_p(0x2000), 1, 0.2, 1, None, None)
    assert rc == _ext.KF_ERR_UNSUPPORTED and "multiple of 8" in _ext.last_error()
    rc = lib.kf_merge_partials(None, None, 1, 1, 64, None, None, 0, None)
    assert rc == _ext.KF_ERR_INVALID


def test_check_maps_status_codes_to_exceptions():
    lib = _ext.load()
    lib.kf_merge_partials(None, None, 1, 1, 64, None, None, 0, None)
    with pytest.raises(ValueError, match="null"):
        _ext.check(_ext.KF_ERR_INVALID, "kf_merge_partials")
    with pytest.raises(RuntimeError):
        _ext.check(_ext.KF_ERR_CUDA, "x")
