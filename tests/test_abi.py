"""CPU tests of the C-ABI boundary: the library loads, exports every function
include/*.h declares, the ctypes binding covers them, and argument validation
rejects bad calls before any device work (no GPU needed)."""
import ctypes as C
import glob
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))
LIB = os.path.join(ROOT, "ternative_b200", "libtvb200.so")


def declared():
    names = set()
    for h in HEADERS:
        txt = open(h).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        names.update(re.findall(r"\b(tvb_[a-z0-9_]+)\s*\(", txt))
    return names


def test_headers_declare_entry_points():
    assert HEADERS
    assert len(declared()) >= 35


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB), "build libtvb200.so first"
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (tvb_[a-z0-9_]+)", out))
    missing = declared() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_binding_covers_header():
    from ternative_b200 import _lib
    missing = declared() - set(_lib.EXPORTED)
    assert not missing, sorted(missing)


def test_library_loads_and_reports_version():
    from ternative_b200 import load
    lib = load()
    assert lib.tvb_version() >= 1
    assert lib.tvb_status_string(5) == b"device wait timed out"


def test_invalid_arguments_rejected_without_device_work():
    from ternative_b200 import TvbError, _lib
    lib = _lib.load()
    # null pointers / bad K are rejected by host-side validation
    assert lib.tvb_gemv_f16(None, None, None, 256, 16, None) == 1
    assert b"null" in lib.tvb_last_error()
    assert lib.tvb_merge_i2s_lora(C.c_void_p(16), 1.0, 100, 4, None, None, 0, 0.0, 1,
                                  C.c_void_p(16), None, None) == 1
    assert b"multiple of 128" in lib.tvb_last_error()
    assert lib.tvb_merge_i2s_lora(C.c_void_p(16), 1.0, 128, 4, None, None, 0, 0.0, 3,
                                  C.c_void_p(16), None, None) == 4   # per-tensor INT8 in merge
    with pytest.raises(TvbError):
        _lib.call("tvb_attention_decode", None, None, None, 4, None, 4, 1, 128, 1.0, None)
    cfg = _lib.ModelConfig(1000, 256, 2, 2, 1, 64, 512, 64, 5e5, 1e-5, 64)
    out = C.c_void_p()
    assert lib.tvb_context_create(C.byref(cfg), C.byref(out)) == 1   # head_dim 64 not built
    assert b"head_dim" in lib.tvb_last_error()
