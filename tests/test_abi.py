"""C-ABI checks that need no GPU: the library loads, exports every symbol the
public header declares, and reports a missing GPU as an error status."""
import ctypes as C
import os
import re

import pytest

import myelith_b200 as myl

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "myl_w8a16.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(myl_[a-z0-9_]+)\s*\(", txt)))


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for s in ("myl_init", "myl_linear_w8a16", "myl_linear_w8a16_pc", "myl_lm_head_w8a16_i32",
              "myl_backend_linear_w8a16", "myl_linear_dev", "myl_linear_acc_dev"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    L = myl.load_library()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, f"not exported: {missing}"


def test_library_is_sm100a_only():
    # The shared object carries sm_100a code only; there is no CPU path in it.
    data = open(myl.LIB_PATH, "rb").read()
    assert b"sm_100a" in data


def test_init_reports_errors_as_status():
    L = myl.load_library()
    h = C.c_void_p()
    rc = L.myl_init(9999, C.byref(h))  # no such device anywhere
    assert rc != 0 and not h.value
    assert L.myl_last_error()


def test_null_arguments_are_rejected():
    L = myl.load_library()
    assert L.myl_linear_w8a16(None, None, None, 1, 0, 0, None) == myl.MYL_ERR_ARG
    assert L.myl_init(0, None) == myl.MYL_ERR_ARG


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(myl.MylError):
        myl._lib_backup = myl._lib
        try:
            myl._lib = None
            myl.load_library(str(tmp_path / "nope.so"))
        finally:
            myl._lib = myl._lib_backup
