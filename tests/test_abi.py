"""The C-ABI library: it loads without a GPU and exports every function include/kh_cuda.h declares;
the Python binding declares the same set; a call without a device fails with a status, not a crash."""
import ctypes
import re
from pathlib import Path

import pytest

from kleinhirn_b200 import backend

HEADER = Path(__file__).resolve().parents[1] / "include" / "kh_cuda.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(kh_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared()
    for must in ("kh_init", "kh_add_tensor", "kh_check", "kh_plan_create", "kh_upload", "kh_run", "kh_read_output",
                 "kh_plan_destroy", "kh_destroy", "kh_last_error", "kh_bulk_create", "kh_run_batch"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(backend.LIB_PATH))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    assert sorted(backend._SIGS) == declared()


def test_init_without_device_returns_a_status():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    lib = backend.load_library()
    h = ctypes.c_void_p()
    devs = (ctypes.c_int * 1)(0)
    st = lib.kh_init(devs, 1, ctypes.byref(h))
    assert st != 0
    assert lib.kh_last_error().decode()


def test_init_refuses_several_devices_in_one_context():
    """A context drives one device: kh_init with two devices is an argument error, not a silent
    drop of the second (a host that uses several devices opens one context per device)."""
    lib = backend.load_library()
    h = ctypes.c_void_p()
    devs = (ctypes.c_int * 2)(0, 1)
    assert lib.kh_init(devs, 2, ctypes.byref(h)) == 1
    assert "one context per device" in lib.kh_last_error().decode()
    assert not h.value
