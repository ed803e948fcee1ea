"""The C-ABI library loads on a machine without a GPU and exports every entry
point include/tessa_sm100.h declares (no compute is called here)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = []
    inc = os.path.join(ROOT, "include")
    for f in sorted(os.listdir(inc)):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            names += re.findall(r"^TESSA_API\s+[\w\s\*]+?\b(tessa_\w+)\(", src, re.M)
    return names


def test_header_declares_entry_points():
    names = _declared()
    assert "tessa_leaf_topk_sq8" in names and "tessa_replay_run_mode" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    from shear_b200 import _capi
    lib = _capi.load()
    for name in _declared():
        assert hasattr(lib, name), name
    # the Python binding declares exactly the header's entry points
    assert sorted(n for n, _, _ in _capi.SIGNATURES) == sorted(_declared())


def test_strerror_and_version_without_device():
    from shear_b200 import _capi
    lib = _capi.load()
    assert lib.tessa_abi_version() == 5
    assert lib.tessa_strerror(-10) == b"subtree partition cannot finish"
    assert lib.tessa_strerror(-11) == b"not now (no free slot, or still running)"
    assert lib.tessa_strerror(0) == b"ok"
    assert lib.tessa_strerror(-4) == b"device wait timed out"
