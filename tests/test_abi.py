"""The C-ABI library loads on a machine without a GPU and exports every
function include/*.h declares (no compute calls here)."""
import ctypes
import os
import re

from conftest import ROOT


def _declared():
    names = set()
    for h in ("dz_host.h", "dz_cuda.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(dz_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol(dz):
    from dranzer_b200 import _native
    L = ctypes.CDLL(_native.LIB_PATH)
    declared = _declared()
    assert len(declared) >= 40
    missing = [n for n in sorted(declared) if not hasattr(L, n)]
    assert not missing, missing
    # the Python binding types every declared function
    assert declared <= set(_native.SIGNATURES), sorted(declared - set(_native.SIGNATURES))


def test_available_is_safe_without_a_device(dz):
    assert dz.available() in (True, False)


def test_errors_are_reported_not_raised_across_the_abi(dz):
    from dranzer_b200 import _native
    L = _native.lib()
    h = ctypes.c_void_p()
    assert L.dz_cuda_cache_create(None, 1, 1, ctypes.byref(h)) == -1
    st, msg = _native.last_error()
    assert st == -1 and msg
