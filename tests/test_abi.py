"""The C ABI library loads and exports every symbol include/b200.h declares (CPU only: no compute calls)."""

import ctypes
import os
import re

import pytest

from conftest import ROOT, load_package


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            text = open(os.path.join(inc, f)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def pkg():
    m = load_package()
    if not os.path.exists(m.LIB_PATH):
        m.build()
    return m


def test_library_exports_every_declared_symbol(pkg):
    L = ctypes.CDLL(pkg.LIB_PATH)
    declared = declared_symbols()
    assert declared, "no declarations found"
    missing = [n for n in sorted(declared) if not hasattr(L, n)]
    assert not missing, f"not exported: {missing}"
    assert declared == set(pkg.EXPORTS), "the Python binding's EXPORTS list differs from the header"


def test_weight_nbytes_matches_ggml_row_sizes(pkg):
    L = pkg.lib()
    assert L.b200_weight_nbytes(pkg.Q8_0, 1024, 3072, 1) == 3072 * 1024 // 32 * 34
    assert L.b200_weight_nbytes(pkg.Q4_K, 2048, 6144, 1) == 6144 * 8 * 144
    assert L.b200_weight_nbytes(pkg.Q6_K, 6144, 2048, 1) == 2048 * 24 * 210
    assert L.b200_weight_nbytes(pkg.BF16, 100, 3, 2) == 1200
    assert L.b200_weight_nbytes(pkg.Q8_0, 1000, 3, 1) == 0  # not whole blocks
    assert L.b200_weight_nbytes(pkg.Q4_K, 128, 3, 1) == 0


def test_context_errors_without_a_device(pkg):
    L = pkg.lib()
    if L.b200_device_count() > 0:
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    assert L.b200_context_create(0, ctypes.byref(h)) == pkg.ERR_INVALID
    assert not h.value
    assert b"no such device" in L.b200_last_error(None)
    with pytest.raises(pkg.B200Error):
        pkg.Context(0)


def test_null_arguments_are_rejected_without_a_device(pkg):
    L = pkg.lib()
    assert L.b200_synchronize(None) == pkg.ERR_INVALID
    w = pkg.Weight()
    assert L.b200_weight_alloc(None, pkg.Q8_0, 32, 1, 1, ctypes.byref(w)) == pkg.ERR_INVALID
    assert L.b200_mul_mat(None, ctypes.byref(w), None, 1, None) == pkg.ERR_INVALID
