"""The C-ABI libraries load and export every entry point include/*.h declares.

Runs without a GPU: loading the libraries and resolving symbols makes no CUDA call.
"""
import ctypes as C
import os
import re

import pytest

from conftest import REPO

PKG = os.path.join(REPO, "opure-voxelengine_b200")
HEADERS = {
    "opure_cuda.h": "libopure_cuda.so",
    "opure_engine.h": "libopure_engine.so",
}


def declared(header):
    text = open(os.path.join(REPO, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(opure_[a-z0-9_]+)\s*\(", text)))


@pytest.mark.parametrize("header", sorted(HEADERS))
def test_library_exports_declared_symbols(header):
    path = os.path.join(REPO, "include", header)
    if not os.path.exists(path):
        pytest.skip(f"{header} not present")
    names = declared(header)
    assert names, header
    lib = C.CDLL(os.path.join(PKG, HEADERS[header]), mode=C.RTLD_GLOBAL)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_strerror_without_device():
    lib = C.CDLL(os.path.join(PKG, "libopure_cuda.so"))
    lib.opure_strerror.restype = C.c_char_p
    assert lib.opure_strerror(0) == b"ok"
    assert b"timed out" in lib.opure_strerror(5)
