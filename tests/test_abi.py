"""The C-ABI library loads and exports every symbol include/sfb200.h declares
(no GPU needed: only argument checks run, which return before any CUDA call)."""
import ctypes
import os
import re

import pytest

from conftest import REPO
from superfloat.python_b200 import _lib, build

HEADER = os.path.join(REPO, "include", "sfb200.h")


def declared_symbols():
    text = open(HEADER).read()
    return re.findall(r"SFB_API\s+[\w\s\*]+?\b(sfb_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_declares_the_bound_symbols():
    names = declared_symbols()
    assert len(names) == len(set(names)) >= 7
    assert set(names) == set(_lib.SIGNATURES), (set(names) ^ set(_lib.SIGNATURES))


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)


def test_abi_version(lib):
    assert lib.sfb_abi_version() == 1


def test_argument_errors_return_codes_without_a_gpu(lib):
    """Bad widths, ops and sizes come back as SFB_EINVAL with a message."""
    assert lib.sfb_elementwise(0, 3, None, None, None, None, None, 8, 0, None, None) == _lib.SFB_EINVAL
    assert b"width 3" in lib.sfb_last_error()
    assert lib.sfb_elementwise(99, 16, ctypes.c_void_p(16), ctypes.c_void_p(16), None, ctypes.c_void_p(16),
                               None, 8, 0, None, None) == _lib.SFB_EINVAL
    assert b"unknown op" in lib.sfb_last_error()
    assert lib.sfb_elementwise(0, 16, ctypes.c_void_p(16), None, None, ctypes.c_void_p(16), None, 8, 0, None,
                               None) == _lib.SFB_EINVAL
    assert lib.sfb_matmul_chain(16, None, None, None, None, None, 1, 4, 4, 4, 4, 4, 0, 0, 16, None,
                                None) == _lib.SFB_EINVAL
    assert lib.sfb_matmul_wide(16, 7, None, None, None, 0, None, None, 1, 4, 4, 4, 4, 4, 0, 0, 16, 0, 0, 0, None,
                               0, None, None) == _lib.SFB_EINVAL
    assert lib.sfb_matmul_wide(16, 0, None, None, None, 40, None, None, 1, 4, 4, 4, 4, 4, 0, 0, 16, 0, 0, 0,
                               None, 0, None, None) == _lib.SFB_EINVAL
    assert b"shift 40" in lib.sfb_last_error()
    assert lib.sfb_matmul_wide_workspace(16, 0, 1, 8, 8, 8) >= 0
    assert lib.sfb_matmul_wide_workspace(2, 0, 1, 8, 8, 8) < 0
    # empty problems are no-ops
    assert lib.sfb_elementwise(0, 16, None, None, None, None, None, 0, 0, None, None) == _lib.SFB_OK


def test_python_errors_map_codes():
    from superfloat.python_b200._errors import SFDeviceError, SFLaunchError, SFShapeError
    with pytest.raises(SFShapeError):
        _lib.check(_lib.SFB_EINVAL, "x")
    with pytest.raises(SFLaunchError):
        _lib.check(_lib.SFB_ERANGE, "x")
    with pytest.raises(SFDeviceError):
        _lib.check(_lib.SFB_ECUDA, "x")


def test_missing_library_fails_loudly(tmp_path):
    from superfloat.python_b200._errors import SFDeviceError
    saved = _lib._lib
    try:
        _lib._lib = None
        with pytest.raises(SFDeviceError, match="missing"):
            _lib.load(str(tmp_path / "nope.so"))
    finally:
        _lib._lib = saved
