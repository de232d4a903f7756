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


def _header_prototypes():
    """name -> (return type, [parameter types]) from include/sfb200.h."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for ret, name, params in re.findall(r"SFB_API\s+([\w\s\*]+?)\s*\b(sfb_\w+)\s*\(([^)]*)\)\s*;", text):
        ps = [p.strip() for p in params.split(",") if p.strip() and p.strip() != "void"]
        out[name] = (ret.strip(), [re.sub(r"\s*\b\w+$", "", p).strip() if not p.endswith("*") else p for p in ps])
    return out


def _ctype_of(c_type):
    t = c_type.replace("const", "").strip()
    if "*" in t or t == "sfb_stream":
        return ctypes.c_void_p
    return {"int": ctypes.c_int, "unsigned": ctypes.c_uint, "int64_t": ctypes.c_int64, "double": ctypes.c_double,
            "const char": ctypes.c_char_p}.get(t)


def test_header_parameter_types_match_the_bindings():
    """Every prototype's parameter list (count and C type) is the ctypes
    signature the Python side binds, so no argument is passed at the wrong width."""
    protos = _header_prototypes()
    assert set(protos) == set(_lib.SIGNATURES)
    for name, (ret, params) in protos.items():
        res, args = _lib.SIGNATURES[name]
        want_res = {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "const char *": ctypes.c_char_p}[ret]
        assert res is want_res, (name, ret, res)
        assert len(params) == len(args), (name, params)
        for i, (p, a) in enumerate(zip(params, args)):
            assert _ctype_of(p) is a, (name, i, p, a)


def test_integration_stub_argtypes_match_the_bindings():
    """The ctypes stub a maintainer copies into the reference
    binds the same argument lists as this package."""
    text = open(os.path.join(REPO, "INTEGRATION.md")).read()
    kinds = {"P": ctypes.c_void_p, "I32": ctypes.c_int, "I64": ctypes.c_int64, "ctypes.c_double": ctypes.c_double}
    found = re.findall(r"_lib\.(sfb_\w+)\.argtypes = \[([^\]]*)\]", text)
    assert {n for n, _ in found} >= {"sfb_elementwise", "sfb_matmul_chain", "sfb_matmul_wide"}
    for name, body in found:
        got = [kinds[t.strip()] for t in body.replace("\n", " ").split(",") if t.strip()]
        assert got == list(_lib.SIGNATURES[name][1]), name


def test_device_side_failures_surface_as_errors():
    """A kernel that gave up on a bounded wait, a chain whose no-saturation
    proof did not hold, and a sign-magnitude word wider than the format each
    leave a count in a reserved slot of sfb_counts; the host turns each into an
    error instead of returning the outputs (no GPU: the counters are host data)."""
    import numpy as np
    from superfloat.python_b200._errors import SFDeviceError
    ok = np.zeros(_lib.N_COUNTS, np.int64)
    ok[:4] = [5, 1, 2, 0]                      # ordinary events are not failures
    _lib.check_counts(ok)
    _lib.check_patterns(ok, 16)
    for slot, what in ((5, "gave up waiting"), (6, "left the range")):
        c = ok.copy()
        c[slot] = 3
        with pytest.raises(SFDeviceError, match=what):
            _lib.check_counts(c)
    c = ok.copy()
    c[7] = 2
    with pytest.raises(ValueError, match="do not fit in 12 bits"):
        _lib.check_patterns(c, 12)
