"""The C-ABI library loads here (no GPU) and exports what include/*.h declares."""
import ctypes
import glob
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = []
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(chronos_\w+)\s*\(", src, flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from project_chronos_b200 import build, _native
    build.build()
    return _native.load_library()


def test_header_declares_the_binding_exports():
    from project_chronos_b200 import _native
    assert set(_declared_functions()) == set(_native.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    for name in _declared_functions():
        assert hasattr(lib, name), name


def test_struct_layout_matches(lib):
    from project_chronos_b200 import _native
    assert lib.chronos_moe_args_size() == ctypes.sizeof(_native.ChronosMoeArgs)
    assert lib.chronos_moe_abi_version() == _native.ABI_VERSION


def test_workspace_size_is_a_function_of_the_shape(lib):
    from project_chronos_b200 import _native as N
    s = N.ChronosMoeShape(8192, 2048, 64, 6, 1408, 2, N.DTYPE_BF16)
    big = lib.chronos_moe_workspace_size(ctypes.byref(s))
    # x copies + hidden + fp32 accumulator dominate
    assert big >= 8192 * 6 * 2048 * 2 + 8192 * 8 * 1408 * 2 + 8192 * 2048 * 4
    s1 = N.ChronosMoeShape(1, 2048, 64, 6, 1408, 2, N.DTYPE_BF16)
    assert 0 < lib.chronos_moe_workspace_size(ctypes.byref(s1)) < big
    bad = N.ChronosMoeShape(4, 2048, 64, 65, 1408, 2, N.DTYPE_BF16)  # k > E
    assert lib.chronos_moe_workspace_size(ctypes.byref(bad)) == 0
    assert b"top_k" in lib.chronos_moe_last_error()


def test_invalid_args_are_rejected_without_touching_the_device(lib):
    from project_chronos_b200 import _native as N
    args = N.ChronosMoeArgs()
    args.shape = N.ChronosMoeShape(4, 64, 4, 2, 64, 1, N.DTYPE_BF16)
    rc = lib.chronos_moe_forward(ctypes.byref(args), None)
    assert rc == N.CHRONOS_ERR_INVALID_ARG
    assert lib.chronos_moe_last_error()
    args.shape = N.ChronosMoeShape(0, 64, 4, 2, 64, 1, N.DTYPE_BF16)
    assert lib.chronos_moe_forward(ctypes.byref(args), None) == N.CHRONOS_OK
