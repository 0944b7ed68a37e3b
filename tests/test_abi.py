"""The C-ABI library loads on a CPU-only machine and exports every function that
include/*.h declares; no compute is called without a GPU."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(pion_v_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def lib():
    from pion_b200 import build
    build.build()
    return ctypes.CDLL(build.LIB)


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    from pion_b200 import _lib
    assert declared_functions() == set(_lib.SIGNATURES)


def test_abi_version_without_gpu():
    from pion_b200 import _lib
    L = _lib.load()
    assert L.pion_v_abi_version() == _lib.ABI_VERSION == 1
    assert L.pion_v_isa() == 100


def test_library_links_no_oracle():
    """The product library must not depend on the CPU oracle."""
    from pion_b200 import build
    data = open(build.LIB, "rb").read()
    assert b"orc_" not in data and b"liboracle" not in data


def test_bad_arguments_are_rejected_without_gpu():
    from pion_b200 import _lib
    L = _lib.load()
    assert L.pion_v_b200_init(0, 0, None) == _lib.EINVAL
    assert L.pion_v_b200_flat_i8_knn(None, None, None, None, 1, 10, None, None, 0) == _lib.EINVAL
    assert L.pion_v_b200_sync(None) == _lib.EINVAL
