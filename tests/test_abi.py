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


STRUCTS = {  # C type in include/pion_vector_b200.h -> ctypes mirror in pion_b200._lib
    "pion_b200_index_desc": "IndexDesc",
    "pion_linear_pool": "LinearPool",
    "pion_beam_view_1536": "BeamView1536",
    "pion_b200_hnsw_layout": "HnswLayout",
    "pion_b200_hnsw_quant_layout": "HnswQuantLayout",
    "pion_heap_node": "HeapNode",
    "pion_heap_list": "HeapList",
    "pion_min_heap": "MinHeap",
    "pion_max_heap": "MaxHeap",
    "pion_quant_beam_view_1536": "QuantBeamView1536",
}


def test_struct_layouts_match_the_header(tmp_path):
    """Every struct of the header has the size and field offsets its ctypes mirror has,
    as the host C compiler lays it out."""
    import shutil
    import subprocess

    from pion_b200 import _lib
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "pion_vector_b200.h"',
             "int main(void) {"]
    want = []
    for cname, pyname in STRUCTS.items():
        cls = getattr(_lib, pyname)
        lines.append(f'printf("%zu\\n", sizeof({cname}));')
        want.append(ctypes.sizeof(cls))
        for fname, _ in cls._fields_:
            lines.append(f'printf("%zu\\n", offsetof({cname}, {fname}));')
            want.append(getattr(cls, fname).offset)
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    got = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True,
                                          text=True).stdout.split()]
    assert got == want
