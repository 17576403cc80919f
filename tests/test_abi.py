"""The C-ABI library: it loads on a CPU-only box and exports every entry point the header declares,
with the ctypes table matching the header. No compute calls (those need a GPU)."""
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "gsdft_b200.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:int64_t|int|size_t|const char\*)\s+(gsdft_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def libpath():
    from gs_dft_b200._lib import LIB_PATH
    if not os.path.exists(LIB_PATH):
        from gs_dft_b200 import _build
        _build.build()
    return LIB_PATH


def test_library_loads_and_exports_every_declared_symbol(libpath):
    from gs_dft_b200._lib import lib
    h = lib.load()
    for name in header_functions():
        assert hasattr(h, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", libpath], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (gsdft_\w+)", out))
    assert set(header_functions()) <= exported


def test_ctypes_table_matches_header():
    from gs_dft_b200._lib import SIGNATURES
    assert sorted(SIGNATURES) == header_functions()


def test_product_path_has_no_cpu_fallback():
    """The host package never imports the oracle: the CUDA library is the only compute path."""
    pkg = os.path.join(ROOT, "gs-dft_b200", "gs_dft_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dirpath, f)).read()
                assert not re.search(r"^\s*(import|from)\s+\S*oracle", src, re.M), f
                assert "gsdft_oracle" not in src, f


def header_arities():
    """{function: parameter count} parsed from the header's prototypes."""
    text = open(HEADER).read()
    out = {}
    for m in re.finditer(r"^(?:int64_t|int|size_t|const char\*)\s+(gsdft_\w+)\s*\(([^;]*?)\);",
                         text, re.M | re.S):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_arity_matches_header():
    from gs_dft_b200._lib import SIGNATURES
    ar = header_arities()
    assert sorted(ar) == header_functions()
    for name, (_, args) in SIGNATURES.items():
        assert len(args) == ar[name], f"{name}: ctypes {len(args)} args, header {ar[name]}"
