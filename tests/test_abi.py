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


def test_python_constants_match_header():
    """Record widths and the inverse-solve size limit used by the host layer equal the header's."""
    from gs_dft_b200 import _lib
    text = open(HEADER).read()
    defs = dict(re.findall(r"^#define\s+(GSDFT_\w+)\s+(\d+)", text, re.M))
    assert int(defs["GSDFT_SIDE_FIELDS"]) == _lib.SIDE_FIELDS
    assert int(defs["GSDFT_SOLVE_INV_MAX"]) == _lib.SOLVE_INV_MAX
    assert int(defs["GSDFT_ABI_VERSION"]) == _lib.ABI_VERSION
    for enum, width in (("GSDFT_REC_FIELDS", _lib.REC_FIELDS), ("GSDFT_VJP_FIELDS", _lib.VJP_FIELDS),
                        ("GSDFT_XC_FIELDS", _lib.XC_FIELDS)):
        body = re.search(r"enum\s*\{([^}]*\b" + enum + r"\b[^}]*)\}", text).group(1)
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        names = [t.strip().split("=")[0].strip() for t in body.split(",") if t.strip()]
        assert names.index(enum) == width, (enum, names)


def test_library_version_matches_package(libpath):
    """The built library implements the ABI version the host layer was written for."""
    from gs_dft_b200._lib import ABI_VERSION, lib
    assert lib.load().gsdft_version() == ABI_VERSION


def test_host_modules_resolve_every_name():
    """Every global name a host module's code loads is bound in that module or in builtins (a
    missing import shows up here, on CPU, rather than on the first GPU call)."""
    import builtins
    import dis
    import importlib
    import pkgutil
    import types
    import gs_dft_b200

    def globals_of(code):
        out = {i.argval for i in dis.get_instructions(code) if i.opname in ("LOAD_GLOBAL", "LOAD_NAME")}
        for c in code.co_consts:
            if isinstance(c, types.CodeType):
                out |= globals_of(c)
        return out

    missing = []
    for info in pkgutil.walk_packages(gs_dft_b200.__path__, "gs_dft_b200."):
        spec = importlib.util.find_spec(info.name)
        if spec is None or not str(spec.origin).endswith(".py"):
            continue
        mod = importlib.import_module(info.name)
        ns = set(vars(mod)) | set(dir(builtins))
        code = compile(open(mod.__file__).read(), mod.__file__, "exec")
        missing += [(info.name, n) for n in sorted(globals_of(code))
                    if n not in ns and not n.startswith("__")]
    assert not missing, missing
