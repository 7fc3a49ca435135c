"""CPU tests of the drop-in boundary: libllama3x_cuda.so loads without a GPU and exports every function that
include/*.h declares, and the Python mirror binds exactly those symbols. No compute call is made here."""
import ctypes
import re
from pathlib import Path

import pytest

from conftest import ROOT, load_package

HEADERS = sorted((ROOT / "include").glob("*.h"))
DECL = re.compile(r"^[A-Za-z_][\w \t\*]*?\b([a-z_][a-z0-9_]*)\s*\(", re.M)


def declared(header):
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    text = "\n".join(l for l in text.splitlines() if not l.lstrip().startswith(("#", "typedef", "}")))
    return {m.group(1) for m in DECL.finditer(text)}


def test_headers_declare_functions():
    names = set().union(*(declared(h) for h in HEADERS))
    assert {"k_quantize", "k_matmul_q8", "k_gemm_q8", "kc_status"} <= names


@pytest.mark.parametrize("header", HEADERS, ids=lambda p: p.name)
def test_library_exports_every_declared_symbol(header):
    mod = load_package()
    lib = ctypes.CDLL(str(mod.LIB_PATH))
    missing = [n for n in sorted(declared(header)) if not hasattr(lib, n)]
    assert not missing, f"{header.name}: not exported: {missing}"


def test_python_mirror_binds_the_kernel_header():
    mod = load_package()
    mod.load()
    assert set(mod.exported_symbols()) == declared(ROOT / "include" / "kernels_cuda.h")


def test_name_is_null_before_init():
    mod = load_package()
    assert mod.load().kernels_name() is None
