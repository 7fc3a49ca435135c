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


def library_for(header):
    mod = load_package()
    return mod.LIB_PATH.parent / ("libllama3x_engine.so" if header.name == "engine_cuda.h" else "libllama3x_cuda.so")


@pytest.mark.parametrize("header", HEADERS, ids=lambda p: p.name)
def test_library_exports_every_declared_symbol(header):
    lib = ctypes.CDLL(str(library_for(header)))
    missing = [n for n in sorted(declared(header)) if not hasattr(lib, n)]
    assert not missing, f"{header.name}: not exported: {missing}"


def test_python_mirror_binds_the_kernel_header():
    mod = load_package()
    mod.load()
    assert set(mod.exported_symbols()) == declared(ROOT / "include" / "kernels_cuda.h")


def test_python_mirror_binds_the_engine_and_device_headers():
    from conftest import load_engine
    eng = load_engine()
    eng.load_library()
    assert set(eng.ENGINE_SIGNATURES) == declared(ROOT / "include" / "engine_cuda.h")
    assert set(eng.DEVICE_SIGNATURES) == declared(ROOT / "include" / "device_cuda.h")
    lib = ctypes.CDLL(str(eng.ENGINE_LIB_PATH))
    assert ctypes.c_int.in_dll(lib, "engine_q8").value == 1


def test_engine_precision_and_layouts():
    from conftest import load_engine
    eng = load_engine()
    lib = eng.load_library()
    assert lib.engine_precision() == b"int8_q8_0"  # the reference's name (src/engine.c:191-195) before any W8A32 load
    # Config and Model keep the reference's x86-64 layout (include/runtime.h:9-17, 86-97): format at byte 28, name at
    # 88, Config 216 bytes, Model.implementation at 216, Model 272 bytes.
    assert eng.Config.format.offset == 28 and eng.Config.name.offset == 88 and ctypes.sizeof(eng.Config) == 216
    assert eng.Model.implementation.offset == 216 and ctypes.sizeof(eng.Model) == 272


def test_c_header_layout_matches(tmp_path):
    """The C header's structs have the same layout as the Python mirror (compiled here with gcc)."""
    src = tmp_path / "layout.c"
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "engine_cuda.h"\n'
                   'int main(void) { printf("%zu %zu %zu %zu\\n", sizeof(Config), offsetof(Config, name), '
                   'offsetof(Model, implementation), sizeof(Model)); return 0; }\n')
    import subprocess
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    assert subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split() == \
        ["216", "88", "216", "272"]


def test_kv_stats_layout():
    """KvStats keeps the reference's x86-64 layout (include/runtime.h:76-85): three size_t, three ints, three size_t."""
    from conftest import load_engine
    eng = load_engine()
    assert eng.KvStats.node.offset == 24 and eng.KvStats.pages_queried.offset == 40 and ctypes.sizeof(eng.KvStats) == 64


def test_attention_work_layout():
    """AttentionWork keeps the reference's x86-64 layout (include/kernels.h:127-132)."""
    mod = load_package()
    W = mod.AttentionWork
    assert [f for f, _ in W._fields_] == ["partial", "max_chunks", "n_heads", "head_dim", "workers", "external",
                                          "capacity"]
    assert W.workers.offset == 20 and W.capacity.offset == 32 and ctypes.sizeof(W) == 40


def test_rope_table_matches_the_oracle():
    """k_rope_table (a host function of the engine library, include/kernels.h:67) equals the oracle's restatement
    of the reference's table (src/kernels_simd.c:194-201, rope_frequency src/kernels.c:49-60) bitwise, with and
    without the Llama 3.1 scaling."""
    import numpy as np
    from conftest import load_engine
    from oracle import oracle as O
    eng = load_engine()
    for rope_type, factor in ((0, 1.0), (1, 8.0)):
        c = eng.Config(head_dim=128, rope_theta=500000.0, rope_type=rope_type, rope_factor=factor, rope_low=1.0,
                       rope_high=4.0, rope_original=8192)
        for pos in (0, 1, 77, 8191):
            got = eng.rope_table(c, pos)
            want = O.rope_table(pos, 128, 500000.0, rope_type, factor, 1.0, 4.0, 8192)
            assert (got.view(np.int32) == want.view(np.int32)).all(), (rope_type, pos)


def test_name_is_null_before_init():
    mod = load_package()
    assert mod.load().kernels_name() is None


def test_pack_s8_vnni_matches_reference_golden():
    """The reference's AMX tile layout, produced on the host by this library (no device): bitwise the reference's
    pack_s8_vnni on a ragged slice with a row stride (tests/golden/q8_golden.npz, vnni_*)."""
    import numpy as np
    from conftest import load_package
    kc = load_package()
    g = np.load(Path(__file__).parent / "golden" / "q8_golden.npz")
    packed = kc.pack_s8_vnni(g["vnni_w"], 37, 200, 256)
    assert packed.shape == g["vnni_packed"].shape and (packed == g["vnni_packed"]).all()

