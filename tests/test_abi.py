"""The C-ABI library loads and exports every symbol the header declares, and the ctypes
struct mirrors match the header field for field (no GPU needed)."""

import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "dsv41_b200.h"


def _declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|void)\s+(dsv41_\w+)\s*\(", text, re.M)))


def _declared_structs():
    text = HEADER.read_text()
    out = {}
    for body, name in re.findall(r"typedef struct \{(.*?)\}\s*(\w+);", text, re.S):
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        fields = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            assert decl.startswith("int64_t"), decl
            fields += [f.strip() for f in decl[len("int64_t"):].split(",")]
        out[name] = fields
    return out


def test_library_exports_every_declared_symbol():
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41.sm100a import build
    build.build()  # a no-op when the library is newer than every source
    lib = ext.lib()
    names = _declared_functions()
    assert names
    for n in names:
        assert hasattr(lib, n), n
    assert lib.dsv41_arch() == 100


def test_struct_mirrors_match_header():
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    decl = _declared_structs()
    assert set(decl) == set(abi.STRUCTS), (set(decl) ^ set(abi.STRUCTS))
    for name, fields in decl.items():
        assert [f for f, _ in abi.STRUCTS[name]._fields_] == fields, name
