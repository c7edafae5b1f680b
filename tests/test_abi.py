"""C-ABI checks that need no GPU: the library loads, exports every entry point
``include/semblend_b200.h`` declares, and the ctypes mirrors of its structs
have the C layout (sizes and field offsets, compiled with gcc from the header)."""

from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from semblend_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_symbols() -> list[str]:
    names = []
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"SB_API\s+[\w\s\*]+?\b(sb_\w+)\s*\(", text)
    return sorted(set(names))


def test_headers_declare_entry_points():
    names = declared_symbols()
    assert "sb_inject" in names and "sb_status_string" in names
    assert len(names) >= 5


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_binding_covers_every_declared_symbol():
    assert set(declared_symbols()) <= set(_lib._SIGNATURES), set(declared_symbols()) - set(_lib._SIGNATURES)


def test_status_strings_without_gpu():
    lib = _lib.load()
    assert lib.sb_status_string(0) == b"ok"
    assert b"workspace" in lib.sb_status_string(-4)
    assert lib.sb_version() >= 100


def _c_layout(tmp_path: Path, structs: dict[str, list[str]]) -> dict[str, int]:
    gcc = shutil.which("gcc") or shutil.which("cc")
    if gcc is None:
        pytest.skip("no C compiler")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "semblend_b200.h"', "int main(void){"]
    for s, fields in structs.items():
        lines.append(f'printf("{s} %zu\\n", sizeof({s}));')
        for f in fields:
            lines.append(f'printf("{s}.{f} %zu\\n", offsetof({s}, {f}));')
    lines.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([gcc, f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return {k: int(v) for k, v in (line.split() for line in out.strip().splitlines())}


def test_struct_layouts_match_header(tmp_path):
    mirrors = {name: cls for name, cls in _lib.__dict__.items() if isinstance(cls, type) and issubclass(cls, ctypes.Structure)}
    c_names = {"SbRows": "sb_rows", "SbInjectDesc": "sb_inject_desc", "SbInjectParams": "sb_inject_params",
               "SbAttnTensor": "sb_attn_tensor"}
    c_names.update({k: v for k, v in getattr(_lib, "C_STRUCT_NAMES", {}).items()})
    structs = {c_names[n]: [f[0] for f in cls._fields_] for n, cls in mirrors.items() if n in c_names}
    layout = _c_layout(tmp_path, structs)
    for n, cls in mirrors.items():
        if n not in c_names:
            continue
        c = c_names[n]
        assert ctypes.sizeof(cls) == layout[c], (c, ctypes.sizeof(cls), layout[c])
        for f in cls._fields_:
            assert getattr(cls, f[0]).offset == layout[f"{c}.{f[0]}"], (c, f[0])


def test_inject_params_flags_field():
    """The params struct's flags word sits where the header puts it (the
    ctypes mirror and the C layout agree) and only known bits are accepted."""
    import ctypes

    from semblend_b200 import _lib

    assert _lib.SbInjectParams.flags.offset == 28 and ctypes.sizeof(_lib.SbInjectParams) == 48
    assert _lib.SB_INJECT_BULK_STAGED == 1
