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


def test_search_entry_points_reject_bad_arguments_without_gpu():
    """sb_cosine_topk, its two phases and sb_topk_merge check their arguments
    before touching the device: rejected calls (and empty query batches) return
    without a CUDA call, so this runs without a GPU."""
    lib = _lib.load()
    p = ctypes.c_void_p(16)  # never dereferenced: every call below returns before launching

    def topk(nq=4, k=8, dim=384, dim_pad=384, cap=64, n_rows=1000, shadow=_lib.SB_DTYPE_F16, status=p):
        return lib.sb_cosine_topk(p, dim, p, dim_pad, shadow, None, n_rows, dim, dim_pad, p, p, dim, nq, k, 0.5, 0,
                                  p, p, cap, p, 1 << 20, status, None)

    def screen(nq=4, k=8, dim=384, dim_pad=384, cap=64, n_rows=1000, shadow=_lib.SB_DTYPE_F16, status=p):
        return lib.sb_cosine_screen(p, dim_pad, shadow, None, n_rows, dim, dim_pad, p, p, dim, nq, k, 0.5, cap, p,
                                    1 << 20, status, None)

    def rescore(nq=4, k=8, dim=384, dim_pad=384, cap=64, n_rows=1000, ids=p, scores=p, status=p):
        return lib.sb_cosine_rescore(p, dim, n_rows, dim, dim_pad, nq, k, 0.5, 0, ids, scores, cap, p, 1 << 20,
                                     status, None)

    inv, uns, big = _lib.SB_ERR_INVALID_ARGUMENT, _lib.SB_ERR_UNSUPPORTED, _lib.SB_ERR_TOO_LARGE
    for fn in (topk, screen, rescore):
        assert fn(k=0) == inv and fn(k=33) == inv
        assert fn(cap=4) == inv and fn(cap=16385) == inv  # capacity below k, above the maximum
        assert fn(dim_pad=400) == uns and fn(dim_pad=576) == uns  # not a multiple of 64, above 512
        assert fn(n_rows=1 << 31) == big
        assert fn(status=None) == inv
        assert fn(nq=0) == _lib.SB_OK  # nothing to do
    assert topk(shadow=_lib.SB_DTYPE_F32) == uns and screen(shadow=_lib.SB_DTYPE_F32) == uns
    assert rescore(ids=None) == inv  # one output without the other
    assert lib.sb_topk_merge(p, 32, p, 32, 17, 4, 8, p, p, None) == inv  # more than 16 lists
    assert lib.sb_topk_merge(p, 31, p, 32, 2, 4, 8, p, p, None) == inv  # list stride below Q * k
