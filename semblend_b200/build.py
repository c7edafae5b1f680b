"""Build the semblend_b200 native library for sm_100a (B200).

Compiles every ``csrc/*.cu`` with nvcc into ``semblend_b200/_native/
libsemblend_b200.so`` (in-tree, so it travels with the source tree).  The
library links the CUDA runtime statically and exports only the ``sb_*`` C ABI
declared in ``include/semblend_b200.h``; it has no dependency on torch.

Usage: ``python -m semblend_b200.build [--force] [-v]``.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_native"
LIB = OUT_DIR / "libsemblend_b200.so"
OBJ_DIR = ROOT / "_build" / "obj"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{ROOT / 'include'}",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the semblend_b200 native library needs CUDA >= 12.8")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers_digest() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*.cuh")) + [ROOT / "include" / "semblend_b200.h"]):
        h.update(p.read_bytes())
    return h.hexdigest()[:16]


def _compile(nvcc: str, src: Path, digest: str, force: bool, verbose: bool) -> Path:
    key = hashlib.sha256(src.read_bytes() + digest.encode() + " ".join(NVCC_FLAGS).encode())
    obj = OBJ_DIR / f"{src.stem}-{key.hexdigest()[:16]}.o"
    if obj.exists() and not force:
        return obj
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile all CUDA sources and link the shared library; returns its path."""
    nvcc = _nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    digest = _headers_digest()
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, digest, force, verbose), srcs))
    stamp = hashlib.sha256("".join(o.name for o in objs).encode()).hexdigest()[:16]
    stamp_file = OUT_DIR / ".stamp"
    if LIB.exists() and not force and stamp_file.exists() and stamp_file.read_text() == stamp:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    # The driver API (TMA tensor-map encoding) is reached through
    # cudaGetDriverEntryPoint, so the library does not link libcuda directly.
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    stamp_file.write_text(stamp)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
