"""Build libdraco_gguf.so in-tree with nvcc for sm_100a.

Usage:  python -m dracort_b200.build [--force]

The library lands in ``dracort_b200/_lib/libdraco_gguf.so`` next to the
sources, so it travels with the repository snapshot (no JIT cache).  A rebuild
is skipped only when the library was built from exactly the current sources,
headers and flags: their SHA-256 is recorded beside the library
(``_lib/build.stamp``) and compared, so a library left over from other
sources (file times are not trusted) is always rebuilt.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libdraco_gguf.so"
STAMP_PATH = LIB_DIR / "build.stamp"
INCLUDE = REPO_DIR / "include"

SOURCES = ["capi.cu", "dequant.cu", "gemv.cu", "gemv_tc.cu", "gemm.cu", "act.cu", "tp.cu", "attn.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libdraco_gguf.so")
    return cand


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES]
    files += sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    return files


def source_hash() -> str:
    """SHA-256 over the compiler flags and every source and header (name and bytes)."""
    h = hashlib.sha256()
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS + SOURCES).encode())
    for f in _inputs():
        h.update(f.name.encode() + b"\0")
        h.update(f.read_bytes())
    return h.hexdigest()


def needs_build() -> bool:
    if not LIB_PATH.exists() or not STAMP_PATH.exists():
        return True
    return STAMP_PATH.read_text().strip() != source_hash()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu into object files (in parallel) and link the .so."""
    if not force and not needs_build():
        return LIB_PATH
    digest = source_hash()
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    procs = []
    objs = []
    for src in SOURCES:
        obj = obj_dir / (Path(src).stem + ".o")
        objs.append(obj)
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    errors = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            errors.append(f"--- {src} ---\n{out.decode(errors='replace')}")
        elif verbose and out:
            print(out.decode(errors="replace"))
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + r.stdout.decode(errors="replace"))
    os.replace(tmp, LIB_PATH)
    STAMP_PATH.write_text(digest + "\n")
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    path = build(force=a.force, verbose=a.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
