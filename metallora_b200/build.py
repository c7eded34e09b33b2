"""Builds ``metallora_b200/lib/libmetallora_b200.so`` from ``metallora_b200/csrc``.

Each ``.cu`` file is compiled for sm_100a (``-gencode arch=compute_100a,code=sm_100a``)
in parallel, then linked into one shared library that exports the C ABI of
``include/metallora_b200.h``.  Object files go to ``metallora_b200/lib/obj``;
a source is recompiled only when it or a header is newer than its object.

    python -m metallora_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB_DIR = PKG / "lib"
OBJ_DIR = LIB_DIR / "obj"
LIB_PATH = LIB_DIR / "libmetallora_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "-DNDEBUG",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(src: Path, obj: Path, newest_header: float) -> bool:
    if not obj.exists():
        return True
    mt = obj.stat().st_mtime
    return src.stat().st_mtime > mt or newest_header > mt


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(CSRC), "-I", str(INCLUDE), "-c", str(src),
           "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr)


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    newest = max((h.stat().st_mtime for h in headers), default=0.0)
    todo = [(s, OBJ_DIR / (s.stem + ".o")) for s in sources]
    todo = [(s, o) for s, o in todo if force or _stale(s, o, newest)]
    if todo:
        workers = min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(workers) as ex:
            futs = [ex.submit(_compile, s, o, verbose) for s, o in todo]
            for f in futs:
                f.result()
    objs = [OBJ_DIR / (s.stem + ".o") for s in sources]
    if force or todo or not LIB_PATH.exists():
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB_PATH), *map(str, objs), "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    sys.exit(0)
