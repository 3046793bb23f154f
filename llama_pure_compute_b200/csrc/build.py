"""Builds the sm_100a C-ABI library ``liblpc_b200.so`` in-tree.

Every ``*.cu`` file of this directory is compiled by nvcc for
``-gencode arch=compute_100a,code=sm_100a`` (objects under ``../_build``) and
linked into ``../lib/liblpc_b200.so``.  Rebuilds only what changed (source,
header or flag changes).  No GPU is needed: nvcc cross-compiles.

    python -m llama_pure_compute_b200.csrc.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
REPO = PKG.parent
INCLUDE = REPO / "include"
BUILD_DIR = PKG / "_build"
LIB_DIR = PKG / "lib"
LIB_NAME = "liblpc_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-DLPC_BUILD",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _headers() -> list[Path]:
    return sorted(HERE.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stamp(src: Path, extra: list[str]) -> str:
    h = hashlib.sha256()
    h.update(src.read_bytes())
    for hd in _headers():
        h.update(hd.read_bytes())
    h.update(" ".join(NVCC_FLAGS + extra).encode())
    return h.hexdigest()


def _compile(nvcc: str, src: Path, obj: Path, extra: list[str], verbose: bool) -> None:
    cmd = [nvcc, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-I", str(HERE), "-c", str(src),
           "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr.strip():
        print(res.stderr, flush=True)


def library_path() -> Path:
    return LIB_DIR / LIB_NAME


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    extra = list(extra_flags or [])
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(HERE.glob("*.cu"))
    todo = []
    objs = []
    for src in sources:
        obj = BUILD_DIR / (src.stem + ".o")
        stamp_file = BUILD_DIR / (src.stem + ".stamp")
        stamp = _stamp(src, extra)
        objs.append(obj)
        if force or not obj.exists() or not stamp_file.exists() or stamp_file.read_text() != stamp:
            todo.append((src, obj, stamp_file, stamp))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, extra, verbose) for s, o, _, _ in todo]
            for f in futs:
                f.result()
        for _, _, sf, st in todo:
            sf.write_text(st)
    lib = library_path()
    if todo or not lib.exists() or force:
        tmp = lib.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, lib)
    return lib


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    lib = build(force=args.force or args.ptxas_info, verbose=args.verbose or args.ptxas_info,
                extra_flags=extra)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
