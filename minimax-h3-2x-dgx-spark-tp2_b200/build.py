"""Build the sm_100a shared library ``h3b/libh3b.so`` from ``csrc/*.cu`` with nvcc (in-tree, no JIT cache).

    python build.py [--force] [--jobs N] [--verbose-ptxas]

Each translation unit is compiled to an object under ``_build/`` in parallel, then linked into one shared library
with the CUDA runtime linked statically (the library exports only the ``h3b_*`` C ABI of ``include/h3b.h``).
Objects are rebuilt when their source, a header or this script's flags change.
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

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "h3b" / "libh3b.so"
BUILD = PKG / "_build"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{REPO / 'include'}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the h3b CUDA library cannot be built")


def _deps_hash(src: Path, extra: list[str]) -> str:
    h = hashlib.sha256()
    h.update(" ".join(ARCH + FLAGS + extra).encode())
    for p in sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.cu")) + [REPO / "include" / "h3b.h", src]:
        h.update(p.read_bytes())
    return h.hexdigest()[:16]


def _compile(src: Path, extra: list[str], force: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    stamp = BUILD / (src.stem + ".hash")
    digest = _deps_hash(src, extra)
    if not force and obj.exists() and stamp.exists() and stamp.read_text() == digest:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if res.stderr.strip():
        sys.stderr.write(res.stderr)
    stamp.write_text(digest)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, force or verbose_ptxas), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not OUT.exists() or OUT.stat().st_mtime < newest:
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, OUT)
    return OUT


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    print(build(args.force, args.jobs, args.verbose_ptxas))


if __name__ == "__main__":
    main()
