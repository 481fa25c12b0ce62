"""Build libvtnk_b200.so in-tree with nvcc for sm_100a.

    python -m rectokens_b200.csrc.build [--force]

Each ``*.cu`` in this folder is compiled to an object under ``_build/`` (in
parallel) and linked into ``rectokens_b200/libvtnk_b200.so``.  The static CUDA
runtime is linked in; the library depends only on the driver at run time.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libvtnk_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h")]
    return obj.stat().st_mtime < max(d.stat().st_mtime for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None,
          out: Path | None = None, build_dir: Path | None = None) -> Path:
    """Compile (stale objects only) and link; ``out`` / ``build_dir`` place a
    tuning build elsewhere."""
    lib = Path(out) if out else LIB
    bdir = Path(build_dir) if build_dir else BUILD
    bdir.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    objs = [bdir / (s.stem + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(o, s)]
    cc = nvcc()

    def compile_one(so):
        s, o = so
        env_extra = os.environ.get("VTNK_NVCC_EXTRA", "").split()
        cmd = [cc, *ARCH, *FLAGS, *(extra or []), *env_extra, "-c", str(s), "-o", str(o)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {s.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, flush=True)
        return o

    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(todo)))) as ex:
        list(ex.map(compile_one, todo))
    if todo or not lib.exists() or force:
        cmd = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(lib)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
