"""Build recipe for libmusemoe.so: nvcc for sm_100a, one object per .cu, linked in-tree.

    python muse-moe-w4a16_b200/build.py [--force] [--verbose]

The library lands next to this file (the package directory), so it travels with the
repository snapshot and is what `_lib.load_library()` opens. Objects go to `_build/`.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = REPO / "_build"
LIB_NAME = "libmusemoe.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-I", str(REPO / "include"), "-I", str(CSRC)]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libmusemoe.so")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((REPO / "include").glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None,
          out: Path | None = None, build_dir: Path | None = None) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libmusemoe.so (or `out`); returns its path.
    A variant build (extra defines) keeps its objects in its own `build_dir`."""
    nvcc = nvcc_path()
    bdir = Path(build_dir) if build_dir else BUILD_DIR
    bdir.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    flags = NVCC_FLAGS + ARCH + (extra_flags or [])
    jobs = []
    for src in _sources():
        obj = bdir / (src.stem + ".o")
        if force or _stale(obj, [src, *headers, Path(__file__)]):
            jobs.append([nvcc, *flags, "-c", str(src), "-o", str(obj)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)

    with cf.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        list(ex.map(run, jobs))
    objs = [bdir / (s.stem + ".o") for s in _sources()]
    lib = Path(out) if out else PKG_DIR / LIB_NAME
    if force or jobs or _stale(lib, objs):
        run([nvcc, *ARCH, "-shared", "-o", str(lib), *map(str, objs)])
    return lib


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage (-Xptxas -v)")
    ap.add_argument("--trace", action="store_true",
                    help="variant with per-role clock stamps (-DMUSE_TRACE); needs --out")
    ap.add_argument("--out", default=None, help="library path of a variant build")
    a = ap.parse_args(argv)
    flags = (["-Xptxas", "-v"] if a.ptxas_v else []) + (["-DMUSE_TRACE"] if a.trace else [])
    if a.trace and not a.out:
        ap.error("--trace builds a variant library: give --out")
    lib = build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra_flags=flags or None,
                out=a.out, build_dir=(BUILD_DIR / "trace") if a.trace else None)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
