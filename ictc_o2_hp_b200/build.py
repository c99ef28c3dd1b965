"""Builds libictc_o2_b200.so (the C-ABI kernel library) in-tree with nvcc for sm_100a.

Usage: ``python -m ictc_o2_hp_b200.build [--force] [--jobs N]``.  Each ``.cu`` file in
``csrc/`` compiles to an object under ``_build/`` (skipped when up to date), then
the objects link into ``ictc_o2_hp_b200/_lib/libictc_o2_b200.so``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIBDIR = PACKAGE / "_lib"
LIBRARY = LIBDIR / "libictc_o2_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-std=c++20", "-O3", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "-Xptxas", "-v",
]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(home) / "bin" / "nvcc"
    if path.exists():
        return str(path)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    newest = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    return obj.stat().st_mtime < newest


def _compile(src: Path, extra: list[str]) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src),
           "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stderr}\n{proc.stdout}")
    return obj, proc.stderr


def build(force: bool = False, jobs: int | None = None, extra: list[str] | None = None,
          verbose: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link the shared library."""
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    todo = [s for s in sources if force or _stale(BUILD / (s.stem + ".o"), s)]
    logs = []
    if todo:
        with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
            for obj, log in pool.map(lambda s: _compile(s, extra or []), todo):
                logs.append((obj, log))
    objects = [BUILD / (s.stem + ".o") for s in sources]
    if todo or not LIBRARY.exists() or any(
            LIBRARY.stat().st_mtime < o.stat().st_mtime for o in objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objects), "-lcudart"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stderr}")
        os.replace(tmp, LIBRARY)
    if verbose:
        for obj, log in logs:
            print(f"== {obj.name}\n{log}")
    return LIBRARY


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
