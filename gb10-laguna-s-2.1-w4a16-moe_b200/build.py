"""Build recipe for the sm_100a shared library ``lib/libw4a16moe_b200.so``.

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` only and links one
position-independent shared object that exports the C ABI declared in
``include/w4a16_moe_b200.h``.  Incremental: a source newer than the library
(or a changed flag set) triggers a rebuild.

Usage: ``python build.py [--force] [--jobs N]``.
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

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PKG_DIR / "_build"
LIB_DIR = PKG_DIR / "lib"
LIB_NAME = "libw4a16moe_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-DW4A16_BUILD",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    for p in ("/usr/local/cuda/bin/nvcc",):
        if os.path.exists(p):
            return p
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _flags_digest(extra: list[str]) -> str:
    return hashlib.sha1(" ".join(ARCH_FLAGS + NVCC_FLAGS + extra).encode()).hexdigest()[:12]


def lib_path() -> Path:
    return LIB_DIR / LIB_NAME


def _needs_build(sources: list[Path], headers: list[Path], out: Path, stamp: Path, digest: str) -> bool:
    if not out.exists() or not stamp.exists() or stamp.read_text().strip() != digest:
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources + headers)


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, diagnostics: bool = False) -> Path:
    """Compile the library.  ``diagnostics`` adds -DW4A16_DIAGNOSTICS: the
    forward then honours the W4A16_*_TRACE / W4A16_DECODE_* environment hooks
    (pipeline timestamps, kernel selection overrides) -- for profiling builds,
    never for production."""
    nvcc = nvcc_path()
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    out = lib_path()
    stamp = BUILD_DIR / "flags.sha1"
    extra = ["-DW4A16_DIAGNOSTICS"] if diagnostics else []
    digest = _flags_digest(extra)
    if not force and not _needs_build(sources, headers, out, stamp, digest):
        return out
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        if verbose and res.stderr:
            print(res.stderr, file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources))
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out)
    stamp.write_text(digest)
    return out


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill info")
    ap.add_argument("--diagnostics", action="store_true", help="enable the environment trace / override hooks")
    args = ap.parse_args(argv)
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose, diagnostics=args.diagnostics))
    return 0


if __name__ == "__main__":
    sys.exit(main())
