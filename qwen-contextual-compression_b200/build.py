"""Build the in-tree C-ABI library ``libqcc_b200.so`` for sm_100a.

Compiles every ``csrc/*.cu`` with nvcc into one shared library next to this
file (the CUDA runtime is linked statically, so the library only needs the
driver).  Rebuilds only when a source or header is newer than the library.

    python qwen-contextual-compression_b200/build.py [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_ROOT / "include"
LIBRARY = PACKAGE_DIR / "libqcc_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-Xcompiler",
              "-O3", "-Xcompiler", "-fvisibility=hidden"]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the qcc_b200 CUDA library cannot be built")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _inputs() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(path.stat().st_mtime <= built for path in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile the library if needed and return its path."""
    if not force and up_to_date():
        return LIBRARY
    nvcc = nvcc_path()
    build_dir = PACKAGE_DIR / "_build"
    build_dir.mkdir(exist_ok=True)
    objects = []
    for src in sources():
        obj = build_dir / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{result.stdout}\n{result.stderr}")
        if ptxas_verbose or verbose:
            sys.stdout.write(result.stdout + result.stderr)
        objects.append(str(obj))
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *objects]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills / shared memory")
    args = parser.parse_args()
    print(build(args.force, args.verbose, args.ptxas_verbose))


if __name__ == "__main__":
    main()
