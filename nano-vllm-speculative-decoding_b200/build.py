"""Builds the C-ABI shared library libspecdec_b200.so in-tree (next to the Python package) for sm_100a.

    python nano-vllm-speculative-decoding_b200/build.py [--force]

Every .cu file under csrc/ is compiled with nvcc for `-gencode arch=compute_100a,code=sm_100a` (B200 only)
and linked into one shared object with the CUDA runtime linked statically.  The TMA tensor-map encoder is
reached through cudaGetDriverEntryPoint, so nothing links against libcuda at build time and the build runs
on a machine without a GPU.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
PACKAGE = HERE / "nanovllm_b200"
LIBRARY = PACKAGE / "libspecdec_b200.so"
BUILD_DIR = HERE / "_build"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the B200 library needs the CUDA toolkit to build")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((HERE.parent / "include").glob("*.h"))


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(path.stat().st_mtime <= built for path in sources() + headers() + [Path(__file__)])


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIBRARY
    BUILD_DIR.mkdir(exist_ok=True)
    compiler = nvcc()
    objects = []
    include = ["-I", str(CSRC), "-I", str(HERE.parent / "include")]
    for source in sources():
        obj = BUILD_DIR / (source.stem + ".o")
        cmd = [compiler, *NVCC_FLAGS, *include, "-c", str(source), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [compiler, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
           *objects, "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("-v", "--verbose", action="store_true")
    args = parser.parse_args()
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
