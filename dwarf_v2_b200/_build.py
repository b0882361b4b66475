"""Builds the engine's C-ABI shared library for sm_100a, in-tree.

``build()`` compiles every ``csrc/*.cu`` with nvcc
(``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``) and links them into
``dwarf_v2_b200/_lib/libdwarf_b200.so``. A rebuild happens only when a source,
a header or the flags changed. nvcc cross-compiles, so this runs without a GPU.
"""

from __future__ import annotations

import concurrent.futures
import hashlib
import os
import shutil
import subprocess
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
SOURCE_DIR = PACKAGE_DIR / "csrc"
INCLUDE_DIR = PACKAGE_DIR.parent / "include"
OUTPUT_DIR = PACKAGE_DIR / "_lib"
LIBRARY_NAME = "libdwarf_b200.so"
LIBRARY_PATH = OUTPUT_DIR / LIBRARY_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.is_file():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _sources() -> list[Path]:
    return sorted(SOURCE_DIR.glob("*.cu"))


def _fingerprint(extra_flags: list[str]) -> str:
    digest = hashlib.sha256()
    digest.update(" ".join(NVCC_FLAGS + extra_flags).encode())
    for path in sorted(
        list(SOURCE_DIR.glob("*.cu"))
        + list(SOURCE_DIR.glob("*.cuh"))
        + list(INCLUDE_DIR.glob("*.h"))
    ):
        digest.update(path.name.encode())
        digest.update(path.read_bytes())
    return digest.hexdigest()


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile (if stale) and return the path of the shared library."""
    extra = list(extra_flags or [])
    OUTPUT_DIR.mkdir(exist_ok=True)
    stamp = OUTPUT_DIR / "build.sha256"
    fingerprint = _fingerprint(extra)
    if (
        not force
        and LIBRARY_PATH.is_file()
        and stamp.is_file()
        and stamp.read_text().strip() == fingerprint
    ):
        return LIBRARY_PATH
    # A snapshot without the toolchain (or without write access) still works
    # when a library built from these exact sources is present.
    nvcc = _nvcc()
    objects_dir = OUTPUT_DIR / "obj"
    objects_dir.mkdir(exist_ok=True)

    def compile_one(source: Path) -> Path:
        obj = objects_dir / (source.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, *extra, "-I", str(INCLUDE_DIR), "-c", str(source), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed on {source.name}:\n{result.stderr}")
        if verbose and result.stderr:
            print(result.stderr)
        return obj

    sources = _sources()
    workers = max(1, min(len(sources), os.cpu_count() or 1))
    with concurrent.futures.ThreadPoolExecutor(workers) as pool:
        objects = list(pool.map(compile_one, sources))
    tmp = OUTPUT_DIR / (LIBRARY_NAME + ".tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects), "-lcuda"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{result.stderr}")
    os.replace(tmp, LIBRARY_PATH)
    stamp.write_text(fingerprint + "\n")
    return LIBRARY_PATH


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
