"""Builds the in-tree C-ABI library ``libsbda_b200.so`` for sm_100a with nvcc.

``python -m sbda_b200.build`` (or ``__graft_entry__.build()``) compiles every
``csrc/*.cu`` file to an object in parallel and links them into
``libsbda_b200.so`` next to this file.  The library is loaded with ctypes; it
has no PyTorch dependency (plain pointers, sizes and a cudaStream_t).
"""

from __future__ import annotations

import concurrent.futures
import hashlib
import os
import shutil
import subprocess
import sys

PACKAGE_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(PACKAGE_DIR)
CSRC = os.path.join(PACKAGE_DIR, "csrc")
INCLUDE = os.path.join(REPO_ROOT, "include")
BUILD_DIR = os.path.join(PACKAGE_DIR, "_build")
LIBRARY = os.path.join(PACKAGE_DIR, "libsbda_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def nvcc_path() -> str:
    candidates = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for candidate in candidates:
        if candidate and os.path.exists(candidate):
            return candidate
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, name) for name in os.listdir(CSRC) if name.endswith(".cu"))


def _fingerprint(sources: list[str]) -> str:
    digest = hashlib.sha256()
    digest.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    headers = [os.path.join(INCLUDE, n) for n in sorted(os.listdir(INCLUDE))]
    headers += [os.path.join(CSRC, n) for n in sorted(os.listdir(CSRC)) if n.endswith((".cuh", ".h"))]
    for path in sources + headers:
        with open(path, "rb") as handle:
            digest.update(path.encode())
            digest.update(handle.read())
    return digest.hexdigest()


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compile and link ``libsbda_b200.so``; skip when sources are unchanged."""
    sources = _sources()
    stamp_path = os.path.join(BUILD_DIR, "stamp")
    fingerprint = _fingerprint(sources)
    if not force and os.path.exists(LIBRARY) and os.path.exists(stamp_path):
        with open(stamp_path) as handle:
            if handle.read().strip() == fingerprint:
                return LIBRARY
    os.makedirs(BUILD_DIR, exist_ok=True)
    nvcc = nvcc_path()

    def compile_one(src: str) -> str:
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{result.stdout}\n{result.stderr}")
        if verbose:
            sys.stderr.write(result.stderr)
        return obj

    workers = max(1, min(len(sources), os.cpu_count() or 1))
    with concurrent.futures.ThreadPoolExecutor(workers) as pool:
        objects = list(pool.map(compile_one, sources))
    tmp = LIBRARY + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objects, "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, LIBRARY)
    with open(stamp_path, "w") as handle:
        handle.write(fingerprint)
    return LIBRARY


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv))
