"""Builds libmkv.so (the C-ABI CUDA library) in place, for sm_100a only.

    python -m <package>.build          (or: python mini-kvllm_b200/build.py)

nvcc compiles every csrc/*.cu with `-gencode arch=compute_100a,code=sm_100a` and links
them into a position-independent shared library next to this file. The CUDA runtime
is linked statically, so the library loads on machines without a GPU (for symbol
checks) and needs only the driver at run time.

A hash of every source, header and of the compiler flags is compiled into the library
(`mkv_source_hash()`) and written beside it (libmkv.so.srchash). The build is skipped
only when that recorded hash equals the hash of the sources as they are now, so a
library compiled before the last edit is always rebuilt, whatever the file times say.
"""
from __future__ import annotations

import concurrent.futures
import hashlib
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_NAME = "libmkv.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
HASH_PATH = LIB_PATH + ".srchash"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-cudart", "static",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: install the CUDA toolkit (12.9+) to build libmkv")
    return cand


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _inputs() -> list[str]:
    files = _sources()
    files += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    files += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    files.append(os.path.abspath(__file__))
    return files


def source_hash() -> str:
    """16 hex digits of SHA-256 over the compiler flags and every source and header
    (name and contents, in name order)."""
    h = hashlib.sha256(" ".join(NVCC_FLAGS).encode())
    for f in sorted(_inputs(), key=lambda x: os.path.relpath(x, REPO_DIR)):
        if f == os.path.abspath(__file__):
            continue
        h.update(os.path.relpath(f, REPO_DIR).encode() + b"\0")
        with open(f, "rb") as fh:
            h.update(fh.read())
        h.update(b"\0")
    return h.hexdigest()[:16]


def built_hash() -> str | None:
    """The source hash recorded when libmkv.so was built (None if there is none)."""
    if not (os.path.exists(LIB_PATH) and os.path.exists(HASH_PATH)):
        return None
    with open(HASH_PATH) as f:
        return f.read().strip() or None


def up_to_date() -> bool:
    return built_hash() == source_hash()


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compiles libmkv.so if needed and returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    nvcc = _nvcc()
    digest = source_hash()
    objdir = os.path.join(PKG_DIR, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs, cmds = [], []
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    for src in _sources():
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        cmds.append([nvcc, *NVCC_FLAGS, *extra, f'-DMKV_SOURCE_HASH="{digest}"', "-I", INCLUDE,
                     "-c", src, "-o", obj])
        objs.append(obj)
    # one nvcc per translation unit, run side by side
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        for cmd in cmds:
            if verbose:
                print(" ".join(cmd), flush=True)
        for f in [ex.submit(subprocess.run, cmd, check=True) for cmd in cmds]:
            f.result()
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *NVCC_FLAGS, "-shared", *objs, "-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    with open(HASH_PATH, "w") as f:
        f.write(digest + "\n")
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas-info" in sys.argv)
    print(path)
