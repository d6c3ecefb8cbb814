"""Builds libbpkv.so (all kernels of this package) for sm_100a with nvcc.

The library is built in-tree under ``unifiedkv_b200/lib/`` so that it ships
with the source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "lib"
LIB = LIBDIR / ("libbpkv_trace.so" if os.environ.get("BPKV_TRACE") == "1" else "libbpkv.so")
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "--extended-lambda",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: cannot build libbpkv.so")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def tree_hash() -> str:
    """SHA-256 (first 16 hex digits) over the names and contents of every source
    the library is built from: csrc/*.cu, csrc/*.cuh, include/*.h."""
    h = hashlib.sha256()
    deps = sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))
    for p in deps:
        h.update(p.name.encode())
        h.update(b"\0")
        h.update(p.read_bytes())
        h.update(b"\0")
    return h.hexdigest()[:16]


def library_hash(lib: Path = LIB) -> str | None:
    """The tree hash the library at ``lib`` was built from (bpkv_build_hash()),
    read in a child process so that this process never maps a library that is
    about to be replaced."""
    if not lib.exists():
        return None
    code = ("import ctypes,sys; L=ctypes.CDLL(sys.argv[1]); f=L.bpkv_build_hash; "
            "f.restype=ctypes.c_char_p; print(f().decode())")
    r = subprocess.run([sys.executable, "-c", code, str(lib)], capture_output=True, text=True)
    return r.stdout.strip() if r.returncode == 0 else None


def _stale() -> bool:
    return library_hash() != tree_hash()


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every ``csrc/*.cu`` into ``lib/libbpkv.so``.  Skipped only when the
    existing library reports the hash of the current sources (bpkv_build_hash)."""
    if not force and not _stale():
        return LIB
    LIBDIR.mkdir(parents=True, exist_ok=True)
    objdir = LIBDIR / ("obj_trace" if os.environ.get("BPKV_TRACE") == "1" else "obj")
    objdir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    stamp = tree_hash()
    objs = []
    procs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), f"-DBPKV_BUILD_HASH=\"{stamp}\"", "-c", str(src),
               "-o", str(obj)]
        if os.environ.get("BPKV_TRACE") == "1":  # debug instrumentation build (separate library)
            cmd += ["-DBPKV_TRACE"]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = []
    for src, pr in procs:
        out, _ = pr.communicate()
        if pr.returncode != 0:
            failed.append((src, out))
        elif out and (verbose or ptxas_verbose):
            print(out)
    if failed:
        msg = "\n".join(f"--- {s.name}\n{o}" for s, o in failed)
        raise RuntimeError(f"nvcc failed:\n{msg}")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_verbose="--ptxas" in sys.argv)
    print(LIB)
