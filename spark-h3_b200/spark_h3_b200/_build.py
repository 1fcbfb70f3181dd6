"""Builds the sm_100a shared library in-tree with nvcc (no JIT cache, no torch extension)."""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC_DIR = PKG_DIR.parent / "csrc"
INCLUDE_DIR = PKG_DIR.parent.parent / "include"
LIB_DIR = PKG_DIR / "_lib"
LIB_NAME = "libsparkh3b200.so"
LIB_PATH = LIB_DIR / LIB_NAME

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = Path("/usr/local/cuda/bin/nvcc")
    if default.exists():
        return str(default)
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build spark_h3_b200")


def sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


STAMP_PATH = LIB_DIR / (LIB_NAME + ".sha256")


def source_digest() -> str:
    """SHA-256 over the compiler flags and every source and header the library is built from."""
    h = hashlib.sha256(" ".join(NVCC_FLAGS).encode())
    for path in sources() + sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h")):
        h.update(path.name.encode())
        h.update(path.read_bytes())
    return h.hexdigest()


def stale() -> bool:
    """True when the library is missing or was built from other sources or flags (compared by
    content, so copied trees with fresh modification times are judged correctly)."""
    if not LIB_PATH.exists() or not STAMP_PATH.exists():
        return True
    return STAMP_PATH.read_text().strip() != source_digest()


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile every .cu under csrc/ for sm_100a and link libsparkh3b200.so."""
    if not force and not stale():
        return LIB_PATH
    digest = source_digest()
    nvcc = _nvcc()
    obj_dir = LIB_DIR / "_obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    procs = []
    objs = []
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        objs.append(obj)
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE_DIR), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        if jobs and len([p for _, p in procs if p.poll() is None]) >= jobs:
            procs[-1][1].wait()
    failed = []
    for src, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            failed.append(f"{src.name}:\n{out.decode(errors='replace')}")
        elif verbose and out:
            print(out.decode(errors="replace"))
    if failed:
        raise RuntimeError("nvcc failed\n" + "\n".join(failed))
    tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
    link = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp), *map(str, objs)]
    subprocess.check_call(link)
    os.replace(tmp, LIB_PATH)
    STAMP_PATH.write_text(digest + "\n")
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
