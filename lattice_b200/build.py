"""Build the native library `lattice_b200/libkcmm.so` (sm_100a).

Kernels are compiled offline with nvcc for `sm_100a`; the host layer is C++17.
The CUDA runtime is linked statically and the driver API is reached through
`cudaGetDriverEntryPoint`, so the library loads on machines without a GPU
driver (the ABI symbol test runs there) and needs only the driver on a GPU
box.  A `libbaseline_llm_os.so` symlink keeps the file name the reference's
ctypes loader searches for.

Usage:  python -m lattice_b200.build [--force]
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libkcmm.so"
ALIAS = PKG / "libbaseline_llm_os.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["kernels/decode.cu", "kernels/decode_noalloc.cu", "kernels/append.cu",
              "kernels/copy.cu", "kernels/prefill.cu", "kernels/tables.cu",
              "kernels/peer.cu"]
CPP_SOURCES = ["pool.cpp", "vmm.cpp", "ffi.cpp", "step_tables.cpp", "policy.cpp"]
HEADERS = ["kcmm_internal.hpp", "launch.hpp", "kernels/ptx.cuh",
           "kernels/tcgen05.cuh", "kernels/pdl.cuh",
           "step_tables.hpp", "policy.hpp"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build")
    return cand


def _cuda_include() -> str:
    return str(Path(_nvcc()).resolve().parent.parent / "include")


def _digest() -> str:
    h = hashlib.sha256()
    for rel in CU_SOURCES + CPP_SOURCES + HEADERS:
        h.update(rel.encode())
        h.update((CSRC / rel).read_bytes())
    h.update((ROOT / "include" / "kcmm.h").read_bytes())
    h.update(" ".join(ARCH).encode())
    return h.hexdigest()


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"command failed: {' '.join(cmd)}")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link libkcmm.so if any source changed; return its path."""
    BUILD.mkdir(exist_ok=True)
    stamp = BUILD / "stamp"
    digest = _digest()
    if not force and LIB.exists() and stamp.exists() and stamp.read_text() == digest:
        return LIB
    nvcc = _nvcc()
    objs: list[str] = []
    for rel in CU_SOURCES:
        obj = BUILD / (Path(rel).stem + ".cu.o")
        cmd = [nvcc, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
               "-c", str(CSRC / rel), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
        objs.append(str(obj))
    for rel in CPP_SOURCES:
        obj = BUILD / (Path(rel).stem + ".cpp.o")
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-Wall", "-fvisibility=default",
              f"-I{_cuda_include()}", "-c", str(CSRC / rel), "-o", str(obj)])
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    _run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs,
          "-Xlinker", "--no-undefined", "-lpthread", "-ldl", "-lrt"])
    os.replace(tmp, LIB)
    if ALIAS.is_symlink() or ALIAS.exists():
        ALIAS.unlink()
    ALIAS.symlink_to(LIB.name)
    stamp.write_text(digest)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
