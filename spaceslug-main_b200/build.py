"""Build recipe for libspaceslug_b200.so (sm_100a only).

Compiles the CUDA kernels and the C-ABI runtime in csrc/ with nvcc into
lib/libspaceslug_b200.so inside this package directory (in-tree, so the built
library travels with the repository snapshot).  nvcc cross-compiles for
sm_100a without a GPU.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libspaceslug_b200.so"
INCLUDE = PKG.parent / "include"
SOURCES = ["runtime_abi.cu", "q4_gemv.cu", "q4_gemm.cu", "q4_gemm_pair.cu", "q4_decode.cu", "q4_gemv_tile.cu", "q4_gemv_imma.cu", "q4_aux.cu", "noalloc.cu", "upload.cu", "cq4.cu", "lora_train.cu", "sgemm_tc.cu", "lora_tc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def _stale() -> bool:
    if not LIB.is_file():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [INCLUDE / "runtime_abi.h"]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile (if stale) and return the library path."""
    if not force and not _stale():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    base = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
            "-I", str(INCLUDE), "-I", str(CSRC), "--expt-relaxed-constexpr"] + (extra or [])
    if verbose:
        base.append("-Xptxas=-v")
    procs = []
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        objs.append(obj)
        procs.append((src, subprocess.Popen(base + ["-c", str(CSRC / src), "-o", str(obj)],
                                            stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = False
    for src, pr in procs:
        out, _ = pr.communicate()
        if out.strip() and (verbose or pr.returncode):
            sys.stderr.write(f"--- {src}\n{out}")
        failed |= pr.returncode != 0
    if failed:
        raise RuntimeError("nvcc compilation failed")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-lrt", "-ldl",
                    "-lpthread"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
