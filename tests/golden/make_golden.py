"""Regenerates the golden fixtures in this directory.

Runs the REFERENCE's own CPU functions (vulkan-runtime/tests/test_q4gemm.cpp:
57-119, compiled from the read-only reference checkout into
oracle/_ref/libq4ref.so by oracle/Makefile) and records their outputs:

  ref_generators.npz  generate_floats / generate_int4 streams for the seeds
                      and ranges the reference test uses (test_q4gemm.cpp:168-176)
                      plus the ranges of the BASELINE configurations;
  ref_q4gemm_256.npz  the reference's own test case (M=N=K=256, same seeds):
                      packed words and cpu_reference output (sha256 of the full
                      arrays plus strided samples);
  cfg_tiny.npz        BASELINE config 1 (X[128x64] ~ N(0,1), W[64x256],
                      scales U[0.01,0.05], seed 0) built with the package's
                      synthetic generator, and cpu_reference's output on it.

Usage (needs the reference checkout, i.e. this container):
    make -C oracle && python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))


def _load_pkg():
    root = ROOT / "spaceslug-main_b200"
    spec = importlib.util.spec_from_file_location("spaceslug_b200", root / "__init__.py",
                                                  submodule_search_locations=[str(root)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["spaceslug_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    from oracle.oracle import Reference, build
    build(with_reference=True)
    _load_pkg()
    from spaceslug_b200 import synth

    ref = Reference()
    gens = {}
    for seed, lo, hi in [(0x12345678, -1.0, 1.0), (0x13579BDF, 0.5, 1.5), (0x9E3779B1, 0.01, 0.05),
                         (0x2545F491, 0.005, 0.02), (0x1B873593, 0.003, 0.01)]:
        gens[f"floats_{seed:08x}_{lo}_{hi}"] = ref.generate_floats(4096, seed, lo, hi)
    for seed in (0x9ABCDEF0, 0, 1, 0xFFFFFFFF):
        gens[f"int4_{seed:08x}"] = ref.generate_int4(4096, seed)
    np.savez_compressed(HERE / "ref_generators.npz", **gens)

    # The reference's own known-answer case (test_q4gemm.cpp:168-176).
    M = N = K = 256
    a = ref.generate_floats(M * K, 0x12345678, -1.0, 1.0).reshape(M, K)
    b = ref.generate_int4(K * N, 0x9ABCDEF0).reshape(K, N)
    s = ref.generate_floats(N * (K // 32), 0x13579BDF, 0.5, 1.5).reshape(N, K // 32)
    packed = ref.pack_q4(b)
    c = ref.cpu_reference(a, b, s)
    np.savez_compressed(HERE / "ref_q4gemm_256.npz",
                        packed_sha256=sha(packed), c_sha256=sha(c),
                        packed_head=packed[:256], c_samples=c.reshape(-1)[::61].copy(),
                        M=M, N=N, K=K)

    # BASELINE config 1 through the package's synthetic inputs.
    inp = synth.make_inputs("tiny")
    c1 = ref.cpu_reference(inp.x, inp.w_kn, inp.scales)
    np.savez_compressed(HERE / "cfg_tiny.npz", x=inp.x, w_kn=inp.w_kn, scales=inp.scales,
                        packed=ref.pack_q4(inp.w_kn), y_ref=c1)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
