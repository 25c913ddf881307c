"""Regenerates cfg_rows.npz: reference outputs on sampled rows of the large
BASELINE configurations (3 prefill 2048x4096x11008, 4 LoRA 512x4096x4096 r=16,
5 70B MLP 4096x8192x28672), for parity checks at full size on the GPU box.

The base product of each sampled row is the REFERENCE's own cpu_reference
(vulkan-runtime/tests/test_q4gemm.cpp:102-119, compiled from the read-only
checkout into oracle/_ref/libq4ref.so by oracle/Makefile), run on the
package's seeded synthetic inputs (spaceslug_b200.synth, the reference's LCG
plus Box-Muller).  Config 4's LoRA term, a shape outside the reference's LoRA
contract, is the oracle's double-precision restatement of
tests/test_lora_delta_api.cpp:14 scaled by alpha/rank (python/spaceslug/lora.py:21-23).

Stored per configuration NAME in {prefill, lora, mlp70b}:
  NAME_rows   int64 [8]        the sampled row indices,
  NAME_y      float32 [8][N]   the reference output of those rows (rounded
                               once from double; 6e-8 relative, far below
                               the GEMM tolerances),
  NAME_xinf   float64          max |x| over the whole X (for the max-abs bound),
  NAME_wabs   float64          8 * max scale, i.e. max |w| (same bound).

Usage (needs the reference checkout, i.e. this container):
    make -C oracle && python tests/golden/make_config_rows.py
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

ROWS = {"prefill": 2048, "lora": 512, "mlp70b": 4096}


def sample_rows(m: int) -> np.ndarray:
    """Eight rows: both ends, the middle, and five spread in between."""
    return np.array(sorted({0, 1, m // 3, m // 2 - 1, m // 2, (2 * m) // 3 + 5, m - 2, m - 1}), np.int64)


def _load_pkg():
    root = ROOT / "spaceslug-main_b200"
    spec = importlib.util.spec_from_file_location("spaceslug_b200", root / "__init__.py",
                                                  submodule_search_locations=[str(root)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["spaceslug_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    from oracle.oracle import Oracle, Reference, build
    build(with_reference=True)
    _load_pkg()
    from spaceslug_b200 import synth

    ref, orc = Reference(), Oracle()
    out = {}
    for name in ROWS:
        cfg = synth.CONFIGS[name]
        inp = synth.make_inputs(cfg)
        rows = sample_rows(cfg.m)
        assert rows.size == 8
        y = ref.cpu_reference(np.ascontiguousarray(inp.x[rows]), inp.w_kn, inp.scales)
        if cfg.rank:
            orc.lora_add(y, np.ascontiguousarray(inp.x[rows]), inp.lora_a, inp.lora_b, cfg.alpha)
        out[f"{name}_rows"] = rows
        out[f"{name}_y"] = y.astype(np.float32)
        out[f"{name}_xinf"] = np.float64(np.max(np.abs(inp.x)))
        out[f"{name}_wabs"] = np.float64(8.0 * np.max(np.abs(inp.scales)))
        print(name, rows.tolist(), float(np.abs(y).max()), flush=True)
    np.savez_compressed(HERE / "cfg_rows.npz", **out)
    print("cfg_rows.npz", (HERE / "cfg_rows.npz").stat().st_size)


if __name__ == "__main__":
    main()
