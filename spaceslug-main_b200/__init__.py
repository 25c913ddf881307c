"""spaceslug_b200 - B200 (sm_100a) int4-dequant GEMM/GEMV with fused LoRA.

Python host side of the native library libspaceslug_b200.so (built from
csrc/ by build.py, C-ABI in include/runtime_abi.h):

  * ``backend``  - ctypes binding in the style of the reference's
                   python/spaceslug/backend.py (BackendSession, BackendError);
  * ``synth``    - seeded synthetic inputs (the reference's LCG generators);
  * ``parity``   - the reference's parity report plus the GEMM error metrics.

The directory name contains a hyphen, so it is imported by path under the
module name ``spaceslug_b200`` (see ``load`` in __graft_entry__.py).
"""
from __future__ import annotations

__all__ = ["backend", "synth", "parity", "build"]
