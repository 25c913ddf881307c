"""GPU: the no-allocation decode entry point (spaceslug_q4gemv_lora_noalloc).

Callers that cannot allocate device memory (allocation-free serving loops,
where an allocation can stall or synchronise the device, and plugin hosts that
own all device memory) call this entry point instead of spaceslug_q4gemm_device:
its LoRA scratch lives in a fixed static device array.  This file sorts last so
that a stop-at-first-failure run has executed every other test first; it also
passes on its own in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest

from spaceslug_b200 import parity, synth

pytestmark = pytest.mark.gpu


def _case(torch, dev, m, k, n, rank, seed):
    w_kn, packed, scales = synth.make_weights(k, n, 0.005, 0.02, seed=seed)
    x = synth.make_x(m, k, seed=seed + 1)
    a = synth.normal(k * rank, seed + 2, 0.02).reshape(k, rank)
    b = synth.normal(rank * n, seed + 3, 0.02).reshape(rank, n)
    t = lambda arr: torch.from_numpy(np.ascontiguousarray(arr)).to(dev)  # noqa: E731
    return {"x": t(x), "p": t(packed.view(np.int32)), "s": t(scales), "a": t(a), "b": t(b),
            "m": m, "k": k, "n": n, "rank": rank}


def _run(session, torch, entry, c, alpha):
    y = torch.full((c["m"], c["n"]), float("nan"), dtype=torch.float32, device=c["x"].device)
    stream = torch.cuda.current_stream().cuda_stream
    code = session.raw(entry)(c["x"].data_ptr(), c["p"].data_ptr(), c["s"].data_ptr(), c["a"].data_ptr(),
                              c["b"].data_ptr(), c["rank"], alpha, y.data_ptr(), c["m"], c["n"], c["k"], stream)
    assert code == 0, (entry, code, session.raw("spaceslug_last_error")())
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_noalloc_matches_regular_entry_point_twice(session, cuda):
    import torch
    alpha = 32.0
    cases = [_case(torch, cuda, 4, 4096, 4096, 16, 101), _case(torch, cuda, 8, 2048, 1000, 64, 202)]
    for c in cases:  # two calls in a row, sharing the static scratch
        y_noalloc = _run(session, torch, "spaceslug_q4gemv_lora_noalloc", c, alpha)
        y_regular = _run(session, torch, "spaceslug_q4gemm_device", c, alpha)
        assert np.all(np.isfinite(y_noalloc))
        rep = parity.compare_float_arrays(y_noalloc, y_regular, tolerance=parity.GEMV_REL_TOL)
        assert rep["status"] == "pass", rep


def test_noalloc_rejects_shapes_beyond_its_limits(session, cuda):
    import torch
    c = _case(torch, cuda, 4, 1024, 64, 8, 7)
    f = session.raw("spaceslug_q4gemv_lora_noalloc")
    stream = torch.cuda.current_stream().cuda_stream
    y = torch.empty((9, 64), dtype=torch.float32, device=cuda)
    args = (c["x"].data_ptr(), c["p"].data_ptr(), c["s"].data_ptr(), c["a"].data_ptr(), c["b"].data_ptr())
    assert f(*args, 65, 1.0, y.data_ptr(), 4, 64, 1024, stream) == 1   # rank above the array
    assert f(*args, 8, 1.0, y.data_ptr(), 9, 64, 1024, stream) == 1    # more rows than the array
    assert b"no-allocation" in session.raw("spaceslug_last_error")()
