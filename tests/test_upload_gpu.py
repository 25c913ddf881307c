"""GPU: the model-load path (pinned staged upload, device-side packing from the
logical int4 matrix) round-trips losslessly to the reference layout."""
from __future__ import annotations

import numpy as np
import pytest

from spaceslug_b200 import synth

pytestmark = pytest.mark.gpu


def _logical(k: int, n: int, seed: int) -> np.ndarray:
    return synth.lcg_int4(k * n, seed).reshape(k, n)


@pytest.mark.parametrize("k,n,c0,c1", [(32, 1, 0, 1), (256, 1000, 0, 1000), (96, 37, 5, 30), (4096, 520, 7, 519)])
def test_logical_upload_packs_like_the_reference(session, oracle, cuda, k, n, c0, c1):
    b = _logical(k, n, k + 3 * n)
    scales = synth.lcg_floats(n * (k // 32), 11, 0.005, 0.02).reshape(n, k // 32)
    with session.weights_logical(b, scales, k, n, c0, c1) as h:
        pk, sc = h.export()
    ref = oracle.pack(b).reshape(n, k // 8)
    assert np.array_equal(pk, ref[c0:c1])
    assert np.array_equal(sc, scales[c0:c1])


def test_logical_upload_spanning_several_staging_slots(session, oracle, cuda):
    # 8192 x 8000 int8 = 62.5 MB of logical weights: several 32 MiB row blocks
    k, n, c0, c1 = 8192, 8064, 64, 8064
    rng = np.random.default_rng(1)
    b = rng.integers(-8, 8, size=(k, n), dtype=np.int8)
    scales = rng.uniform(0.005, 0.02, size=(n, k // 32)).astype(np.float32)
    with session.weights_logical(b, scales, k, n, c0, c1) as h:
        pk, _ = h.export()
    assert np.array_equal(pk, session.q4_pack(b[:, c0:c1]).reshape(c1 - c0, k // 8))


def test_logical_upload_keeps_low_nibble_of_out_of_range_values(session, oracle, cuda):
    b = np.array(np.arange(-64, 64).reshape(32, 4), dtype=np.int8)
    scales = np.ones((4, 1), np.float32)
    with session.weights_logical(b, scales, 32, 4) as h:
        pk, _ = h.export()
    assert np.array_equal(pk.reshape(-1), oracle.pack(b))


@pytest.mark.parametrize("pinned", [False, True])
def test_staged_upload_round_trip(session, cuda, pinned):
    # 4096 x 4096: 8 MB of packed words (staged above 1 MB from pageable memory)
    import torch
    k, n = 4096, 4096
    rng = np.random.default_rng(2)
    packed = rng.integers(0, 2**32, size=n * k // 8, dtype=np.uint32)
    scales = rng.uniform(0.005, 0.02, size=(n, k // 32)).astype(np.float32)
    if pinned:
        tp = torch.from_numpy(packed.view(np.int32)).pin_memory()
        packed = tp.numpy().view(np.uint32)
    with session.weights(packed, scales, k, n, 1000, 3000) as h:
        pk, sc = h.export()
    assert np.array_equal(pk, packed.reshape(n, k // 8)[1000:3000])
    assert np.array_equal(sc, scales[1000:3000])


def test_logical_handle_computes_like_packed_handle(session, oracle, cuda):
    cfg = synth.CONFIGS["decode"]
    w_kn, packed, scales = synth.make_weights(cfg.k, cfg.n, cfg.scale_lo, cfg.scale_hi, 3)
    x = synth.make_x(4, cfg.k, 5)
    with session.weights(packed, scales, cfg.k, cfg.n) as h1, \
            session.weights_logical(w_kn, scales, cfg.k, cfg.n) as h2:
        y1, y2 = h1.run_host(x), h2.run_host(x)
    assert np.array_equal(y1, y2)
