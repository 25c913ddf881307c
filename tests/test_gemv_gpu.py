"""GPU parity of the decode GEMV (M <= 8) against the double-precision oracle.

Bar (fp32 GEMV path): the reference criterion |y - ref| / max(1, |ref|),
with tolerance 1e-4 (tighter than the reference test's 1e-3,
vulkan-runtime/tests/test_q4gemm.cpp:49).
"""
from __future__ import annotations

import numpy as np
import pytest

from spaceslug_b200 import parity, synth

pytestmark = pytest.mark.gpu

TOL = parity.GEMV_REL_TOL


@pytest.fixture(params=["imma", "tile", "mma", "gemv"])
def decode_variant(request, session):
    prev = session.set_decode_variant(request.param)
    yield request.param
    session.set_decode_variant(prev)


@pytest.fixture(scope="module")
def decode_weights():
    cfg = synth.CONFIGS["decode"]
    return synth.make_weights(cfg.k, cfg.n, cfg.scale_lo, cfg.scale_hi, 0)


@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 6, 7, 8])
def test_gemv_config2_full(session, oracle, cuda, decode_weights, decode_variant, m):
    w_kn, packed, scales = decode_weights
    x = synth.make_x(m, 4096, seed=m)
    y = session.q4gemm(x, packed, scales, 4096)
    ref = oracle.gemm(x, w_kn, scales)
    rep = parity.compare_float_arrays(y, ref, tolerance=TOL)
    assert rep["status"] == "pass", rep


@pytest.mark.parametrize("m,n,k", [(1, 1, 32), (2, 5, 64), (3, 200, 96), (8, 1000, 64), (5, 37, 4096),
                                   (1, 4096, 8192), (4, 300, 1024), (8, 64, 2048), (6, 129, 160)])
def test_gemv_ragged_shapes(session, oracle, cuda, decode_variant, m, n, k):
    w_kn, packed, scales = synth.make_weights(k, n, 0.005, 0.02, seed=n + k)
    x = synth.make_x(m, k, seed=m * 7 + 1)
    y = session.q4gemm(x, packed, scales, n)
    ref = oracle.gemm(x, w_kn, scales)
    rep = parity.compare_float_arrays(y, ref, tolerance=TOL)
    assert rep["status"] == "pass", (m, n, k, rep)


@pytest.mark.parametrize("m", [1, 4, 8])
def test_gemv_fused_lora(session, oracle, cuda, decode_variant, m):
    k, n, r, alpha = 1024, 768, 16, 32.0
    w_kn, packed, scales = synth.make_weights(k, n, 0.005, 0.02, seed=5)
    x = synth.make_x(m, k, seed=9)
    a = synth.normal(k * r, 21, 0.02).reshape(k, r)
    b = synth.normal(r * n, 22, 0.02).reshape(r, n)
    y = session.q4gemm(x, packed, scales, n, a, b, alpha)
    ref = oracle.gemm(x, w_kn, scales)
    oracle.lora_add(ref, x, a, b, alpha)
    rep = parity.compare_float_arrays(y, ref, tolerance=TOL)
    assert rep["status"] == "pass", rep


def test_gemv_device_api_matches_host_api(session, cuda, decode_weights):
    import torch
    w_kn, packed, scales = decode_weights
    x = synth.make_x(4, 4096, seed=3)
    y_host = session.q4gemm(x, packed, scales, 4096)
    dx = torch.from_numpy(x).to(cuda)
    dp = torch.from_numpy(packed.view(np.int32)).to(cuda)
    ds = torch.from_numpy(scales).to(cuda)
    dy = torch.empty((4, 4096), dtype=torch.float32, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    session.q4gemm_device(dx.data_ptr(), dp.data_ptr(), ds.data_ptr(), dy.data_ptr(), 4, 4096, 4096, stream)
    torch.cuda.synchronize()
    assert np.array_equal(dy.cpu().numpy(), y_host), "device and host entry points must be bit-identical"
    assert session.device_status(0) == 0


def test_gemv_is_deterministic(session, cuda, decode_weights, decode_variant):
    w_kn, packed, scales = decode_weights
    x = synth.make_x(8, 4096, seed=4)
    y1 = session.q4gemm(x, packed, scales, 4096)
    y2 = session.q4gemm(x, packed, scales, 4096)
    assert np.array_equal(y1, y2)


def test_gemv_resident_weights_and_shards(session, oracle, cuda, decode_weights):
    w_kn, packed, scales = decode_weights
    x = synth.make_x(2, 4096, seed=12)
    ref = oracle.gemm(x, w_kn, scales)
    full = session.weights(packed, scales, 4096, 4096)
    try:
        y = full.run_host(x)
    finally:
        full.close()
    assert parity.compare_float_arrays(y, ref, tolerance=TOL)["status"] == "pass"
    # four column shards reproduce the full result (to fp32 summation order:
    # the integer-MMA GEMV splits K differently for 1024 and 4096 columns)
    parts = []
    for r in range(4):
        with session.weights(packed, scales, 4096, 4096, r * 1024, (r + 1) * 1024) as h:
            parts.append(h.run_host(x))
    rep = parity.compare_float_arrays(np.concatenate(parts, axis=1), y, tolerance=1e-5)
    assert rep["status"] == "pass", rep


# Shapes for the integer-tensor-core GEMV's geometry: K split over 1, 2 or 4
# CTAs of a cluster, 1 to 7 tiles of 16 columns per CTA, ragged last tiles.
@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (3, 4096, 2048), (8, 512, 1024), (5, 100, 4096),
                                   (2, 1700, 3072), (7, 11008, 4096), (6, 4001, 8192), (4, 16, 1024)])
def test_gemv_imma_geometries(session, oracle, cuda, m, n, k):
    prev = session.set_decode_variant("imma")
    try:
        w_kn, packed, scales = synth.make_weights(k, n, 0.005, 0.02, seed=3 * n + k)
        x = synth.make_x(m, k, seed=m + 40)
        y = session.q4gemm(x, packed, scales, n)
    finally:
        session.set_decode_variant(prev)
    rep = parity.compare_float_arrays(y, oracle.gemm(x, w_kn, scales), tolerance=TOL)
    assert rep["status"] == "pass", (m, n, k, rep)


def test_gemv_imma_magnitudes_and_zero_rows(session, oracle, cuda):
    # rows of very different scales (each row and K slice gets its own power
    # of two), an all-zero row, and tiny group scales
    m, n, k = 6, 640, 4096
    w_kn, packed, scales = synth.make_weights(k, n, 1e-6, 4e-6, seed=77)
    x = synth.make_x(m, k, seed=78)
    x[0] *= np.float32(1e6)
    x[1] *= np.float32(1e-6)
    x[2] = 0.0
    x[3, :1024] *= np.float32(1e4)  # one K slice far larger than the others
    prev = session.set_decode_variant("imma")
    try:
        y = session.q4gemm(x, packed, scales, n)
    finally:
        session.set_decode_variant(prev)
    ref = oracle.gemm(x, w_kn, scales)
    assert np.all(y[2] == 0.0)
    for r in range(m):  # relative to each row's own magnitude
        rel = np.max(np.abs(y[r] - ref[r])) / max(np.max(np.abs(ref[r])), 1e-300)
        assert rel <= TOL, (r, rel)


def test_gemv_imma_non_finite_row(session, cuda):
    m, n, k = 3, 256, 1024
    w_kn, packed, scales = synth.make_weights(k, n, 0.005, 0.02, seed=5)
    x = synth.make_x(m, k, seed=6)
    x_ok = x.copy()
    x[1, 17] = np.inf
    prev = session.set_decode_variant("imma")
    try:
        y = session.q4gemm(x, packed, scales, n)
        y_ok = session.q4gemm(x_ok, packed, scales, n)
    finally:
        session.set_decode_variant(prev)
    assert np.all(np.isnan(y[1]))  # a row holding inf or NaN gives NaN outputs
    assert np.array_equal(y[[0, 2]], y_ok[[0, 2]])
