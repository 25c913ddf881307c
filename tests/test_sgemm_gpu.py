"""GPU: spaceslug_sgemm, the reference's fp32 GEMM ABI
(vulkan-runtime/src/api/sgemm_api.h:5-9), at its own test case
(tests/test_sgemm.cpp: 256^3, LCG inputs, |gpu - ref| <= 1e-3 * max(1, |ref|)),
computed on the tcgen05 tensor cores with three TF32 products per term
(hi*hi + hi*lo + lo*hi), checked against an fp64 product at 1e-4."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from spaceslug_b200 import synth

pytestmark = pytest.mark.gpu


def _check(c, a, b, tol=1e-3):
    ref = a.astype(np.float64) @ b.astype(np.float64)
    err = np.abs(c - ref) / np.maximum(1.0, np.abs(ref))
    assert float(err.max()) <= tol, float(err.max())


def test_reference_case(session, cuda):
    a = synth.lcg_floats(256 * 256, 0x12345678, -1.0, 1.0).reshape(256, 256)
    b = synth.lcg_floats(256 * 256, 0x9ABCDEF0, -1.0, 1.0).reshape(256, 256)
    _check(session.sgemm(a, b), a, b)


@pytest.mark.parametrize("m,n,k", [(64, 64, 32), (128, 192, 96), (1024, 1024, 1024), (64, 4096, 512),
                                   (2048, 2048, 2048), (256, 64, 8192)])
def test_shapes(session, cuda, m, n, k):
    # fp32-level: 1e-4 of max(1, |ref|) (the reference test's bar is 1e-3)
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    _check(session.sgemm(a, b), a, b, 1e-4)


def test_device_entry_any_shape(session, cuda):
    import torch
    rng = np.random.default_rng(1)
    a = rng.standard_normal((37, 100)).astype(np.float32)
    b = rng.standard_normal((100, 51)).astype(np.float32)
    da, db = torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)
    dc = torch.empty((37, 51), device=cuda)
    session.sgemm_device(da.data_ptr(), db.data_ptr(), dc.data_ptr(), 37, 51, 100,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    _check(dc.cpu().numpy(), a, b, 1e-4)


def test_reports_zero_error_like_the_reference(session, cuda):
    a = np.ones((64, 32), np.float32)
    b = np.ones((32, 64), np.float32)
    c = np.empty((64, 64), np.float32)
    err = ctypes.c_float(-1.0)
    f = lambda x: x.ctypes.data_as(ctypes.POINTER(ctypes.c_float))  # noqa: E731
    assert session.raw("spaceslug_sgemm")(f(a), f(b), f(c), 64, 64, 32, ctypes.byref(err)) == 0
    assert err.value == 0.0 and np.all(c == 32.0)


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (37, 51, 37), (130, 17, 5), (300, 129, 1000), (5, 2000, 64),
                                   (2000, 1800, 700), (2300, 2600, 333)])
def test_device_entry_ragged(session, cuda, m, n, k):
    # tiles of 128 rows x 16/32/64/128 columns, ragged in every dimension, K not a multiple of 4;
    # the last two run on CTA pairs (256 x 256 tiles; 2300 x 2600 gives most pairs two tiles)
    import torch
    rng = np.random.default_rng(m * n + k)
    a = (rng.standard_normal((m, k)) * 3).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    da, db = torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)
    dc = torch.full((m, n), float("nan"), device=cuda)
    session.sgemm_device(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    _check(dc.cpu().numpy(), a, b, 1e-4)
    assert session.device_status(0) == 0


@pytest.mark.parametrize("k", [1024, 8192])
def test_accuracy_is_fp32_level(session, cuda, k):
    # 3xTF32 keeps about 22 bits of every operand, and the accumulator is
    # summed in fp32 with round-to-nearest every 32 k (the tensor core's own
    # accumulation truncates): normwise error near fp32 GEMM rounding and no
    # bias growing with K (single-pass TF32 would be ~3e-4 normwise)
    rng = np.random.default_rng(9)
    a = rng.standard_normal((512, k)).astype(np.float32)
    b = rng.standard_normal((k, 512)).astype(np.float32)
    c = session.sgemm(a, b)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert np.linalg.norm(c - ref) / np.linalg.norm(ref) < 2e-6
    assert abs(float(np.mean((c - ref) * np.sign(ref)))) < 2e-6 * np.sqrt(k)  # no pull toward zero


@pytest.mark.parametrize("m,n,k", [(2048, 2048, 8192), (2304, 2560, 992), (4096, 4096, 1024)])
def test_pair_tiles_accuracy(session, cuda, m, n, k):
    # problems this large run on CTA pairs (cta_group::2, 256 x 256 tiles of C;
    # 4096 x 4096 gives most pairs four tiles):
    # the bars of the single-CTA accuracy test above (normwise near fp32
    # rounding, no bias growing with K) and the reference's elementwise 1e-3
    rng = np.random.default_rng(m + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    c = session.sgemm(a, b)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    err = np.abs(c - ref) / np.maximum(1.0, np.abs(ref))
    assert float(err.max()) <= 1e-3, float(err.max())
    assert np.linalg.norm(c - ref) / np.linalg.norm(ref) < 2e-6
    assert abs(float(np.mean((c - ref) * np.sign(ref)))) < 2e-6 * np.sqrt(k)
