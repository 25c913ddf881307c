"""GPU: the CQ4 quant matmul (activation transform + codebook dequant on the
tcgen05 GEMM) against the reference's own CPU oracle, with the reference
test's tolerances (tests/test_cq4.cpp:452, :470: fp16 abs 2e-2 / rel 1e-2 for
C, 1e-3 / 1e-2 for the transform)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import cq4

pytestmark = pytest.mark.gpu


def _handle(session, fx: cq4.Fixture):
    return session.cq4_weights(k=fx.K, n=fx.N, group_size=fx.gs, num_groups=fx.ng, flags=fx.flags,
                               codebook=fx.codebook, norms=fx.norms, packed=fx.packed, input_scale=fx.input_scale,
                               input_scale_recip=fx.input_scale_recip, left_signs=fx.left, right_signs=fx.right,
                               permutation=fx.perm, rotation=fx.rotation)


def _reference_c(fx):
    if cq4.CQ4Reference.available():
        return cq4.CQ4Reference().quant_matmul(fx)
    return cq4.quant_matmul(fx)  # the restatement, pinned to it by test_cq4_cpu.py


@pytest.mark.parametrize("spec", cq4.REFERENCE_FIXTURES, ids=[s[0] for s in cq4.REFERENCE_FIXTURES])
def test_reference_fixtures(session, cuda, spec):
    fx = cq4.make_fixture(*spec)
    with _handle(session, fx) as h:
        c = h.matmul_host(fx.a)
        a1 = h.transform_host(fx.a)
    rep = cq4.compare_fp16(c, _reference_c(fx), 2e-2, 1e-2)
    assert rep["ok"], rep
    # transform: the reference test's check against the double transform in fp16 ...
    tref = cq4.transform_double(fx).astype(np.float32).astype(np.float16).view(np.uint16)
    trep = cq4.compare_fp16(a1, tref, 1e-3, 1e-2)
    assert trep["ok"], trep
    # ... and bit-exactness against the fp32 transform of the reference CPU path, rounded to fp16
    f32 = cq4.transform_orthogonal_f32(fx) if fx.orthogonal else cq4.transform_hadamard(fx)
    assert np.array_equal(a1.reshape(-1), f32.astype(np.float16).view(np.uint16).reshape(-1))


@pytest.mark.parametrize("M,N,gs,ng,il,sp,orth", [
    (256, 384, 128, 8, False, True, False),   # signs + permutation, several groups
    (300, 260, 64, 16, True, False, False),   # ragged M and N tiles, interleaved panels
    (1, 512, 128, 4, True, True, False),      # decode row
    (37, 96, 32, 8, False, True, False),      # smallest group
    (130, 132, 256, 2, True, True, False),    # largest group
    (96, 128, 256, 1, True, False, True),     # orthogonal, interleaved lm_head layout
    (8, 200, 128, 4, False, True, False),     # decode kernel, 8 rows, ragged column block
    (5, 64, 256, 2, True, False, False),      # decode kernel, 5 rows
    (1, 64, 256, 1, False, False, True),      # decode kernel after the orthogonal transform
])
def test_random_shapes_match_the_oracle(session, cuda, M, N, gs, ng, il, sp, orth):
    fx = cq4.random_fixture(M, N, gs, ng, il, sp, orth, seed=M + N + gs)
    with _handle(session, fx) as h:
        c = h.matmul_host(fx.a)
    rep = cq4.compare_fp16(c, cq4.quant_matmul(fx), 2e-2, 1e-2)
    assert rep["ok"], rep


def test_reference_bench_size_sampled_rows(session, cuda):
    # bench_cq4gemm.cpp:51-55, 1024 x 1024 x 1024 at group size 128: rows sampled for the oracle
    fx = cq4.random_fixture(1024, 1024, 128, 8, True, True, False, seed=11)
    with _handle(session, fx) as h:
        c = h.matmul_host(fx.a).reshape(1024, 1024)
    rows = np.r_[0:4, 511:515, 1020:1024]
    sub = cq4.Fixture(**{**fx.__dict__, "M": len(rows), "a": fx.a.reshape(1024, -1)[rows].reshape(-1)})
    rep = cq4.compare_fp16(c[rows], cq4.quant_matmul(sub), 2e-2, 1e-2)
    assert rep["ok"], rep
    assert np.all(np.isfinite(c.view(np.float16)))


def test_device_entry_point_matches_host(session, cuda):
    import torch
    fx = cq4.random_fixture(64, 256, 128, 4, False, True, False, seed=3)
    with _handle(session, fx) as h:
        ref = h.matmul_host(fx.a)
        a = torch.from_numpy(fx.a.view(np.int16).reshape(64, -1).copy()).to(cuda)
        c = torch.empty((64, 256), dtype=torch.int16, device=cuda)
        h.matmul(a.data_ptr(), c.data_ptr(), 64, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
    assert np.array_equal(c.cpu().numpy().view(np.uint16), ref)
