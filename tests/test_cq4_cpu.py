"""CPU: the CQ4 oracle restatement is pinned bit-exactly to the reference's own
cactus_quant_matmul (built from its sources into oracle/_ref), and the CQ4
C-ABI rejects bad matrices before any device work."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import cq4

needs_ref = pytest.mark.skipif(not cq4.CQ4Reference.available(), reason="oracle/_ref/libcq4ref.so not built")


@needs_ref
@pytest.mark.parametrize("spec", cq4.REFERENCE_FIXTURES, ids=[s[0] for s in cq4.REFERENCE_FIXTURES])
def test_restatement_matches_reference_cpu_oracle(spec):
    fx = cq4.make_fixture(*spec)
    ref = cq4.CQ4Reference()
    assert np.array_equal(cq4.quant_matmul(fx), ref.quant_matmul(fx))
    if not fx.orthogonal:
        assert np.array_equal(cq4.transform_hadamard(fx).view(np.uint32), ref.transform_hadamard(fx).view(np.uint32))


@needs_ref
def test_restatement_matches_reference_on_random_signed_permuted_groups():
    fx = cq4.random_fixture(5, 20, 64, 3, False, True, False, seed=4)
    assert np.array_equal(cq4.quant_matmul(fx), cq4.CQ4Reference().quant_matmul(fx))


def test_fixture_generators_are_the_reference_streams():
    # m6c1::gen_f32 with seed 1 over [0, 1): u = (s >> 8) / 2^24 of the first LCG state
    s1 = (1 * 1664525 + 1013904223) & 0xFFFFFFFF
    assert cq4.gen_f32(1, 1, 0.0, 1.0)[0] == np.float32((s1 >> 8) / 16777216.0)
    p = cq4.gen_permutation(128, 7)
    assert sorted(p.tolist()) == list(range(128))
    assert set(cq4.gen_signs(64, 3).tolist()) <= {-1, 1}


def test_interleaved_packing_round_trip():
    idx = np.random.default_rng(0).integers(0, 16, (8, 256), dtype=np.uint32)
    packed = cq4.pack_interleaved_4row(idx, 8, 128, 2)
    fx = cq4.make_fixture("t", 1, 8, 128, 2, True, False, False, False)
    fx.packed, fx.idx = packed, idx
    # decode every index back through the stored-layout rule of extract_idx_interleaved_4row
    for n in range(8):
        for k in range(256):
            g, kk = divmod(k, 128)
            panel = ((n // 4) * 2 + g) * (4 * 64)
            b = packed[panel + (kk // 8) * 16 + (n & 3) * 4 + (kk & 3)]
            assert ((b >> 4) if kk & 4 else (b & 0xF)) == idx[n, k]


def test_cq4_create_rejects_bad_matrices(session):
    from spaceslug_b200.backend import CQ4Matrix
    cb = np.zeros(16, np.uint16)
    nm = np.ones(64, np.uint16)
    pk = np.zeros(64 * 64, np.uint8)
    h = ctypes.c_void_p()
    f = session.raw("spaceslug_cq4_weights_create")

    def call(**kw):
        d = dict(bits=4, k=128, n=64, group_size=128, num_groups=1, flags=0)
        d.update(kw)
        m = CQ4Matrix(d["bits"], d["k"], d["n"], d["group_size"], d["num_groups"], d["flags"])
        m.codebook, m.norms, m.packed_indices = cb.ctypes.data, nm.ctypes.data, pk.ctypes.data
        if "perm" in kw:
            m.permutation = kw["perm"].ctypes.data
        return f(ctypes.addressof(m), 0, ctypes.byref(h))

    assert f(None, 0, ctypes.byref(h)) == 1
    assert call(bits=3) == 1
    assert call(k=112, group_size=112) == 1           # K % 32
    assert call(k=96, group_size=48, num_groups=2) == 1  # group size not a power of two
    assert call(k=256, group_size=128, num_groups=1) == 1  # K != gs * ng
    assert call(flags=cq4.FLAG_INTERLEAVED_4ROW, n=62) == 1
    assert call(flags=cq4.FLAG_ORTHOGONAL) == 1       # no rotation
    assert call(perm=np.full(128, 128, np.uint32)) == 1
    assert session.raw("spaceslug_cq4_weights_destroy")(None) == 1
    assert session.raw("spaceslug_cq4_matmul_host")(None, None, None, 1) == 1
