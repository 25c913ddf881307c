"""CPU: the oracle restatement and the synthetic generators against the
golden vectors produced by the reference's own code (tests/golden/)."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

from spaceslug_b200 import synth


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _parse_float_key(key):
    _, seed, lo, hi = key.split("_")
    return int(seed, 16), float(lo), float(hi)


def test_oracle_generators_match_reference(oracle, golden):
    g = golden["ref_generators"]
    for key in g.files:
        if key.startswith("floats_"):
            seed, lo, hi = _parse_float_key(key)
            assert np.array_equal(oracle.lcg_floats(4096, seed, lo, hi).view(np.uint32), g[key].view(np.uint32)), key
        else:
            seed = int(key.split("_")[1], 16)
            assert np.array_equal(oracle.lcg_int4(4096, seed), g[key]), key


def test_synth_generators_match_reference(golden):
    g = golden["ref_generators"]
    for key in g.files:
        if key.startswith("floats_"):
            seed, lo, hi = _parse_float_key(key)
            assert np.array_equal(synth.lcg_floats(4096, seed, lo, hi).view(np.uint32), g[key].view(np.uint32)), key
        else:
            seed = int(key.split("_")[1], 16)
            assert np.array_equal(synth.lcg_int4(4096, seed), g[key]), key


def _reference_case(oracle):
    M = N = K = 256
    a = oracle.lcg_floats(M * K, 0x12345678, -1.0, 1.0).reshape(M, K)
    b = oracle.lcg_int4(K * N, 0x9ABCDEF0).reshape(K, N)
    s = oracle.lcg_floats(N * (K // 32), 0x13579BDF, 0.5, 1.5).reshape(N, K // 32)
    return a, b, s


def test_oracle_pack_and_gemm_match_reference_case(oracle, golden):
    g = golden["ref_q4gemm_256"]
    a, b, s = _reference_case(oracle)
    packed = oracle.pack(b)
    assert _sha(packed) == str(g["packed_sha256"])
    assert np.array_equal(packed[:256], g["packed_head"])
    c = oracle.gemm(a, b, s)
    assert _sha(c) == str(g["c_sha256"]), "oracle GEMM must be bit-identical to the reference cpu_reference"
    assert np.array_equal(c.reshape(-1)[::61], g["c_samples"])
    # the packed-layout form of the oracle reads the same values
    assert np.array_equal(oracle.gemm_packed(a, packed, s, 256), c)


def test_oracle_matches_reference_on_config1(oracle, golden):
    t = golden["cfg_tiny"]
    assert np.array_equal(oracle.pack(t["w_kn"]), t["packed"])
    y = oracle.gemm(t["x"], t["w_kn"], t["scales"])
    assert np.array_equal(y, t["y_ref"])


def test_synth_config1_inputs_are_stable(golden):
    t = golden["cfg_tiny"]
    inp = synth.make_inputs("tiny")
    assert np.array_equal(inp.x.view(np.uint32), t["x"].view(np.uint32))
    assert np.array_equal(inp.w_kn, t["w_kn"])
    assert np.array_equal(inp.scales.view(np.uint32), t["scales"].view(np.uint32))
    assert np.array_equal(inp.packed, t["packed"])


@pytest.mark.parametrize("k,n", [(32, 1), (64, 3), (96, 40), (256, 256)])
def test_pack_unpack_round_trip(oracle, k, n):
    b = synth.lcg_int4(k * n, k * 1000 + n).reshape(k, n)
    p = synth.pack(b)
    assert np.array_equal(p, oracle.pack(b))
    assert np.array_equal(synth.unpack(p, k, n), b)
    assert np.array_equal(oracle.unpack(p, k, n), b)


def test_every_nibble_in_every_byte_lane(oracle):
    # K = 32, N = 16: column n holds the values (n + k) mod 16 - 8, so every
    # nibble value appears at every k parity and byte lane.
    k, n = 32, 16
    b = ((np.arange(k)[:, None] + np.arange(n)[None, :]) % 16 - 8).astype(np.int8)
    p = synth.pack(b)
    assert np.array_equal(p, oracle.pack(b))
    s = np.linspace(0.5, 2.0, n * (k // 32), dtype=np.float32).reshape(n, k // 32)
    w = oracle.dequant(p, s, k, n)
    assert np.array_equal(w, b.astype(np.float32) * s[:, 0][None, :])


def test_normal_generator_moments():
    z = synth.normal(1 << 20, 11)
    assert abs(float(z.mean())) < 5e-3 and abs(float(z.std()) - 1.0) < 5e-3
    assert np.all(np.isfinite(z))


def test_lora_oracle_matches_formula(oracle):
    rng = np.random.default_rng(3)
    m, k, n, r = 5, 64, 48, 4
    x = rng.standard_normal((m, k)).astype(np.float32)
    a = rng.standard_normal((k, r)).astype(np.float32)
    bb = rng.standard_normal((r, n)).astype(np.float32)
    out = np.zeros((m, n))
    oracle.lora_add(out, x, a, bb, 8.0)
    ref = (8.0 / r) * (x.astype(np.float64) @ a.astype(np.float64)) @ bb.astype(np.float64)
    assert np.allclose(out, ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", ["prefill", "lora", "mlp70b"])
def test_oracle_matches_reference_rows_of_large_configs(oracle, name):
    # cfg_rows.npz holds the reference's own cpu_reference (plus the LoRA
    # restatement for configs[3]) on sampled rows of configs[2]-[4]; the
    # double-precision restatement rounds to the same float32 values.
    t = np.load(Path(__file__).resolve().parent / "golden" / "cfg_rows.npz")
    inp = synth.make_inputs(name)
    rows = t[f"{name}_rows"][[0, -1]]
    y = oracle.gemm(np.ascontiguousarray(inp.x[rows]), inp.w_kn, inp.scales)
    if inp.rank:
        oracle.lora_add(y, np.ascontiguousarray(inp.x[rows]), inp.lora_a, inp.lora_b, inp.alpha)
    assert np.array_equal(y.astype(np.float32), t[f"{name}_y"][[0, -1]])
    assert float(t[f"{name}_xinf"]) == float(np.max(np.abs(inp.x)))
