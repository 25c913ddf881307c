"""GPU: bit-exact dequant, device packer, the legacy LoRA delta ABI, and the
re-layout of all-gathered column shards."""
from __future__ import annotations

import numpy as np
import pytest

from spaceslug_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k,n", [(32, 16), (64, 256), (4096, 512), (96, 37)])
def test_dequant_bit_exact(session, oracle, cuda, k, n):
    w_kn, packed, scales = synth.make_weights(k, n, 0.005, 0.02, seed=k + n)
    w = session.q4_dequant(packed, scales, k, n)
    ref = oracle.dequant(packed, scales, k, n)
    assert np.array_equal(w.view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(w, w_kn.astype(np.float32) * np.repeat(scales.T, 32, axis=0))


def test_dequant_every_nibble_and_lane(session, oracle, cuda):
    k, n = 64, 16
    b = ((np.arange(k)[:, None] * 3 + np.arange(n)[None, :]) % 16 - 8).astype(np.int8)
    s = synth.lcg_floats(n * 2, 77, -3.0, 3.0).reshape(n, 2)  # signed scales too
    p = synth.pack(b)
    w = session.q4_dequant(p, s, k, n)
    assert np.array_equal(w.view(np.uint32), oracle.dequant(p, s, k, n).view(np.uint32))


def test_device_pack_matches_host_pack(session, cuda):
    import torch
    k, n = 256, 1000
    b = synth.lcg_int4(k * n, 5).reshape(k, n)
    db = torch.from_numpy(b).to(cuda)
    dp = torch.empty(k * n // 8, dtype=torch.int32, device=cuda)
    session.q4_pack_device(db.data_ptr(), k, n, dp.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(dp.cpu().numpy().view(np.uint32), session.q4_pack(b))


def test_lora_delta_reference_case(session, cuda):
    # vulkan-runtime/tests/test_lora_delta_api.cpp:9-18 (m=3, rank=4, tolerance 2e-4)
    m, rank = 3, 4
    x = np.sin(np.arange(m * 64, dtype=np.float32) * np.float32(0.07)).astype(np.float32)
    a = (np.cos(np.arange(64 * rank, dtype=np.float32) * np.float32(0.11)) * np.float32(0.1)).astype(np.float32)
    b = (np.sin(np.arange(rank * 64, dtype=np.float32) * np.float32(0.13)) * np.float32(0.1)).astype(np.float32)
    y = session.lora_delta(x, a, b, m, rank)
    ref = ((x.reshape(m, 64).astype(np.float64) @ a.reshape(64, rank)) @ b.reshape(rank, 64)).reshape(-1)
    assert float(np.max(np.abs(y - ref))) <= 2e-4


@pytest.mark.parametrize("m,rank", [(1, 1), (17, 8), (128, 3)])
def test_lora_delta_against_shader_restatement(session, oracle, cuda, m, rank):
    rng = np.random.default_rng(m * 10 + rank)
    x = rng.standard_normal(m * 64).astype(np.float32)
    a = rng.standard_normal(64 * rank).astype(np.float32)
    b = rng.standard_normal(rank * 64).astype(np.float32)
    y = session.lora_delta(x, a, b, m, rank)
    ref = oracle.lora_delta_f32(x, a, b, m, rank)
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("parts,rows,width,n_total,ld", [(2, 300, 1024, 2048, 2048), (8, 64, 3584, 28672, 28672),
                                                        (2, 5, 104, 200, 200), (3, 7, 13, 37, 41), (4, 33, 8, 30, 64)])
def test_shards_relayout(session, cuda, parts, rows, width, n_total, ld):
    """Rank-major [parts][rows][width] -> rows of Y [rows][ld], columns [0, n_total),
    bit-exact; the padding columns of the last shard and Y's columns >= n_total untouched."""
    import torch
    g = torch.from_numpy(synth.lcg_floats(parts * rows * width, 9, -4.0, 4.0)).to(cuda)
    y = torch.full((rows, ld), 123.0, dtype=torch.float32, device=cuda)
    session.shards_relayout(g.data_ptr(), y.data_ptr(), parts, rows, width, n_total, ld,
                            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = g.cpu().numpy().reshape(parts, rows, width).transpose(1, 0, 2).reshape(rows, parts * width)[:, :n_total]
    out = y.cpu().numpy()
    assert np.array_equal(out[:, :n_total].view(np.uint32), ref.view(np.uint32))
    assert (out[:, n_total:] == 123.0).all()
