"""GPU: LoRA training -- the reference's hidden-64 ABI at its own test cases
and tolerances (vulkan-runtime/tests/test_lora_{gradients,sgd,train}_api.cpp),
and backward/SGD/AdamW on a resident handle against float64 numpy."""
from __future__ import annotations

import numpy as np
import pytest

from spaceslug_b200 import synth

pytestmark = pytest.mark.gpu


def _ref_inputs(m, rank):
    # test_lora_gradients_api.cpp:9-13
    x = np.sin(np.arange(m * 64, dtype=np.float32) * np.float32(0.07)).astype(np.float32)
    dy = np.cos(np.arange(m * 64, dtype=np.float32) * np.float32(0.03)).astype(np.float32)
    a = (np.cos(np.arange(64 * rank, dtype=np.float32) * np.float32(0.11)) * np.float32(0.1)).astype(np.float32)
    b = (np.sin(np.arange(rank * 64, dtype=np.float32) * np.float32(0.13)) * np.float32(0.1)).astype(np.float32)
    return x.reshape(m, 64), dy.reshape(m, 64), a.reshape(64, rank), b.reshape(rank, 64)


@pytest.mark.parametrize("m,rank", [(3, 4), (1, 1), (128, 8), (77, 5)])
def test_reference_gradients(session, cuda, m, rank):
    x, dy, a, b = _ref_inputs(m, rank)
    da, db = session.lora_gradients(x, dy, a, b, m, rank)
    X, DY, A, B = (v.astype(np.float64) for v in (x, dy, a, b))
    assert np.max(np.abs(da - X.T @ DY @ B.T)) <= 3e-4 * max(1.0, m / 3)
    assert np.max(np.abs(db - (X @ A).T @ DY)) <= 3e-4 * max(1.0, m / 3)


def test_reference_sgd(session, cuda):
    # test_lora_sgd_api.cpp: 1e-6 abs
    rank, lr = 4, np.float32(0.05)
    i = np.arange(64 * rank, dtype=np.float32)
    a, b = np.sin(i * np.float32(0.07)), np.cos(i * np.float32(0.03))
    da, db = np.cos(i * np.float32(0.11)), np.sin(i * np.float32(0.13))
    a1, b1 = session.lora_sgd(a, b, da, db, lr, rank)
    assert np.max(np.abs(a1 - (a - lr * da))) <= 1e-6
    assert np.max(np.abs(b1 - (b - lr * db))) <= 1e-6


def test_reference_train_step(session, cuda):
    # test_lora_train_api.cpp: forward delta, gradients at the old A/B, SGD; 3e-4 abs
    m, rank, lr = 3, 4, 0.05
    x, dy, a, b = _ref_inputs(m, rank)
    y, a1, b1 = session.lora_train_step(x, dy, a, b, lr, m, rank)
    X, DY, A, B = (v.astype(np.float64) for v in (x, dy, a, b))
    assert np.max(np.abs(y - X @ A @ B)) <= 3e-4
    assert np.max(np.abs(a1.reshape(64, rank) - (A - lr * X.T @ DY @ B.T))) <= 3e-4
    assert np.max(np.abs(b1.reshape(rank, 64) - (B - lr * (X @ A).T @ DY))) <= 3e-4


def test_reference_abi_rejects_bad_arguments(session):
    import ctypes
    f = session.raw("spaceslug_lora_gradients")
    z = np.zeros(64 * 8 * 4, np.float32).ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    assert f(z, z, z, z, z, z, 0, 4) == 1 and f(z, z, z, z, z, z, 129, 4) == 1 and f(z, z, z, z, z, z, 3, 9) == 1
    assert session.raw("spaceslug_lora_sgd")(z, z, z, z, 0.0, 4) == 1
    assert session.raw("spaceslug_lora_train_step")(z, z, z, z, z, -1.0, 3, 4) == 1


@pytest.mark.parametrize("m,k,n,rank,c0,c1", [(64, 4096, 4096, 16, 0, 4096), (33, 512, 700, 5, 100, 600),
                                             (300, 1024, 256, 64, 0, 256)])
def test_handle_backward_sgd_adamw(session, cuda, m, k, n, rank, c0, c1):
    import torch
    rng = np.random.default_rng(m + k + n)
    w_kn, packed, scales = synth.make_weights(k, n, 0.005, 0.02, seed=3)
    A = rng.standard_normal((k, rank)).astype(np.float32) * np.float32(0.02)
    B = rng.standard_normal((rank, n)).astype(np.float32) * np.float32(0.02)
    alpha = 2.0 * rank
    s = alpha / rank
    x = rng.standard_normal((m, k)).astype(np.float32)
    nl = c1 - c0
    dy = rng.standard_normal((m, nl)).astype(np.float32)
    with session.weights(packed, scales, k, n, c0, c1) as h:
        h.set_lora(A, B, alpha)
        xd, dyd = torch.from_numpy(x).to(cuda), torch.from_numpy(dy).to(cuda)
        h.lora_backward(xd.data_ptr(), dyd.data_ptr(), m, torch.cuda.current_stream().cuda_stream)
        a0, b0, da, db = h.get_lora(rank, grads=True)
        X, DY, A64, B64 = x.astype(np.float64), dy.astype(np.float64), A.astype(np.float64), B[:, c0:c1].astype(np.float64)
        da_ref = s * X.T @ (DY @ B64.T)
        db_ref = s * (X @ A64).T @ DY
        assert np.max(np.abs(da - da_ref)) <= 1e-4 * np.max(np.abs(da_ref))
        assert np.max(np.abs(db - db_ref)) <= 1e-4 * np.max(np.abs(db_ref))
        assert np.array_equal(b0, B[:, c0:c1])
        lr = 0.01
        h.lora_sgd(lr, torch.cuda.current_stream().cuda_stream)
        a1, b1 = h.get_lora(rank)
        assert np.max(np.abs(a1 - (a0 - np.float32(lr) * da))) <= 1e-6 * max(1.0, float(np.max(np.abs(a0))))
        assert np.max(np.abs(b1 - (b0 - np.float32(lr) * db))) <= 1e-6 * max(1.0, float(np.max(np.abs(b0))))
        # two AdamW steps on the same gradients against a float64 restatement
        p_a, p_b = a1.astype(np.float64), b1.astype(np.float64)
        ma = va = np.zeros_like(p_a)
        mb = vb = np.zeros_like(p_b)
        b1c, b2c, eps, wd, lr2 = 0.9, 0.999, 1e-8, 0.01, 1e-3
        for t in (1, 2):
            h.lora_adamw(lr2, b1c, b2c, eps, wd, torch.cuda.current_stream().cuda_stream)
            ga, gb = da.astype(np.float64), db.astype(np.float64)
            ma, va = b1c * ma + (1 - b1c) * ga, b2c * va + (1 - b2c) * ga * ga
            mb, vb = b1c * mb + (1 - b1c) * gb, b2c * vb + (1 - b2c) * gb * gb
            p_a = p_a - lr2 * ((ma / (1 - b1c ** t)) / (np.sqrt(va / (1 - b2c ** t)) + eps) + wd * p_a)
            p_b = p_b - lr2 * ((mb / (1 - b1c ** t)) / (np.sqrt(vb / (1 - b2c ** t)) + eps) + wd * p_b)
        a2, b2 = h.get_lora(rank)
        assert np.max(np.abs(a2 - p_a)) <= 1e-5
        assert np.max(np.abs(b2 - p_b)) <= 1e-5


@pytest.mark.parametrize("m,k,n,rank,c0,c1", [(512, 4096, 4096, 16, 0, 4096), (300, 1024, 700, 5, 100, 600),
                                             (200, 512, 384, 64, 0, 384), (333, 2048, 1024, 24, 0, 1024),
                                             (128, 256, 160, 8, 0, 160)])
def test_handle_backward_tensor_core_path(session, cuda, m, k, n, rank, c0, c1):
    # M >= 128 with 16-byte rows: the tcgen05 passes (T, G, dB, dA), against
    # float64 on the device; ragged tiles, every padded rank (8, 16, 32, 64),
    # a column shard; a second call is bit-identical (fixed-order split sums)
    import torch
    rng = np.random.default_rng(m * 7 + rank)
    _, packed, scales = synth.make_weights(k, n, 0.005, 0.02, seed=5)
    A = rng.standard_normal((k, rank)).astype(np.float32) * np.float32(0.02)
    B = rng.standard_normal((rank, n)).astype(np.float32) * np.float32(0.02)
    alpha = 2.0 * rank
    x = torch.randn((m, k), device=cuda)
    dy = torch.randn((m, c1 - c0), device=cuda)
    with session.weights(packed, scales, k, n, c0, c1) as h:
        h.set_lora(A, B, alpha)
        h.lora_backward(x.data_ptr(), dy.data_ptr(), m)
        _, _, da, db = h.get_lora(rank, grads=True)
        h.lora_backward(x.data_ptr(), dy.data_ptr(), m)
        _, _, da2, db2 = h.get_lora(rank, grads=True)
    X, DY = x.double(), dy.double()
    A64 = torch.from_numpy(A).to(cuda).double()
    B64 = torch.from_numpy(np.ascontiguousarray(B[:, c0:c1])).to(cuda).double()
    s = alpha / rank
    da_ref = (s * X.T @ (DY @ B64.T)).cpu().numpy()
    db_ref = (s * (X @ A64).T @ DY).cpu().numpy()
    assert np.max(np.abs(da - da_ref)) <= 1e-5 * np.max(np.abs(da_ref))
    assert np.max(np.abs(db - db_ref)) <= 1e-5 * np.max(np.abs(db_ref))
    assert np.array_equal(da, da2) and np.array_equal(db, db2)


def test_handle_backward_configs4_size(session, cuda):
    # the configs[4]-sized backward (X 4096 x 8192, dY 4096 x 28672, rank 16)
    # against float64 on the device
    import torch
    m, k, n, rank = 4096, 8192, 28672, 16
    rng = np.random.default_rng(44)
    _, packed, scales = synth.make_weights(k, n, 0.003, 0.01, seed=0)
    A = rng.standard_normal((k, rank)).astype(np.float32) * np.float32(0.02)
    B = rng.standard_normal((rank, n)).astype(np.float32) * np.float32(0.02)
    gen = torch.Generator(device=cuda).manual_seed(7)
    x = torch.randn((m, k), device=cuda, generator=gen)
    dy = torch.randn((m, n), device=cuda, generator=gen)
    with session.weights(packed, scales, k, n) as h:
        h.set_lora(A, B, 32.0)
        h.lora_backward(x.data_ptr(), dy.data_ptr(), m)
        _, _, da, db = h.get_lora(rank, grads=True)
    X, DY = x.double(), dy.double()
    s = 32.0 / rank
    da_ref = (s * X.T @ (DY @ torch.from_numpy(B).to(cuda).double().T)).cpu().numpy()
    db_ref = (s * (X @ torch.from_numpy(A).to(cuda).double()).T @ DY).cpu().numpy()
    assert np.max(np.abs(da - da_ref)) <= 1e-5 * np.max(np.abs(da_ref))
    assert np.max(np.abs(db - db_ref)) <= 1e-5 * np.max(np.abs(db_ref))


def test_training_reduces_the_loss(session, cuda):
    # fit the adapter to a teacher adapter through the fused forward (MSE)
    import torch
    rng = np.random.default_rng(9)
    k, n, m, rank = 512, 384, 128, 8
    _, packed, scales = synth.make_weights(k, n, 0.005, 0.02, seed=4)
    At = rng.standard_normal((k, rank)).astype(np.float32) * np.float32(0.05)
    Bt = rng.standard_normal((rank, n)).astype(np.float32) * np.float32(0.05)
    x = rng.standard_normal((m, k)).astype(np.float32)
    xd = torch.from_numpy(x).to(cuda)
    with session.weights(packed, scales, k, n) as teacher, session.weights(packed, scales, k, n) as h:
        teacher.set_lora(At, Bt, float(rank))
        target = torch.empty((m, n), device=cuda)
        teacher.run(xd.data_ptr(), target.data_ptr(), m)
        h.set_lora(rng.standard_normal((k, rank)).astype(np.float32) * np.float32(0.01),
                   np.zeros((rank, n), np.float32), float(rank))
        y = torch.empty((m, n), device=cuda)
        losses = []
        for _ in range(40):
            h.run(xd.data_ptr(), y.data_ptr(), m)
            diff = (y - target).contiguous()
            losses.append(float((diff * diff).mean()))
            grad = (diff * (2.0 / (m * n))).contiguous()
            h.lora_backward(xd.data_ptr(), grad.data_ptr(), m)
            h.lora_adamw(3e-3)
        torch.cuda.synchronize()
    assert losses[-1] < 0.5 * losses[0], losses[::8]
