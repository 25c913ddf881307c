"""GPU: the timeout path of the kernels' bounded waits, exercised without
faulting or hanging the GPU.

The test hook spaceslug_q4_debug_wait_test shortens the decode kernels' wait
limit to 1 ms and makes one warp per CTA wait on a barrier phase that nothing
arms.  That wait runs out, the kernel records the timeout in the status word,
raises its abort flag and returns; the host reports it as the ABI's code 3
(the reference's error-code contract: vulkan-runtime/src/api/lora_delta_api.cpp:44, 84,
extended with 3 = timeout).  Every case then checks that the next normal call
on the same context is correct.
"""
from __future__ import annotations

import numpy as np
import pytest

from spaceslug_b200 import parity, synth
from spaceslug_b200.backend import BackendError

pytestmark = pytest.mark.gpu

TIMEOUT = 3
K, N, M = 1024, 512, 2


@pytest.fixture
def stall(session, cuda):
    hook = session.raw("spaceslug_q4_debug_wait_test")
    assert hook(1_000_000, 1) == 0  # 1 ms wait limit, one stalled warp per CTA
    yield
    assert hook(0, 0) == 0
    session.device_status(0)  # leave no code behind for later tests


@pytest.fixture(params=["imma", "tile", "gemv"])
def decode_kernel(request, session):
    prev = session.set_decode_variant(request.param)
    yield request.param
    session.set_decode_variant(prev)


def _case():
    w_kn, packed, scales = synth.make_weights(K, N, 0.005, 0.02, seed=11)
    x = synth.make_x(M, K, seed=12)
    return w_kn, packed, scales, x


def _clear_hook(session):
    assert session.raw("spaceslug_q4_debug_wait_test")(0, 0) == 0


def test_synchronous_call_returns_timeout_then_recovers(session, oracle, cuda, decode_kernel, stall):
    w_kn, packed, scales, x = _case()
    with pytest.raises(BackendError) as info:
        session.q4gemm(x, packed, scales, N)
    assert info.value.code == TIMEOUT
    assert session.device_status(0) == 0  # the call read and cleared the word
    _clear_hook(session)
    y = session.q4gemm(x, packed, scales, N)
    rep = parity.compare_float_arrays(y, oracle.gemm(x, w_kn, scales), tolerance=parity.GEMV_REL_TOL)
    assert rep["status"] == "pass", rep
    assert session.device_status(0) == 0


def test_asynchronous_call_reports_through_device_status(session, oracle, cuda, decode_kernel, stall):
    import torch
    w_kn, packed, scales, x = _case()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    dx, dp, ds = t(x), t(packed.view(np.int32)), t(scales)
    dy = torch.empty((M, N), dtype=torch.float32, device=cuda)
    session.q4gemm_device(dx.data_ptr(), dp.data_ptr(), ds.data_ptr(), dy.data_ptr(), M, N, K)  # returns 0: async
    code = session.device_status(0)
    assert code != 0, "the stalled kernel's timeout was not recorded"
    assert session.device_status(0) == 0  # read and cleared
    _clear_hook(session)
    session.q4gemm_device(dx.data_ptr(), dp.data_ptr(), ds.data_ptr(), dy.data_ptr(), M, N, K)
    torch.cuda.synchronize()
    rep = parity.compare_float_arrays(dy.cpu().numpy(), oracle.gemm(x, w_kn, scales), tolerance=parity.GEMV_REL_TOL)
    assert rep["status"] == "pass", rep
    assert session.device_status(0) == 0


def test_pinned_host_call_returns_timeout_then_recovers(session, oracle, cuda, stall):
    # spaceslug_q4_weights_run_host with pinned X and Y: the status word rides
    # to the host with Y (a small copy kernel into a mapped host word), and the
    # host waits on the completion word that kernel's last CTA sets
    import ctypes

    import torch
    w_kn, packed, scales, x = _case()
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.empty((M, N), dtype=torch.float32).pin_memory()
    fp = ctypes.POINTER(ctypes.c_float)
    run_host = session.raw("spaceslug_q4_weights_run_host")
    with session.weights(packed, scales, K, N) as h:
        call = lambda: run_host(h.handle, ctypes.cast(xh.data_ptr(), fp), ctypes.cast(yh.data_ptr(), fp), M)  # noqa: E731
        assert call() == TIMEOUT
        assert call() == TIMEOUT  # the word was cleared and set again, not left over
        _clear_hook(session)
        assert call() == 0
    rep = parity.compare_float_arrays(yh.numpy(), oracle.gemm(x, w_kn, scales), tolerance=parity.GEMV_REL_TOL)
    assert rep["status"] == "pass", rep


def test_noalloc_entry_point_reports_through_device_status(session, oracle, cuda, stall):
    import torch
    w_kn, packed, scales, x = _case()
    rank, alpha = 8, 16.0
    a = synth.normal(K * rank, 13, 0.02).reshape(K, rank)
    b = synth.normal(rank * N, 14, 0.02).reshape(rank, N)
    t = lambda arr: torch.from_numpy(np.ascontiguousarray(arr)).to(cuda)  # noqa: E731
    args = [t(x), t(packed.view(np.int32)), t(scales), t(a), t(b)]
    dy = torch.empty((M, N), dtype=torch.float32, device=cuda)
    f = session.raw("spaceslug_q4gemv_lora_noalloc")
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        return f(*(v.data_ptr() for v in args), rank, alpha, dy.data_ptr(), M, N, K, stream)
    assert call() == 0  # asynchronous: the timeout is not known yet
    assert session.device_status(0) != 0
    assert session.device_status(0) == 0
    _clear_hook(session)
    assert call() == 0
    torch.cuda.synchronize()
    assert session.device_status(0) == 0
    ref = oracle.gemm(x, w_kn, scales)
    oracle.lora_add(ref, x, a, b, alpha)
    rep = parity.compare_float_arrays(dy.cpu().numpy(), ref, tolerance=parity.GEMV_REL_TOL)
    assert rep["status"] == "pass", rep
