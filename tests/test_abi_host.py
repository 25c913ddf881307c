"""CPU: the C-ABI library loads, exports every declared symbol, and its host
logic (packer, vector_add, argument validation) behaves like the reference."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from spaceslug_b200 import synth

HEADER = Path(__file__).resolve().parent.parent / "include" / "runtime_abi.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(spaceslug_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(session):
    lib = session._native()
    names = declared_symbols()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_backend_binds_every_declared_symbol(session):
    assert sorted(session.exported_symbols()) == declared_symbols()


def test_vector_add_reference_values(session):
    # native/runtime_abi_test.cpp:4-7
    out = session.vector_add([0.25, 1.5, -2.0], [0.75, 2.5, 3.0])
    assert out.tolist() == [1.0, 4.0, 1.0]
    f = session.raw("spaceslug_vector_add")
    assert f(None, None, None, 3) == 1


def test_vector_add_million(session):
    # native/runtime_api_client.cpp:5-11
    a = np.ones(1 << 20, np.float32)
    b = np.full(1 << 20, 2.0, np.float32)
    out = session.vector_add(a, b)
    assert out[0] == 3.0 and out[-1] == 3.0


# the host packer splits the k/8 output chunks over threads: 1 chunk, chunk
# counts that do not divide evenly, and a large matrix
@pytest.mark.parametrize("k,n", [(32, 1), (64, 256), (96, 37), (4096, 64), (1000 // 8 * 8 // 32 * 32, 3),
                                 (2080, 777), (8192, 513)])
def test_host_pack_matches_oracle(session, oracle, k, n):
    b = synth.lcg_int4(k * n, 7 * k + n).reshape(k, n)
    assert np.array_equal(session.q4_pack(b), oracle.pack(b))


def test_host_pack_out_of_range_values_like_reference(session, oracle):
    b = np.array(np.arange(-64, 64).reshape(32, 4), dtype=np.int8)  # values outside [-8,7] keep v & 0xF
    assert np.array_equal(session.q4_pack(b), oracle.pack(b))


def _f(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _u(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))


def test_invalid_arguments_return_1_before_device_work(session):
    x = np.zeros((4, 64), np.float32)
    p = np.zeros(64 * 64 // 8, np.uint32)
    s = np.ones((64, 2), np.float32)
    y = np.zeros((4, 64), np.float32)
    g = session.raw("spaceslug_q4gemm")
    assert g(None, _u(p), _f(s), _f(y), 4, 64, 64) == 1
    assert g(_f(x), _u(p), _f(s), _f(y), 0, 64, 64) == 1
    assert g(_f(x), _u(p), _f(s), _f(y), 4, 0, 64) == 1
    assert g(_f(x), _u(p), _f(s), _f(y), 4, 64, 48) == 1  # K % 32
    assert g(_f(x), _u(p), _f(s), _f(y), 4, 64, 0) == 1
    gl = session.raw("spaceslug_q4gemm_lora")
    a = np.zeros((64, 4), np.float32)
    b = np.zeros((4, 64), np.float32)
    assert gl(_f(x), _u(p), _f(s), None, _f(b), 4, 1.0, _f(y), 4, 64, 64) == 1
    assert gl(_f(x), _u(p), _f(s), _f(a), _f(b), 0, 1.0, _f(y), 4, 64, 64) == 1
    assert gl(_f(x), _u(p), _f(s), _f(a), _f(b), 65, 1.0, _f(y), 4, 64, 64) == 1
    assert gl(_f(x), _u(p), _f(s), _f(a), _f(b), 4, float("nan"), _f(y), 4, 64, 64) == 1
    gd = session.raw("spaceslug_q4gemm_device")
    assert gd(8, 16, 16, None, None, 0, 0.0, 16, 1, 1, 32, None) == 1  # x not 16-byte aligned
    pk = session.raw("spaceslug_q4_pack")
    w = np.zeros((32, 4), np.int8)
    assert pk(None, 32, 4, _u(p)) == 1
    assert pk(w.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)), 48, 4, _u(p)) == 1
    dq = session.raw("spaceslug_q4_dequant")
    assert dq(_u(p), _f(s), 48, 64, _f(y)) == 1
    wc = session.raw("spaceslug_q4_weights_create")
    h = ctypes.c_void_p()
    assert wc(_u(p), _f(s), 64, 64, 10, 5, 0, ctypes.byref(h)) == 1  # empty column range
    assert wc(_u(p), _f(s), 64, 64, 0, 65, 0, ctypes.byref(h)) == 1  # beyond n
    wl = session.raw("spaceslug_q4_weights_create_logical")
    assert wl(None, _f(s), 64, 64, 0, 64, 0, ctypes.byref(h)) == 1
    assert wl(w.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)), _f(s), 48, 4, 0, 4, 0, ctypes.byref(h)) == 1  # K % 32
    assert wl(w.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)), _f(s), 32, 4, 3, 3, 0, ctypes.byref(h)) == 1
    assert session.raw("spaceslug_q4_weights_export")(None, _u(p), _f(s)) == 1
    sg = session.raw("spaceslug_sgemm")
    e = ctypes.c_float()
    assert sg(_f(x), _f(x), _f(y), 64, 64, 48, ctypes.byref(e)) == 1   # K % 32 (sgemm_api.cpp:25)
    assert sg(_f(x), _f(x), _f(y), 32, 64, 32, ctypes.byref(e)) == 1   # M % 64
    assert sg(_f(x), _f(x), _f(y), 64, 64, 32, None) == 1
    assert session.raw("spaceslug_sgemm_device")(None, None, None, 1, 1, 1, None) == 1
    assert session.raw("spaceslug_q4_weights_run")(None, 16, 16, 1, None) == 1
    rs = session.raw("spaceslug_q4_weights_run_strided")
    assert rs(None, 16, 16, 1, 64, None) == 1
    assert session.raw("spaceslug_ipc_export")(None, None, None) == 1
    assert session.raw("spaceslug_ipc_open")(None, 0, 0, None, None) == 1
    assert session.raw("spaceslug_ipc_close")(None) == 1
    c2 = session.raw("spaceslug_copy_2d")
    assert c2(None, 64, 16, 64, 64, 1, None) == 1
    assert c2(16, 32, 16, 64, 64, 1, None) == 1   # width > dpitch
    assert c2(16, 64, 16, 64, 0, 1, None) == 0    # nothing to copy
    rl = session.raw("spaceslug_shards_relayout")
    assert rl(None, 16, 2, 4, 8, 16, 16, None) == 1
    assert rl(16, 16, 2, 4, 8, 17, 17, None) == 1   # n_total > parts * width
    assert rl(16, 16, 2, 4, 8, 16, 15, None) == 1   # ld_y < n_total
    assert rl(16, 16, 0, 4, 8, 16, 16, None) == 1
    assert rl(16, 16, 2, 0, 8, 16, 16, None) == 0   # nothing to move, no device work
    assert session.raw("spaceslug_q4_weights_destroy")(None) == 1
    assert session.raw("spaceslug_q4_set_operand_type")(7) == -1


def test_lora_delta_argument_contract(session):
    # vulkan-runtime/src/api/lora_delta_api.cpp:44: 1 <= m <= 128, 1 <= rank <= 8
    f = session.raw("spaceslug_lora_delta")
    x = np.zeros(64 * 129, np.float32)
    a = np.zeros(64 * 9, np.float32)
    y = np.zeros(64 * 129, np.float32)
    assert f(_f(x), _f(a), _f(a), _f(y), 0, 4) == 1
    assert f(_f(x), _f(a), _f(a), _f(y), 129, 4) == 1
    assert f(_f(x), _f(a), _f(a), _f(y), 3, 0) == 1
    assert f(_f(x), _f(a), _f(a), _f(y), 3, 9) == 1
    assert f(None, _f(a), _f(a), _f(y), 3, 4) == 1


def test_last_error_describes_failure(session):
    g = session.raw("spaceslug_q4gemm")
    x = np.zeros((1, 64), np.float32)
    assert g(_f(x), None, _f(x), _f(x), 1, 1, 64) == 1
    assert b"null" in session.raw("spaceslug_last_error")()


def test_capabilities(session):
    caps = session.capabilities()
    for c in ("vector_add", "lora_delta_abi", "q4gemm", "q4gemm_lora_fused", "q4_weights_resident"):
        assert c in caps
