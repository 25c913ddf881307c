"""ctypes front end of the CPU oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and
by bench.py's CPU-baseline leg, always as the checker (or the timed CPU
baseline), never by the shipped library.

Two libraries are exposed:
  * ``Oracle``    -> oracle/liboracle.so, the C restatement in q4_oracle.c;
  * ``Reference`` -> oracle/_ref/libq4ref.so, the reference's own CPU
    functions (vulkan-runtime/tests/test_q4gemm.cpp:57-119) compiled from its
    sources by oracle/Makefile.  Absent where the reference checkout was not
    available at build time (callers must handle ``available() is False``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_ORACLE_SO = HERE / "liboracle.so"
_REF_SO = HERE / "_ref" / "libq4ref.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i8p = ctypes.POINTER(ctypes.c_int8)
_u32p = ctypes.POINTER(ctypes.c_uint32)


def build(with_reference: bool = True, reference_root: str | None = None) -> None:
    """Compile the oracle (and the reference library when its sources exist).

    reference_root overrides the Makefile's REF (the reference checkout)."""
    target = "all" if with_reference else "oracle"
    extra = [f"REF={reference_root}"] if reference_root else []
    subprocess.run(["make", "-s", "-C", str(HERE), target, *extra], check=True)


def _ptr(arr: np.ndarray, typ):
    assert arr.flags["C_CONTIGUOUS"]
    return arr.ctypes.data_as(typ)


class Oracle:
    """The C restatement (oracle/q4_oracle.c)."""

    def __init__(self) -> None:
        if not _ORACLE_SO.is_file():
            build(with_reference=False)
        lib = ctypes.CDLL(str(_ORACLE_SO))
        lib.oq4_lcg_floats.argtypes = [ctypes.c_size_t, ctypes.c_uint32, ctypes.c_float, ctypes.c_float, _f32p]
        lib.oq4_lcg_int4.argtypes = [ctypes.c_size_t, ctypes.c_uint32, _i8p]
        lib.oq4_pack.argtypes = [_i8p, ctypes.c_uint32, ctypes.c_uint32, _u32p]
        lib.oq4_pack.restype = ctypes.c_int
        lib.oq4_unpack.argtypes = [_u32p, ctypes.c_uint32, ctypes.c_uint32, _i8p]
        lib.oq4_dequant.argtypes = [_u32p, _f32p, ctypes.c_uint32, ctypes.c_uint32, _f32p]
        lib.oq4_gemm_ref_rows.argtypes = [_f32p, _i8p, _f32p] + [ctypes.c_uint32] * 5 + [_f64p]
        lib.oq4_gemm_ref_packed_rows.argtypes = [_f32p, _u32p, _f32p] + [ctypes.c_uint32] * 4 + [_f64p]
        lib.oq4_lora_ref_rows.argtypes = [_f32p, _f32p, _f32p, ctypes.c_uint32, ctypes.c_uint32,
                                          ctypes.c_uint32, ctypes.c_float, ctypes.c_uint32, ctypes.c_uint32, _f64p]
        lib.oq4_lora_delta_f32.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_uint32, ctypes.c_uint32]
        lib.oq4_vector_add.argtypes = [_f32p, _f32p, _f32p, ctypes.c_size_t]
        lib.oq4_vector_add.restype = ctypes.c_int
        self.lib = lib

    def lcg_floats(self, n: int, seed: int, lo: float, hi: float) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.lib.oq4_lcg_floats(n, seed, lo, hi, _ptr(out, _f32p))
        return out

    def lcg_int4(self, n: int, seed: int) -> np.ndarray:
        out = np.empty(n, np.int8)
        self.lib.oq4_lcg_int4(n, seed, _ptr(out, _i8p))
        return out

    def pack(self, b_kn: np.ndarray) -> np.ndarray:
        k, n = b_kn.shape
        b = np.ascontiguousarray(b_kn, np.int8)
        out = np.empty(k * n // 8, np.uint32)
        assert self.lib.oq4_pack(_ptr(b, _i8p), k, n, _ptr(out, _u32p)) == 0
        return out

    def unpack(self, packed: np.ndarray, k: int, n: int) -> np.ndarray:
        out = np.empty((k, n), np.int8)
        self.lib.oq4_unpack(_ptr(np.ascontiguousarray(packed, np.uint32), _u32p), k, n, _ptr(out, _i8p))
        return out

    def dequant(self, packed: np.ndarray, scales: np.ndarray, k: int, n: int) -> np.ndarray:
        out = np.empty((k, n), np.float32)
        self.lib.oq4_dequant(_ptr(np.ascontiguousarray(packed, np.uint32), _u32p),
                             _ptr(np.ascontiguousarray(scales, np.float32), _f32p), k, n, _ptr(out, _f32p))
        return out

    def gemm(self, x: np.ndarray, b_kn: np.ndarray, scales: np.ndarray, rows=None) -> np.ndarray:
        """Double-precision reference C = X * dequant(B) (rows [m0, m1) if given)."""
        m, k = x.shape
        n = b_kn.shape[1]
        m0, m1 = rows if rows is not None else (0, m)
        out = np.empty((m1 - m0, n), np.float64)
        self.lib.oq4_gemm_ref_rows(_ptr(np.ascontiguousarray(x, np.float32), _f32p),
                                   _ptr(np.ascontiguousarray(b_kn, np.int8), _i8p),
                                   _ptr(np.ascontiguousarray(scales, np.float32), _f32p),
                                   m, n, k, m0, m1, _ptr(out, _f64p))
        return out

    def gemm_packed(self, x: np.ndarray, packed: np.ndarray, scales: np.ndarray, n: int, rows=None) -> np.ndarray:
        m, k = x.shape
        m0, m1 = rows if rows is not None else (0, m)
        out = np.empty((m1 - m0, n), np.float64)
        self.lib.oq4_gemm_ref_packed_rows(_ptr(np.ascontiguousarray(x, np.float32), _f32p),
                                          _ptr(np.ascontiguousarray(packed, np.uint32), _u32p),
                                          _ptr(np.ascontiguousarray(scales, np.float32), _f32p),
                                          n, k, m0, m1, _ptr(out, _f64p))
        return out

    def lora_add(self, out: np.ndarray, x: np.ndarray, lora_a: np.ndarray, lora_b: np.ndarray,
                 alpha: float, rows=None) -> np.ndarray:
        """out += (alpha/rank) * X[rows] A B, in double."""
        m, k = x.shape
        rank, n = lora_b.shape
        m0, m1 = rows if rows is not None else (0, m)
        assert out.shape == (m1 - m0, n) and out.dtype == np.float64 and out.flags["C_CONTIGUOUS"]
        self.lib.oq4_lora_ref_rows(_ptr(np.ascontiguousarray(x, np.float32), _f32p),
                                   _ptr(np.ascontiguousarray(lora_a, np.float32), _f32p),
                                   _ptr(np.ascontiguousarray(lora_b, np.float32), _f32p),
                                   k, n, rank, alpha, m0, m1, _ptr(out, _f64p))
        return out

    def lora_delta_f32(self, x: np.ndarray, a: np.ndarray, b: np.ndarray, m: int, rank: int) -> np.ndarray:
        y = np.empty(m * 64, np.float32)
        self.lib.oq4_lora_delta_f32(_ptr(np.ascontiguousarray(x, np.float32), _f32p),
                                    _ptr(np.ascontiguousarray(a, np.float32), _f32p),
                                    _ptr(np.ascontiguousarray(b, np.float32), _f32p),
                                    _ptr(y, _f32p), m, rank)
        return y


class Reference:
    """The reference's own CPU functions, compiled from its sources."""

    @staticmethod
    def available() -> bool:
        return _REF_SO.is_file()

    def __init__(self) -> None:
        if not _REF_SO.is_file():
            raise FileNotFoundError(f"reference oracle not built: {_REF_SO}")
        lib = ctypes.CDLL(str(_REF_SO))
        lib.ref_generate_floats.argtypes = [ctypes.c_size_t, ctypes.c_uint32, ctypes.c_float, ctypes.c_float, _f32p]
        lib.ref_generate_int4.argtypes = [ctypes.c_size_t, ctypes.c_uint32, _i8p]
        lib.ref_pack_q4.argtypes = [_i8p, ctypes.c_uint32, ctypes.c_uint32, _u32p]
        lib.ref_cpu_reference.argtypes = [_f32p, _i8p, _f32p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, _f64p]
        lib.ref_prepare.argtypes = [_f32p, _i8p, _f32p] + [ctypes.c_uint32] * 4
        lib.ref_prepare.restype = ctypes.c_void_p
        lib.ref_run.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.ref_run.restype = ctypes.c_int
        lib.ref_gather.argtypes = [ctypes.c_void_p, _f64p]
        lib.ref_release.argtypes = [ctypes.c_void_p]
        self.lib = lib

    def generate_floats(self, n: int, seed: int, lo: float, hi: float) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.lib.ref_generate_floats(n, seed, lo, hi, _ptr(out, _f32p))
        return out

    def generate_int4(self, n: int, seed: int) -> np.ndarray:
        out = np.empty(n, np.int8)
        self.lib.ref_generate_int4(n, seed, _ptr(out, _i8p))
        return out

    def pack_q4(self, b_kn: np.ndarray) -> np.ndarray:
        k, n = b_kn.shape
        out = np.empty(k * n // 8, np.uint32)
        self.lib.ref_pack_q4(_ptr(np.ascontiguousarray(b_kn, np.int8), _i8p), k, n, _ptr(out, _u32p))
        return out

    def cpu_reference(self, x: np.ndarray, b_kn: np.ndarray, scales: np.ndarray) -> np.ndarray:
        m, k = x.shape
        n = b_kn.shape[1]
        out = np.empty((m, n), np.float64)
        self.lib.ref_cpu_reference(_ptr(np.ascontiguousarray(x, np.float32), _f32p),
                                   _ptr(np.ascontiguousarray(b_kn, np.int8), _i8p),
                                   _ptr(np.ascontiguousarray(scales, np.float32), _f32p),
                                   m, n, k, _ptr(out, _f64p))
        return out


class PreparedReference:
    """A reference problem split into column shards for multi-threaded timing."""

    def __init__(self, ref: Reference, x: np.ndarray, b_kn: np.ndarray, scales: np.ndarray, parts: int) -> None:
        m, k = x.shape
        n = b_kn.shape[1]
        self.ref, self.m, self.n = ref, m, n
        self.h = ref.lib.ref_prepare(_ptr(np.ascontiguousarray(x, np.float32), _f32p),
                                     _ptr(np.ascontiguousarray(b_kn, np.int8), _i8p),
                                     _ptr(np.ascontiguousarray(scales, np.float32), _f32p), m, n, k, parts)
        if not self.h:
            raise ValueError("reference problem could not be split into the requested shards")
        self.parts = parts

    def run(self, threads: int) -> None:
        self.ref.lib.ref_run(self.h, threads)

    def result(self) -> np.ndarray:
        out = np.empty((self.m, self.n), np.float64)
        self.ref.lib.ref_gather(self.h, _ptr(out, _f64p))
        return out

    def close(self) -> None:
        if self.h:
            self.ref.lib.ref_release(self.h)
            self.h = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
