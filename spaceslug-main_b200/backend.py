"""ctypes binding of libspaceslug_b200.so, in the style of the reference host.

Mirrors python/spaceslug/backend.py of the reference: the native library is
loaded lazily with ``ctypes.CDLL`` (backend.py:53-62), each symbol's argtypes
/ restype are declared only ``if hasattr(...)`` (backend.py:64-200), the bound
symbols become capabilities (backend.py:369-400), and a non-zero return code
raises ``BackendError`` (backend.py:1689).  There is no CPU fallback: a
missing library or a failing call raises.

Host-pointer entry points take numpy arrays (float32 / int8 / uint32, C
contiguous); device entry points take raw device addresses (ints, e.g.
``tensor.data_ptr()``) and a CUDA stream handle (int, 0 = default stream).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
DEFAULT_LIBRARY = PKG / "lib" / "libspaceslug_b200.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_vp = ctypes.c_void_p
_u32 = ctypes.c_uint32

# name -> (argtypes, restype); mirrors include/runtime_abi.h
_SIGNATURES = {
    "spaceslug_vector_add": ([_f32p, _f32p, _f32p, ctypes.c_size_t], ctypes.c_int),
    "spaceslug_lora_delta": ([_f32p, _f32p, _f32p, _f32p, _u32, _u32], ctypes.c_int),
    "spaceslug_q4_pack": ([_i8p, _u32, _u32, _u32p], ctypes.c_int),
    "spaceslug_q4_pack_device": ([_vp, _u32, _u32, _vp, _vp], ctypes.c_int),
    "spaceslug_q4_dequant": ([_u32p, _f32p, _u32, _u32, _f32p], ctypes.c_int),
    "spaceslug_q4_dequant_device": ([_vp, _vp, _u32, _u32, _vp, _vp], ctypes.c_int),
    "spaceslug_q4gemm": ([_f32p, _u32p, _f32p, _f32p, _u32, _u32, _u32], ctypes.c_int),
    "spaceslug_q4gemm_lora": ([_f32p, _u32p, _f32p, _f32p, _f32p, _u32, ctypes.c_float, _f32p, _u32, _u32, _u32],
                              ctypes.c_int),
    "spaceslug_q4gemm_device": ([_vp, _vp, _vp, _vp, _vp, _u32, ctypes.c_float, _vp, _u32, _u32, _u32, _vp],
                                ctypes.c_int),
    "spaceslug_q4gemv_lora_noalloc": ([_vp, _vp, _vp, _vp, _vp, _u32, ctypes.c_float, _vp, _u32, _u32, _u32, _vp],
                                      ctypes.c_int),
    "spaceslug_q4_weights_create": ([_u32p, _f32p, _u32, _u32, _u32, _u32, ctypes.c_int, ctypes.POINTER(_vp)],
                                    ctypes.c_int),
    "spaceslug_q4_weights_create_logical": ([_i8p, _f32p, _u32, _u32, _u32, _u32, ctypes.c_int, ctypes.POINTER(_vp)],
                                            ctypes.c_int),
    "spaceslug_q4_weights_export": ([_vp, _u32p, _f32p], ctypes.c_int),
    "spaceslug_q4_weights_set_lora": ([_vp, _f32p, _f32p, _u32, ctypes.c_float], ctypes.c_int),
    "spaceslug_q4_weights_run": ([_vp, _vp, _vp, _u32, _vp], ctypes.c_int),
    "spaceslug_q4_weights_run_host": ([_vp, _f32p, _f32p, _u32], ctypes.c_int),
    "spaceslug_q4_weights_destroy": ([_vp], ctypes.c_int),
    "spaceslug_q4_set_operand_type": ([ctypes.c_int], ctypes.c_int),
    "spaceslug_q4_set_gemm_variant": ([ctypes.c_int], ctypes.c_int),
    "spaceslug_q4_set_decode_variant": ([ctypes.c_int], ctypes.c_int),
    "spaceslug_q4_device_status": ([ctypes.c_int], ctypes.c_int),
    "spaceslug_q4_debug_wait_test": ([ctypes.c_uint64, ctypes.c_int], ctypes.c_int),
    "spaceslug_q4_launch_count": ([], ctypes.c_uint64),
    "spaceslug_last_error": ([], ctypes.c_char_p),
    "spaceslug_sgemm": ([_f32p, _f32p, _f32p, _u32, _u32, _u32, _f32p], ctypes.c_int),
    "spaceslug_sgemm_device": ([_vp, _vp, _vp, _u32, _u32, _u32, _vp], ctypes.c_int),
    "spaceslug_shards_relayout": ([_vp, _vp, _u32, _u32, _u32, _u32, ctypes.c_uint64, _vp], ctypes.c_int),
    "spaceslug_q4_weights_run_strided": ([_vp, _vp, _vp, _u32, ctypes.c_uint64, _vp], ctypes.c_int),
    "spaceslug_q4_weights_set_sm_budget": ([_vp, _u32], ctypes.c_int),
    "spaceslug_q4_weights_run_push": ([_vp, _vp, _vp, _u32, ctypes.c_uint64, ctypes.POINTER(_vp), _u32, _vp],
                                      ctypes.c_int),
    "spaceslug_push_rows": ([_vp, ctypes.POINTER(_vp), _u32, _u32, _u32, ctypes.c_uint64, _u32, _vp], ctypes.c_int),
    "spaceslug_ipc_export": ([_vp, _vp, ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "spaceslug_ipc_open": ([_vp, ctypes.c_uint64, ctypes.c_int, ctypes.POINTER(_vp), ctypes.POINTER(_vp)],
                           ctypes.c_int),
    "spaceslug_ipc_close": ([_vp], ctypes.c_int),
    "spaceslug_copy_2d": ([_vp, ctypes.c_uint64, _vp, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _vp],
                          ctypes.c_int),
    "spaceslug_lora_gradients": ([_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _u32, _u32], ctypes.c_int),
    "spaceslug_lora_sgd": ([_f32p, _f32p, _f32p, _f32p, ctypes.c_float, _u32], ctypes.c_int),
    "spaceslug_lora_train_step": ([_f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_float, _u32, _u32], ctypes.c_int),
    "spaceslug_q4_weights_lora_backward": ([_vp, _vp, _vp, _u32, _vp], ctypes.c_int),
    "spaceslug_q4_weights_lora_sgd": ([_vp, ctypes.c_float, _vp], ctypes.c_int),
    "spaceslug_q4_weights_lora_adamw": ([_vp, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                         ctypes.c_float, _vp], ctypes.c_int),
    "spaceslug_q4_weights_get_lora": ([_vp, _f32p, _f32p, _f32p, _f32p], ctypes.c_int),
    "spaceslug_cq4_weights_create": ([_vp, ctypes.c_int, ctypes.POINTER(_vp)], ctypes.c_int),
    "spaceslug_cq4_matmul": ([_vp, _vp, _vp, _u32, _vp], ctypes.c_int),
    "spaceslug_cq4_matmul_host": ([_vp, _vp, _vp, _u32], ctypes.c_int),
    "spaceslug_cq4_transform_host": ([_vp, _vp, _vp, _u32], ctypes.c_int),
    "spaceslug_cq4_weights_destroy": ([_vp], ctypes.c_int),
}

# symbol -> capability name reported by capabilities()
_CAPABILITIES = {
    "spaceslug_vector_add": "vector_add",
    "spaceslug_lora_delta": "lora_delta_abi",
    "spaceslug_q4_pack": "q4_pack",
    "spaceslug_q4_dequant": "q4_dequant",
    "spaceslug_q4gemm": "q4gemm",
    "spaceslug_q4gemm_lora": "q4gemm_lora_fused",
    "spaceslug_q4gemm_device": "q4gemm_device",
    "spaceslug_q4_weights_create": "q4_weights_resident",
    "spaceslug_q4_weights_create_logical": "q4_weights_device_pack",
    "spaceslug_cq4_matmul": "cq4_quant_matmul",
    "spaceslug_lora_train_step": "lora_train_step_abi",
    "spaceslug_sgemm": "sgemm",
    "spaceslug_q4_weights_lora_backward": "lora_training",
}


class CQ4Matrix(ctypes.Structure):
    """spaceslug_cq4_matrix (include/runtime_abi.h), field for field the
    reference's CactusQuantMatrixBridge."""
    _fields_ = [("bits", ctypes.c_uint32), ("k", ctypes.c_uint32), ("n", ctypes.c_uint32),
                ("group_size", ctypes.c_uint32), ("num_groups", ctypes.c_uint32), ("flags", ctypes.c_uint32),
                ("codebook", _vp), ("input_scale", _vp), ("input_scale_recip", _vp), ("norms", _vp),
                ("packed_indices", _vp), ("left_signs", _vp), ("right_signs", _vp), ("permutation", _vp),
                ("rotation", _vp), ("expanded", _vp), ("norm_f32", _vp)]


class BackendError(RuntimeError):
    """A structured backend invocation failure."""

    def __init__(self, message: str, code: int | None = None) -> None:
        super().__init__(message)
        self.code = code


def _arr(a, dtype) -> np.ndarray:
    out = np.ascontiguousarray(a, dtype=dtype)
    return out


def _p(a: np.ndarray, typ):
    return a.ctypes.data_as(typ)


class BackendSession:
    """Session over the native library (no CPU fallback)."""

    def __init__(self, library_path: str | Path | None = None) -> None:
        self._library_path = Path(library_path) if library_path else DEFAULT_LIBRARY
        self._library: ctypes.CDLL | None = None

    # ------------------------------------------------------------ loading --
    def _native(self) -> ctypes.CDLL:
        if self._library is None:
            if not self._library_path.is_file():
                raise BackendError(f"runtime shared library is missing: {self._library_path}")
            try:
                lib = ctypes.CDLL(str(self._library_path))
            except OSError as exc:
                raise BackendError(f"failed to load {self._library_path}: {exc}") from exc
            for name, (argtypes, restype) in _SIGNATURES.items():
                if hasattr(lib, name):
                    fn = getattr(lib, name)
                    fn.argtypes = argtypes
                    fn.restype = restype
            self._library = lib
        return self._library

    @property
    def library_path(self) -> Path:
        return self._library_path

    def capabilities(self) -> list[str]:
        lib = self._native()
        return [cap for sym, cap in _CAPABILITIES.items() if hasattr(lib, sym)]

    def exported_symbols(self) -> list[str]:
        lib = self._native()
        return [s for s in _SIGNATURES if hasattr(lib, s)]

    def _call(self, name: str, *args) -> int:
        lib = self._native()
        if not hasattr(lib, name):
            raise BackendError(f"native symbol {name} is unavailable")
        code = getattr(lib, name)(*args)
        if code != 0:
            msg = lib.spaceslug_last_error().decode(errors="replace") if hasattr(lib, "spaceslug_last_error") else ""
            raise BackendError(f"native {name} returned {code}: {msg}", code)
        return code

    def raw(self, name: str):
        """The bound ctypes function (returns codes instead of raising)."""
        return getattr(self._native(), name)

    # -------------------------------------------------------------- ops --
    def vector_add(self, left, right) -> np.ndarray:
        l, r = _arr(left, np.float32), _arr(right, np.float32)
        if l.shape != r.shape:
            raise BackendError("tensor shape mismatch")
        out = np.empty_like(l)
        self._call("spaceslug_vector_add", _p(l, _f32p), _p(r, _f32p), _p(out, _f32p), l.size)
        return out

    def lora_delta(self, x, a, b, m: int, rank: int) -> np.ndarray:
        """Legacy Y[M,64] = X A B (reference backend.py:1678-1690)."""
        xx, aa, bb = _arr(x, np.float32), _arr(a, np.float32), _arr(b, np.float32)
        y = np.empty(m * 64, np.float32)
        self._call("spaceslug_lora_delta", _p(xx, _f32p), _p(aa, _f32p), _p(bb, _f32p), _p(y, _f32p), m, rank)
        return y

    def q4_pack(self, w_kn) -> np.ndarray:
        w = _arr(w_kn, np.int8)
        k, n = w.shape
        out = np.empty(k * n // 8, np.uint32)
        self._call("spaceslug_q4_pack", _p(w, _i8p), k, n, _p(out, _u32p))
        return out

    def q4_dequant(self, packed, scales, k: int, n: int) -> np.ndarray:
        pk, sc = _arr(packed, np.uint32), _arr(scales, np.float32)
        out = np.empty((k, n), np.float32)
        self._call("spaceslug_q4_dequant", _p(pk, _u32p), _p(sc, _f32p), k, n, _p(out, _f32p))
        return out

    def q4gemm(self, x, packed, scales, n: int, lora_a=None, lora_b=None, alpha: float = 0.0) -> np.ndarray:
        xx, pk, sc = _arr(x, np.float32), _arr(packed, np.uint32), _arr(scales, np.float32)
        m, k = xx.shape
        y = np.empty((m, n), np.float32)
        if lora_a is None:
            self._call("spaceslug_q4gemm", _p(xx, _f32p), _p(pk, _u32p), _p(sc, _f32p), _p(y, _f32p), m, n, k)
        else:
            la, lb = _arr(lora_a, np.float32), _arr(lora_b, np.float32)
            rank = la.shape[1]
            self._call("spaceslug_q4gemm_lora", _p(xx, _f32p), _p(pk, _u32p), _p(sc, _f32p), _p(la, _f32p),
                       _p(lb, _f32p), rank, float(alpha), _p(y, _f32p), m, n, k)
        return y

    def q4gemm_device(self, x: int, packed: int, scales: int, y: int, m: int, n: int, k: int, stream: int = 0,
                      lora_a: int = 0, lora_b: int = 0, rank: int = 0, alpha: float = 0.0) -> None:
        self._call("spaceslug_q4gemm_device", x, packed, scales, lora_a or None, lora_b or None, rank, float(alpha),
                   y, m, n, k, stream or None)

    def q4_dequant_device(self, packed: int, scales: int, k: int, n: int, out: int, stream: int = 0) -> None:
        self._call("spaceslug_q4_dequant_device", packed, scales, k, n, out, stream or None)

    def q4_pack_device(self, w_kn: int, k: int, n: int, packed: int, stream: int = 0) -> None:
        self._call("spaceslug_q4_pack_device", w_kn, k, n, packed, stream or None)

    def set_operand_type(self, kind: str) -> str:
        prev = self.raw("spaceslug_q4_set_operand_type")({"f16": 0, "bf16": 1}[kind])
        return {0: "f16", 1: "bf16"}.get(prev, "?")

    def set_gemm_variant(self, variant: str) -> str:
        names = {"auto": 0, "single": 1, "pair": 2, "single256": 3}
        prev = self.raw("spaceslug_q4_set_gemm_variant")(names[variant])
        return {v: k for k, v in names.items()}.get(prev, "?")

    def set_decode_variant(self, variant: str) -> str:
        names = {"auto": 0, "gemv": 1, "mma": 2, "tile": 3, "imma": 4}
        prev = self.raw("spaceslug_q4_set_decode_variant")(names[variant])
        return {v: k for k, v in names.items()}.get(prev, "?")

    def device_status(self, device: int = 0) -> int:
        return int(self.raw("spaceslug_q4_device_status")(device))

    def launch_count(self) -> int:
        return int(self.raw("spaceslug_q4_launch_count")())

    def weights(self, packed, scales, k: int, n: int, col_begin: int = 0, col_end: int | None = None,
                device: int = 0) -> "Q4Weights":
        return Q4Weights(self, packed, scales, k, n, col_begin, n if col_end is None else col_end, device)

    def sgemm(self, a, b) -> np.ndarray:
        """The reference's spaceslug_sgemm: fp32 C = A B (M, N % 64, K % 32), host arrays."""
        aa, bb = _arr(a, np.float32), _arr(b, np.float32)
        m, k = aa.shape
        n = bb.shape[1]
        c = np.empty((m, n), np.float32)
        err = ctypes.c_float(-1.0)
        self._call("spaceslug_sgemm", _p(aa, _f32p), _p(bb, _f32p), _p(c, _f32p), m, n, k, ctypes.byref(err))
        return c

    def sgemm_device(self, a: int, b: int, c: int, m: int, n: int, k: int, stream: int = 0) -> None:
        self._call("spaceslug_sgemm_device", a, b, c, m, n, k, stream or None)

    def shards_relayout(self, gathered: int, y: int, parts: int, rows: int, width: int, n_total: int, ld_y: int,
                        stream: int = 0) -> None:
        """Device pointers: rank-major gathered shards [parts][rows][width] -> Y rows [rows][ld_y]."""
        self._call("spaceslug_shards_relayout", gathered, y, parts, rows, width, n_total, ld_y, stream or None)

    def ipc_export(self, ptr: int) -> tuple[bytes, int]:
        """(64-byte CUDA IPC handle of the allocation holding ptr, byte offset of ptr in it)."""
        h = ctypes.create_string_buffer(64)
        off = ctypes.c_uint64()
        self._call("spaceslug_ipc_export", ptr, h, ctypes.byref(off))
        return h.raw, int(off.value)

    def ipc_open(self, handle: bytes, offset: int, device: int) -> tuple[int, int]:
        """Maps a peer's allocation on `device`: (pointer, base to pass to ipc_close)."""
        if len(handle) != 64:
            raise ValueError("an IPC handle has 64 bytes")
        ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
        self._call("spaceslug_ipc_open", ctypes.create_string_buffer(handle, 64), offset, device,
                   ctypes.byref(ptr), ctypes.byref(base))
        return int(ptr.value), int(base.value)

    def ipc_close(self, base: int) -> None:
        self._call("spaceslug_ipc_close", base)

    def push_rows(self, src: int, peer_dst: list[int], rows: int, width: int, ld: int, ctas: int,
                  stream: int = 0) -> None:
        """Device pointers: rows x width floats (pitch ld) from src to the same offsets in each peer buffer."""
        arr = (_vp * max(1, len(peer_dst)))(*peer_dst)
        self._call("spaceslug_push_rows", src, arr, len(peer_dst), rows, width, ld, ctas, stream or None)

    def copy_2d(self, dst: int, dpitch: int, src: int, spitch: int, width_bytes: int, rows: int,
                stream: int = 0) -> None:
        self._call("spaceslug_copy_2d", dst, dpitch, src, spitch, width_bytes, rows, stream or None)

    def lora_gradients(self, x, dy, a, b, m: int, rank: int):
        """The reference's hidden-64 spaceslug_lora_gradients: (dA [64, r], dB [r, 64])."""
        xx, yy, aa, bb = (_arr(v, np.float32) for v in (x, dy, a, b))
        da, db = np.empty(64 * rank, np.float32), np.empty(rank * 64, np.float32)
        self._call("spaceslug_lora_gradients", _p(xx, _f32p), _p(yy, _f32p), _p(aa, _f32p), _p(bb, _f32p),
                   _p(da, _f32p), _p(db, _f32p), m, rank)
        return da.reshape(64, rank), db.reshape(rank, 64)

    def lora_sgd(self, a, b, da, db, learning_rate: float, rank: int):
        aa, bb = _arr(a, np.float32).copy(), _arr(b, np.float32).copy()
        ga, gb = _arr(da, np.float32), _arr(db, np.float32)
        self._call("spaceslug_lora_sgd", _p(aa, _f32p), _p(bb, _f32p), _p(ga, _f32p), _p(gb, _f32p),
                   float(learning_rate), rank)
        return aa, bb

    def lora_train_step(self, x, dy, a, b, learning_rate: float, m: int, rank: int):
        """(y [m, 64], new A, new B) of the reference's spaceslug_lora_train_step."""
        xx, yy = _arr(x, np.float32), _arr(dy, np.float32)
        aa, bb = _arr(a, np.float32).copy(), _arr(b, np.float32).copy()
        y = np.empty(m * 64, np.float32)
        self._call("spaceslug_lora_train_step", _p(xx, _f32p), _p(yy, _f32p), _p(aa, _f32p), _p(bb, _f32p),
                   _p(y, _f32p), float(learning_rate), m, rank)
        return y.reshape(m, 64), aa, bb

    def cq4_weights(self, *, k: int, n: int, group_size: int, num_groups: int, flags: int, codebook, norms, packed,
                    input_scale=None, input_scale_recip=None, left_signs=None, right_signs=None, permutation=None,
                    rotation=None, bits: int = 4, device: int = 0) -> "CQ4Weights":
        """A CQ4 matrix (fp16 arrays as uint16 bits) resident on `device`."""
        return CQ4Weights(self, dict(bits=bits, k=k, n=n, group_size=group_size, num_groups=num_groups, flags=flags,
                                     codebook=codebook, input_scale=input_scale, input_scale_recip=input_scale_recip,
                                     norms=norms, packed=packed, left_signs=left_signs, right_signs=right_signs,
                                     permutation=permutation, rotation=rotation), device)

    def weights_logical(self, w_kn, scales, k: int, n: int, col_begin: int = 0, col_end: int | None = None,
                        device: int = 0) -> "Q4Weights":
        """Handle from the logical int4 matrix w_kn [k, n] (int8 in [-8, 7]),
        packed on the device during the upload."""
        return Q4Weights(self, None, scales, k, n, col_begin, n if col_end is None else col_end, device, w_kn=w_kn)


class Q4Weights:
    """Device-resident int4 weights (a handle of the C-ABI)."""

    def __init__(self, session: BackendSession, packed, scales, k: int, n: int, col_begin: int, col_end: int,
                 device: int, w_kn=None) -> None:
        self.session = session
        sc = _arr(scales, np.float32)
        self.k, self.n_total, self.col_begin, self.col_end = k, n, col_begin, col_end
        self.n = col_end - col_begin
        h = _vp()
        if w_kn is None:
            pk = _arr(packed, np.uint32)
            session._call("spaceslug_q4_weights_create", _p(pk, _u32p), _p(sc, _f32p), k, n, col_begin, col_end,
                          device, ctypes.byref(h))
        else:
            wk = _arr(w_kn, np.int8)
            session._call("spaceslug_q4_weights_create_logical", _p(wk, _i8p), _p(sc, _f32p), k, n, col_begin,
                          col_end, device, ctypes.byref(h))
        self.handle = h

    def export(self) -> tuple[np.ndarray, np.ndarray]:
        """The handle's packed words [n, k/8] and scales [n, k/32] (its columns)."""
        pk = np.empty((self.n, self.k // 8), np.uint32)
        sc = np.empty((self.n, self.k // 32), np.float32)
        self.session._call("spaceslug_q4_weights_export", self.handle, _p(pk, _u32p), _p(sc, _f32p))
        return pk, sc

    def set_lora(self, lora_a, lora_b, alpha: float) -> None:
        if lora_a is None:
            self.session._call("spaceslug_q4_weights_set_lora", self.handle, None, None, 0, 0.0)
            return
        la, lb = _arr(lora_a, np.float32), _arr(lora_b, np.float32)
        self.session._call("spaceslug_q4_weights_set_lora", self.handle, _p(la, _f32p), _p(lb, _f32p),
                           la.shape[1], float(alpha))

    def run(self, x: int, y: int, m: int, stream: int = 0) -> None:
        self.session._call("spaceslug_q4_weights_run", self.handle, x, y, m, stream or None)

    def set_sm_budget(self, sms: int) -> None:
        """At most `sms` SMs for this handle's GEMM launches (0: all)."""
        self.session._call("spaceslug_q4_weights_set_sm_budget", self.handle, sms)

    def run_push(self, x: int, y: int, m: int, ld_y: int, peer_y: list[int], stream: int = 0) -> None:
        """run_strided that also stores Y's rows to the same places in the peers' buffers."""
        arr = (_vp * max(1, len(peer_y)))(*peer_y)
        self.session._call("spaceslug_q4_weights_run_push", self.handle, x, y, m, ld_y, arr, len(peer_y),
                           stream or None)

    def run_strided(self, x: int, y: int, m: int, ld_y: int, stream: int = 0) -> None:
        """Y rows with pitch ld_y floats (this handle's columns only)."""
        self.session._call("spaceslug_q4_weights_run_strided", self.handle, x, y, m, ld_y, stream or None)

    # ---- LoRA training (device pointers, asynchronous) ----
    def lora_backward(self, x: int, dy: int, m: int, stream: int = 0) -> None:
        self.session._call("spaceslug_q4_weights_lora_backward", self.handle, x, dy, m, stream or None)

    def lora_sgd(self, learning_rate: float, stream: int = 0) -> None:
        self.session._call("spaceslug_q4_weights_lora_sgd", self.handle, float(learning_rate), stream or None)

    def lora_adamw(self, learning_rate: float, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
                   weight_decay: float = 0.0, stream: int = 0) -> None:
        self.session._call("spaceslug_q4_weights_lora_adamw", self.handle, float(learning_rate), float(beta1),
                           float(beta2), float(eps), float(weight_decay), stream or None)

    def get_lora(self, rank: int, grads: bool = False):
        """(A [k, r], B [r, n]) and, with grads, (dA, dB) as well."""
        a = np.empty((self.k, rank), np.float32)
        b = np.empty((rank, self.n), np.float32)
        da = np.empty_like(a) if grads else None
        db = np.empty_like(b) if grads else None
        self.session._call("spaceslug_q4_weights_get_lora", self.handle, _p(a, _f32p), _p(b, _f32p),
                           None if da is None else _p(da, _f32p), None if db is None else _p(db, _f32p))
        return (a, b, da, db) if grads else (a, b)

    def run_host(self, x) -> np.ndarray:
        xx = _arr(x, np.float32)
        m = xx.shape[0]
        y = np.empty((m, self.n), np.float32)
        self.session._call("spaceslug_q4_weights_run_host", self.handle, _p(xx, _f32p), _p(y, _f32p), m)
        return y

    def close(self) -> None:
        if self.handle:
            self.session._call("spaceslug_q4_weights_destroy", self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class CQ4Weights:
    """Device-resident CQ4 matrix (a handle of the C-ABI)."""

    def __init__(self, session: BackendSession, d: dict, device: int) -> None:
        self.session = session
        self.k, self.n = d["k"], d["n"]
        keep = {
            "codebook": _arr(d["codebook"], np.uint16), "norms": _arr(d["norms"], np.uint16),
            "packed_indices": _arr(d["packed"], np.uint8),
            "input_scale": None if d["input_scale"] is None else _arr(d["input_scale"], np.uint16),
            "input_scale_recip": None if d["input_scale_recip"] is None else _arr(d["input_scale_recip"], np.uint16),
            "left_signs": None if d["left_signs"] is None else _arr(d["left_signs"], np.int8),
            "right_signs": None if d["right_signs"] is None else _arr(d["right_signs"], np.int8),
            "permutation": None if d["permutation"] is None else _arr(d["permutation"], np.uint32),
            "rotation": None if d["rotation"] is None else _arr(d["rotation"], np.uint16),
        }
        m = CQ4Matrix(d["bits"], d["k"], d["n"], d["group_size"], d["num_groups"], d["flags"])
        for name, arr in keep.items():
            setattr(m, name, None if arr is None else arr.ctypes.data)
        h = _vp()
        session._call("spaceslug_cq4_weights_create", ctypes.addressof(m), device, ctypes.byref(h))
        self.handle = h

    def matmul_host(self, a_bits) -> np.ndarray:
        """C (fp16 bits [m, n]) = cactus_quant_matmul(W, A) for A fp16 bits [m, k]."""
        a = _arr(a_bits, np.uint16).reshape(-1, self.k)
        c = np.empty((a.shape[0], self.n), np.uint16)
        self.session._call("spaceslug_cq4_matmul_host", self.handle, a.ctypes.data, c.ctypes.data, a.shape[0])
        return c

    def matmul(self, a_dev: int, c_dev: int, m: int, stream: int = 0) -> None:
        self.session._call("spaceslug_cq4_matmul", self.handle, a_dev, c_dev, m, stream or None)

    def transform_host(self, a_bits) -> np.ndarray:
        a = _arr(a_bits, np.uint16).reshape(-1, self.k)
        out = np.empty_like(a)
        self.session._call("spaceslug_cq4_transform_host", self.handle, a.ctypes.data, out.ctypes.data, a.shape[0])
        return out

    def close(self) -> None:
        if self.handle:
            self.session._call("spaceslug_cq4_weights_destroy", self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
