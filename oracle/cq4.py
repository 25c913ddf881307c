"""CQ4 (Cactus-Quants) oracle -- TEST INFRASTRUCTURE ONLY.

Nothing in the shipped library imports this module.  It holds:

* ``make_fixture`` -- the reference's own test fixtures
  (vulkan-runtime/tests/test_cq4.cpp:362-440 ``run_fixture``), generated with
  the same LCG streams (m6c1_common.h:33-42 ``gen_f32``, test_cq4.cpp:72-91
  ``gen_permutation``/``gen_signs``, :395-402 indices) and packed with the same
  layouts (:93-130 ``pack_4bit_lsb``/``pack_interleaved_4row``, :135-145
  ``layout_norms``);
* ``CQ4Reference`` -- ctypes access to the reference's own CPU oracle
  (``cactus_quant_matmul``, vulkan-runtime/src/cactus/cactus_x86.cpp:384-397,
  and ``transform_hadamard_group`` :85-110), built from the reference sources
  by oracle/Makefile into the git-ignored oracle/_ref/libcq4ref.so;
* ``quant_matmul`` -- a numpy restatement of cactus_quant_matmul (fp32 ops in
  the reference's order, pinned bit-exactly to the reference library by
  tests/test_cq4_cpu.py);
* ``transform_double`` -- the double-precision activation transform of the
  reference test (test_cq4.cpp:147-163 ``fwht_d`` and its transform checks).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

import numpy as np

FLAG_ORTHOGONAL = 1 << 2        # CACTUS_BRIDGE_QUANT_FLAG_ORTHOGONAL (cactus_x86_bridge.h)
FLAG_INTERLEAVED_4ROW = 1 << 3  # CACTUS_BRIDGE_QUANT_FLAG_INTERLEAVED_4ROW

_HERE = Path(__file__).resolve().parent
_LIB = _HERE / "_ref" / "libcq4ref.so"

_A, _C = np.uint32(1664525), np.uint32(1013904223)


def _lcg(n: int, seed: int) -> np.ndarray:
    """States s_1..s_n of s <- s * 1664525 + 1013904223 (mod 2^32)."""
    out = np.empty(n, np.uint32)
    s = np.uint32(seed)
    with np.errstate(over="ignore"):
        for i in range(n):
            s = np.uint32(s * _A + _C)
            out[i] = s
    return out


def gen_f32(n: int, seed: int, lo: float, hi: float) -> np.ndarray:
    """m6c1::gen_f32: lo + u * (hi - lo), u = (s >> 8) / 2^24, fp32 arithmetic."""
    u = (_lcg(n, seed) >> np.uint32(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    return (np.float32(lo) + u * np.float32(np.float32(hi) - np.float32(lo))).astype(np.float32)


def to_fp16_bits(f: np.ndarray) -> np.ndarray:
    return np.asarray(f, np.float32).astype(np.float16).view(np.uint16)


def f16(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)


def gen_signs(n: int, seed: int) -> np.ndarray:
    st = _lcg(n, seed)
    return np.where(((st >> np.uint32(8)) & np.uint32(1)) != 0, 1, -1).astype(np.int8)


def gen_permutation(n: int, seed: int) -> np.ndarray:
    p = np.arange(n, dtype=np.uint32)
    s = np.uint32(seed)
    with np.errstate(over="ignore"):
        for i in range(n, 1, -1):
            s = np.uint32(s * _A + _C)
            j = int((s >> np.uint32(8)) % np.uint32(i))
            p[i - 1], p[j] = p[j], p[i - 1]
    return p


def pack_4bit_lsb(idx_flat: np.ndarray) -> np.ndarray:
    idx = np.asarray(idx_flat, np.uint32) & 0xF
    if idx.size % 2:
        idx = np.concatenate([idx, np.zeros(1, np.uint32)])
    return (idx[0::2] | (idx[1::2] << 4)).astype(np.uint8)


def pack_interleaved_4row(idx: np.ndarray, n: int, gs: int, ng: int) -> np.ndarray:
    """idx [n][ng*gs] -> panels of 4 rows per group: byte chunk*16 + r*4 + (sub & 3),
    low nibble for sub < 4, high nibble otherwise."""
    pgb = (gs * 4 + 7) // 8
    panel_bytes = 4 * pgb
    out = np.zeros((n // 4) * ng * panel_bytes, np.uint8)
    k = np.arange(gs)
    chunk, sub = k // 8, k & 7
    off = chunk * 16 + (sub & 3)
    hi = (sub & 4) != 0
    for panel in range(n // 4):
        for g in range(ng):
            base = (panel * ng + g) * panel_bytes
            for r in range(4):
                vals = np.asarray(idx[panel * 4 + r, g * gs:(g + 1) * gs], np.uint32) & 0xF
                pos = base + off + r * 4
                out[pos[~hi]] |= vals[~hi].astype(np.uint8)
                out[pos[hi]] |= (vals[hi] << 4).astype(np.uint8)
    return out


def layout_norms(logical: np.ndarray, n: int, ng: int, interleaved: bool) -> np.ndarray:
    if not interleaved:
        return logical.copy()
    out = np.empty_like(logical)
    for nn in range(n):
        for g in range(ng):
            out[((nn // 4) * ng + g) * 4 + (nn & 3)] = logical[nn * ng + g]
    return out


@dataclass
class Fixture:
    name: str
    M: int
    K: int
    N: int
    gs: int
    ng: int
    flags: int
    codebook: np.ndarray        # uint16 [16] fp16 bits
    input_scale: np.ndarray | None        # uint16 [K]
    input_scale_recip: np.ndarray | None  # uint16 [K]
    norms: np.ndarray           # uint16, stored layout
    packed: np.ndarray          # uint8
    left: np.ndarray | None     # int8 [gs]
    right: np.ndarray | None
    perm: np.ndarray | None     # uint32 [gs]
    rotation: np.ndarray | None # uint16 [K*K]
    a: np.ndarray               # uint16 [M*K]
    idx: np.ndarray             # uint32 [N][K] logical indices
    bits: int = 4

    @property
    def orthogonal(self) -> bool:
        return bool(self.flags & FLAG_ORTHOGONAL)

    @property
    def interleaved(self) -> bool:
        return bool(self.flags & FLAG_INTERLEAVED_4ROW)

    def recip_f32(self) -> np.ndarray:
        """input_scale_recip1 per element (cactus_x86.cpp:73-77)."""
        if self.input_scale_recip is not None:
            return f16(self.input_scale_recip)
        if self.input_scale is not None:
            return (np.float32(1.0) / f16(self.input_scale)).astype(np.float32)
        return np.ones(self.K, np.float32)


# The reference test's five fixtures (test_cq4.cpp:483-487):
# name, M, N, gs, ng, interleaved, signs+perm, input_scale, orthogonal
REFERENCE_FIXTURES = [
    ("cq4_interleaved", 64, 64, 128, 1, True, False, False, False),
    ("cq4_hadamard_signs", 64, 64, 128, 1, False, True, True, False),
    ("cq4_orthogonal", 64, 64, 64, 1, False, False, False, True),
    ("cq4_interleaved_multigroup_m1", 1, 64, 128, 4, True, False, False, False),
    ("cq4_interleaved_m1_n512", 1, 512, 128, 4, True, False, False, False),
]


def make_fixture(name: str, M: int, N: int, gs: int, ng: int, interleaved: bool, signs_perm: bool,
                 input_scale: bool, orthogonal: bool) -> Fixture:
    K = gs * ng
    seed = 0x0C170000 if orthogonal else 0x0C170100
    codebook = to_fp16_bits(gen_f32(16, seed + 1, -1.0, 1.0))
    norms = to_fp16_bits(gen_f32(N if orthogonal else N * ng, seed + 2, 0.5, 1.5))
    norms_stored = layout_norms(norms, N, ng, interleaved and not orthogonal)
    recip = scale = None
    if orthogonal or not input_scale:
        recip = to_fp16_bits(gen_f32(K, seed + 3, 0.5, 1.5))
    else:
        scale = to_fp16_bits(gen_f32(K, seed + 3, 0.5, 1.5))
    left = right = perm = None
    if signs_perm:
        left, right, perm = gen_signs(gs, seed + 4), gen_signs(gs, seed + 5), gen_permutation(gs, seed + 6)
    idx = ((_lcg(N * K, seed + 7) >> np.uint32(8)) % np.uint32(16)).astype(np.uint32).reshape(N, K)
    packed = pack_interleaved_4row(idx, N, gs, ng) if interleaved else pack_4bit_lsb(idx.reshape(-1))
    rotation = to_fp16_bits(gen_f32(K * K, seed + 8, -0.5, 0.5)) if orthogonal else None
    a = to_fp16_bits(gen_f32(M * K, seed + 9, -1.0, 1.0))
    flags = (FLAG_INTERLEAVED_4ROW if interleaved else 0) | (FLAG_ORTHOGONAL if orthogonal else 0)
    return Fixture(name, M, K, N, gs, ng, flags, codebook, scale, recip, norms_stored, packed, left, right, perm,
                   rotation, a, idx)


def random_fixture(M: int, N: int, gs: int, ng: int, interleaved: bool, signs_perm: bool, orthogonal: bool,
                   seed: int) -> Fixture:
    """Larger fixtures with numpy's generator (same construction as make_fixture)."""
    rng = np.random.default_rng(seed)
    K = gs * ng
    codebook = to_fp16_bits(rng.uniform(-1, 1, 16).astype(np.float32))
    norms = to_fp16_bits(rng.uniform(0.5, 1.5, N if orthogonal else N * ng).astype(np.float32))
    norms_stored = layout_norms(norms, N, ng, interleaved and not orthogonal)
    recip = to_fp16_bits(rng.uniform(0.5, 1.5, K).astype(np.float32))
    left = right = perm = None
    if signs_perm:
        left = rng.choice(np.array([-1, 1], np.int8), gs)
        right = rng.choice(np.array([-1, 1], np.int8), gs)
        perm = rng.permutation(gs).astype(np.uint32)
    idx = rng.integers(0, 16, (N, K), dtype=np.uint32)
    packed = pack_interleaved_4row(idx, N, gs, ng) if interleaved else pack_4bit_lsb(idx.reshape(-1))
    rotation = to_fp16_bits(rng.uniform(-0.5, 0.5, K * K).astype(np.float32) / np.float32(np.sqrt(K / 64))) \
        if orthogonal else None
    a = to_fp16_bits(rng.uniform(-1, 1, M * K).astype(np.float32))
    flags = (FLAG_INTERLEAVED_4ROW if interleaved else 0) | (FLAG_ORTHOGONAL if orthogonal else 0)
    return Fixture(f"random_{M}x{N}x{K}", M, K, N, gs, ng, flags, codebook, None, recip, norms_stored, packed, left,
                   right, perm, rotation, a, idx)


# ------------------------------------------------------- numpy restatement --
def _norm(fx: Fixture, n: int, g: int) -> np.float32:
    nb = fx.norms
    if fx.orthogonal:
        i = (n // 4) * 4 + (n & 3) if fx.interleaved else n
    elif fx.interleaved:
        i = ((n // 4) * fx.ng + g) * 4 + (n & 3)
    else:
        i = n * fx.ng + g
    return f16(nb[i:i + 1])[0]


def transform_hadamard(fx: Fixture) -> np.ndarray:
    """Code-basis activations in fp32, in the reference's operation order
    (cactus_x86.cpp:85-110 with fwht_normalized :56-69)."""
    a = f16(fx.a).reshape(fx.M, fx.K)
    recip = fx.recip_f32()
    gs = fx.gs
    inv = np.float32(1.0) / np.sqrt(np.float32(gs), dtype=np.float32)
    out = np.empty((fx.M, fx.K), np.float32)
    for g in range(fx.ng):
        sl = slice(g * gs, (g + 1) * gs)
        work = (a[:, sl] * recip[sl]).astype(np.float32)
        if fx.left is not None:
            work = (work * fx.left.astype(np.float32)).astype(np.float32)
        h = 1
        while h < gs:
            w = work.reshape(fx.M, gs // (2 * h), 2, h)
            x, y = w[:, :, 0, :].copy(), w[:, :, 1, :].copy()
            w[:, :, 0, :] = x + y
            w[:, :, 1, :] = x - y
            work = w.reshape(fx.M, gs)
            h <<= 1
        work = (work * inv).astype(np.float32)
        if fx.right is not None:
            work = (work * fx.right.astype(np.float32)).astype(np.float32)
        if fx.perm is not None:
            work = work[:, fx.perm]
        out[:, sl] = work
    return out


def transform_orthogonal_f32(fx: Fixture) -> np.ndarray:
    a = f16(fx.a).reshape(fx.M, fx.K)
    recip = fx.recip_f32()
    rot = f16(fx.rotation).reshape(fx.K, fx.K)
    ar = np.zeros((fx.M, fx.K), np.float32)
    for k in range(fx.K):
        av = (a[:, k] * recip[k]).astype(np.float32)
        ar = (ar + (av[:, None] * rot[k][None, :]).astype(np.float32)).astype(np.float32)
    return ar


def quant_matmul(fx: Fixture) -> np.ndarray:
    """cactus_quant_matmul (cactus_x86.cpp:133-235): fp32 accumulation in the
    reference's order, fp16 result bits [M][N]."""
    cb = f16(fx.codebook)
    w_cb = cb[fx.idx]  # [N][K] codebook values
    if fx.orthogonal:
        ar = transform_orthogonal_f32(fx)
        acc = np.zeros((fx.M, fx.N), np.float32)
        for i in range(fx.K):
            acc = (acc + (w_cb[:, i][None, :] * ar[:, i][:, None]).astype(np.float32)).astype(np.float32)
        norm = np.array([_norm(fx, n, 0) for n in range(fx.N)], np.float32)
        return (acc * norm).astype(np.float32).astype(np.float16).view(np.uint16).reshape(-1)
    basis = transform_hadamard(fx)
    norms = np.array([[_norm(fx, n, g) for g in range(fx.ng)] for n in range(fx.N)], np.float32)  # [N][ng]
    acc = np.zeros((fx.M, fx.N), np.float32)
    for g in range(fx.ng):
        for kk in range(fx.gs):
            k = g * fx.gs + kk
            t = (basis[:, k][:, None] * norms[:, g][None, :]).astype(np.float32)
            acc = (acc + (t * w_cb[:, k][None, :]).astype(np.float32)).astype(np.float32)
    return acc.astype(np.float16).view(np.uint16).reshape(-1)


def transform_double(fx: Fixture) -> np.ndarray:
    """The reference test's double-precision transform (test_cq4.cpp
    cpu_transform_hadamard / cpu_transform_orthogonal), fp64 [M][K]."""
    a = f16(fx.a).reshape(fx.M, fx.K).astype(np.float64)
    recip = fx.recip_f32().astype(np.float64)
    if fx.orthogonal:
        return (a * recip) @ f16(fx.rotation).reshape(fx.K, fx.K).astype(np.float64)
    gs = fx.gs
    out = np.empty_like(a)
    for g in range(fx.ng):
        sl = slice(g * gs, (g + 1) * gs)
        w = a[:, sl] * recip[sl]
        if fx.left is not None:
            w = w * fx.left
        h = 1
        while h < gs:
            v = w.reshape(fx.M, gs // (2 * h), 2, h)
            x, y = v[:, :, 0, :].copy(), v[:, :, 1, :].copy()
            v[:, :, 0, :] = x + y
            v[:, :, 1, :] = x - y
            w = v.reshape(fx.M, gs)
            h <<= 1
        w = w / np.sqrt(gs)
        if fx.right is not None:
            w = w * fx.right
        if fx.perm is not None:
            w = w[:, fx.perm]
        out[:, sl] = w
    return out


def compare_fp16(got_bits: np.ndarray, ref_bits: np.ndarray, abs_tol: float, rel_tol: float) -> dict:
    """The reference's pass criterion (m6c1_common.h:286-304): an element fails
    when its error exceeds BOTH abs_tol and rel_tol * |ref|."""
    g = f16(np.asarray(got_bits).reshape(-1)).astype(np.float64)
    r = f16(np.asarray(ref_bits).reshape(-1)).astype(np.float64)
    err = np.abs(g - r)
    bad = (err > abs_tol) & (err > rel_tol * np.abs(r))
    return {"ok": bool(not bad.any() and np.all(np.isfinite(g))), "max_abs": float(err.max(initial=0.0)),
            "max_rel": float((err / np.maximum(1.0, np.abs(r))).max(initial=0.0)), "bad": int(bad.sum())}


# ------------------------------------------------------ reference library --
class CQ4Reference:
    @staticmethod
    def available() -> bool:
        return _LIB.is_file()

    def __init__(self) -> None:
        lib = ctypes.CDLL(str(_LIB))
        vp = ctypes.c_void_p
        u32 = ctypes.c_uint32
        lib.ref_cq4_quant_matmul.argtypes = [u32] * 6 + [vp] * 10 + [u32, vp]
        lib.ref_cq4_quant_matmul.restype = None
        lib.ref_cq4_transform_hadamard_row.argtypes = [u32, u32, u32] + [vp] * 7
        lib.ref_cq4_transform_hadamard_row.restype = None
        self.lib = lib

    @staticmethod
    def _p(a):
        return None if a is None else np.ascontiguousarray(a).ctypes.data_as(ctypes.c_void_p)

    def quant_matmul(self, fx: Fixture) -> np.ndarray:
        c = np.zeros(fx.M * fx.N, np.uint16)
        keep = [np.ascontiguousarray(x) if x is not None else None for x in
                (fx.codebook, fx.input_scale, fx.input_scale_recip, fx.norms, fx.packed, fx.left, fx.right, fx.perm,
                 fx.rotation, fx.a)]
        p = [self._p(x) for x in keep]
        self.lib.ref_cq4_quant_matmul(fx.bits, fx.K, fx.N, fx.gs, fx.ng, fx.flags, *p[:9], p[9], fx.M,
                                      c.ctypes.data_as(ctypes.c_void_p))
        return c

    def transform_hadamard(self, fx: Fixture) -> np.ndarray:
        out = np.zeros((fx.M, fx.K), np.float32)
        keep = [np.ascontiguousarray(x) if x is not None else None for x in
                (fx.input_scale, fx.input_scale_recip, fx.left, fx.right, fx.perm)]
        p = [self._p(x) for x in keep]
        a = np.ascontiguousarray(fx.a.reshape(fx.M, fx.K))
        for m in range(fx.M):
            self.lib.ref_cq4_transform_hadamard_row(fx.K, fx.gs, fx.ng, *p, a[m].ctypes.data_as(ctypes.c_void_p),
                                                    out[m].ctypes.data_as(ctypes.c_void_p))
        return out
