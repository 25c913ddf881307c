"""Seeded synthetic inputs for the int4 GEMM/GEMV + LoRA configurations.

The uniform and int4 streams are the reference's own LCG generators
(vulkan-runtime/tests/test_q4gemm.cpp:58-80, s = s*1664525 + 1013904223),
reproduced bit-exactly but vectorised with LCG jump-ahead so the 235 M nibbles
of the largest configuration take seconds.  Normal variates (the benchmark
configurations ask for N(0, sigma^2) activations and LoRA factors, which the
reference generators do not provide) are Box-Muller transforms of pairs of
that LCG stream, computed in float64 and rounded to float32.

Packing to the reference layout (q4gemm.comp:7-19) is vectorised here too, so
this module only needs numpy.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

LCG_A = 1664525
LCG_C = 1013904223
_MASK = 0xFFFFFFFF
_BLOCK = 1 << 16


def _affine_table(length: int) -> tuple[np.ndarray, np.ndarray]:
    """(A_i, C_i) for i = 1..length with s_i = A_i * s_0 + C_i (mod 2^32)."""
    a = np.empty(length, np.uint64)
    c = np.empty(length, np.uint64)
    a[0], c[0] = LCG_A, LCG_C
    filled = 1
    while filled < length:
        take = min(filled, length - filled)
        a_l, c_l = int(a[filled - 1]), int(c[filled - 1])  # composition of `filled` steps
        # s_{filled+i} = A_filled * s_i + C_filled applied after i steps:
        # A_{filled+i} = A_filled * A_i ; C_{filled+i} = A_filled * C_i + C_filled
        a[filled:filled + take] = (a[:take] * np.uint64(a_l)) & np.uint64(_MASK)
        c[filled:filled + take] = (c[:take] * np.uint64(a_l) + np.uint64(c_l)) & np.uint64(_MASK)
        filled += take
    return a, c


_TABLE = None


def _table():
    global _TABLE
    if _TABLE is None:
        _TABLE = _affine_table(_BLOCK)
    return _TABLE


def _lcg_chunks(n: int, seed: int):
    """Yields (offset, states) covering the first n LCG states after `seed`.

    The stream is cut into blocks of _BLOCK states: block b starts from the
    state reached after b * _BLOCK steps (a short sequential recurrence over
    the blocks), and state i of a block is A_i * s_b + C_i mod 2^32, computed
    for 64 blocks at a time in wrapping uint32 arithmetic.
    """
    a_tab, c_tab = _table()
    a32, c32 = a_tab.astype(np.uint32), c_tab.astype(np.uint32)
    nblocks = (n + _BLOCK - 1) // _BLOCK
    a_block, c_block = int(a_tab[-1]), int(c_tab[-1])
    starts = np.empty(max(nblocks, 1), np.uint32)
    s = seed & _MASK
    for b in range(nblocks):
        starts[b] = s
        s = (a_block * s + c_block) & _MASK
    step = 64
    buf = np.empty((step, _BLOCK), np.uint32)
    for b0 in range(0, nblocks, step):
        b1 = min(nblocks, b0 + step)
        out = buf[:b1 - b0]
        np.multiply(starts[b0:b1, None], a32[None, :], out=out)
        out += c32[None, :]
        off = b0 * _BLOCK
        yield off, out.reshape(-1)[:max(0, min(n - off, (b1 - b0) * _BLOCK))]


def lcg_states(n: int, seed: int) -> np.ndarray:
    """The first n LCG states after `seed` (state i = i+1 steps), as uint32."""
    out = np.empty(n, np.uint32)
    for off, ch in _lcg_chunks(n, seed):
        out[off:off + ch.size] = ch
    return out


def lcg_floats(n: int, seed: int, lo: float, hi: float) -> np.ndarray:
    """Uniform floats in [lo, hi), bit-exact with test_q4gemm.cpp:58-68."""
    u = (lcg_states(n, seed) >> np.uint32(8)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    span = np.float32(np.float32(hi) - np.float32(lo))
    return (np.float32(lo) + (u * span).astype(np.float32)).astype(np.float32)


def lcg_int4(n: int, seed: int) -> np.ndarray:
    """int4 values in [-8, 7], bit-exact with test_q4gemm.cpp:71-80."""
    v = np.empty(n, np.int8)
    for off, ch in _lcg_chunks(n, seed):
        ch >>= np.uint32(8)
        ch &= np.uint32(15)  # (s >> 8) % 16
        v[off:off + ch.size] = ch
    v -= np.int8(8)
    return v


def normal(n: int, seed: int, std: float = 1.0) -> np.ndarray:
    """N(0, std^2) float32 via Box-Muller on consecutive LCG pairs.

    u1 = ((s >> 8) + 1) / 2^24 in (0, 1], u2 = (s >> 8) / 2^24 in [0, 1);
    z0 = sqrt(-2 ln u1) cos(2 pi u2), z1 = sqrt(-2 ln u1) sin(2 pi u2).
    """
    pairs = (n + 1) // 2
    st = (lcg_states(2 * pairs, seed) >> np.uint32(8)).astype(np.float64)
    u1 = (st[0::2] + 1.0) / 16777216.0
    u2 = st[1::2] / 16777216.0
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * pairs, np.float64)
    z[0::2] = r * np.cos(2.0 * np.pi * u2)
    z[1::2] = r * np.sin(2.0 * np.pi * u2)
    return (z[:n] * std).astype(np.float32)


def pack(b_kn: np.ndarray) -> np.ndarray:
    """Logical int4 b[k][n] -> reference-layout uint32 words (K*N/8).

    Same result as pack_q4 (test_q4gemm.cpp:84-99): column n's K/2 bytes are
    contiguous, even k in the low nibble, little-endian words.
    """
    k, n = b_kn.shape
    if k % 8:
        raise ValueError("K must be a multiple of 8")
    nib = (b_kn.astype(np.uint8) & np.uint8(0xF)).T  # [N][K]
    bytes_ = nib[:, 0::2] | (nib[:, 1::2] << np.uint8(4))  # [N][K/2]
    return np.ascontiguousarray(bytes_).view(np.uint32).reshape(-1).copy()


def unpack(packed: np.ndarray, k: int, n: int) -> np.ndarray:
    """Inverse of pack: reference-layout words -> logical int8 b[k][n]."""
    by = np.ascontiguousarray(packed, np.uint32).view(np.uint8).reshape(n, k // 2)
    lo = (by & np.uint8(0xF)).astype(np.int16)
    hi = (by >> np.uint8(4)).astype(np.int16)
    nib = np.empty((n, k), np.int16)
    nib[:, 0::2] = lo
    nib[:, 1::2] = hi
    nib = np.where(nib >= 8, nib - 16, nib)
    return np.ascontiguousarray(nib.T.astype(np.int8))


@dataclass
class Config:
    """One BASELINE configuration (shapes, value ranges, seed)."""
    name: str
    m: int
    k: int
    n: int
    scale_lo: float
    scale_hi: float
    rank: int = 0
    alpha: float = 0.0
    lora_std: float = 0.02
    seed: int = 0
    m_sweep: tuple = field(default_factory=tuple)


CONFIGS = {
    "tiny": Config("tiny", 128, 64, 256, 0.01, 0.05),
    "decode": Config("decode", 1, 4096, 4096, 0.005, 0.02, m_sweep=(1, 2, 4, 8)),
    "prefill": Config("prefill", 2048, 4096, 11008, 0.005, 0.02),
    "lora": Config("lora", 512, 4096, 4096, 0.005, 0.02, rank=16, alpha=32.0),
    "mlp70b": Config("mlp70b", 4096, 8192, 28672, 0.003, 0.01),
}


def _seeds(seed: int) -> dict:
    base = (seed * 0x9E3779B1) & _MASK
    return {name: (base + i * 0x632BE5AB) & _MASK for i, name in enumerate(("x", "w", "s", "a", "b"))}


@dataclass
class Inputs:
    x: np.ndarray          # [M][K] float32
    w_kn: np.ndarray       # [K][N] int8 in [-8, 7] (logical)
    packed: np.ndarray     # K*N/8 uint32 (reference layout)
    scales: np.ndarray     # [N][K/32] float32
    lora_a: np.ndarray | None = None   # [K][rank]
    lora_b: np.ndarray | None = None   # [rank][N]
    rank: int = 0
    alpha: float = 0.0


def make_weights(k: int, n: int, scale_lo: float, scale_hi: float, seed: int = 0):
    s = _seeds(seed)
    w_kn = lcg_int4(k * n, s["w"]).reshape(k, n)
    scales = lcg_floats(n * (k // 32), s["s"], scale_lo, scale_hi).reshape(n, k // 32)
    return w_kn, pack(w_kn), scales


def make_x(m: int, k: int, seed: int = 0) -> np.ndarray:
    return normal(m * k, _seeds(seed)["x"]).reshape(m, k)


def make_inputs(cfg: Config | str, m: int | None = None, seed: int | None = None, weights=None) -> Inputs:
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    seed = cfg.seed if seed is None else seed
    m = cfg.m if m is None else m
    w_kn, packed, scales = weights if weights is not None else make_weights(cfg.k, cfg.n, cfg.scale_lo, cfg.scale_hi, seed)
    x = make_x(m, cfg.k, seed)
    inp = Inputs(x, w_kn, packed, scales)
    if cfg.rank:
        s = _seeds(seed)
        inp.lora_a = normal(cfg.k * cfg.rank, s["a"], cfg.lora_std).reshape(cfg.k, cfg.rank)
        inp.lora_b = normal(cfg.rank * cfg.n, s["b"], cfg.lora_std).reshape(cfg.rank, cfg.n)
        inp.rank, inp.alpha = cfg.rank, cfg.alpha
    return inp
