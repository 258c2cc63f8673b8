"""Seeded random-init layers at the benchmark shapes (no checkpoints exist
here): int8 weights uniform in [-127, 127], per-row power-of-two shifts that
keep outputs mostly unsaturated, int16 activations rounded N(0, 1024^2).
"""
from __future__ import annotations

import math

import numpy as np

# BASELINE config 4
MOE_CONFIG4 = dict(H=2048, I=1408, E=64, k=4, shared_I=5632, T=4096)


def kbits(K: int) -> int:
    """Per-row weight shift that keeps outputs unsaturated: round(log2(73.6*sqrt(K)))."""
    return int(round(math.log2(73.6 * math.sqrt(K))))


def activations(rng, shape, sigma: float = 1024.0) -> np.ndarray:
    return np.clip(np.rint(rng.normal(0, sigma, size=shape)), -32767, 32767).astype(np.int16)


def exp_lut14() -> np.ndarray:
    """exp(-i / 256) at 14 fractional bits, 16384 entries."""
    return np.array([int(round(math.exp(-i / 256.0) * (1 << 14))) for i in range(16384)], np.int16)


def silu_lut() -> np.ndarray:
    """SiLU over [-128, 128) at 6 fractional input bits, 8 output bits; offset 8192."""
    xs = (np.arange(16384) - 8192) / 64.0
    return np.clip(np.round(xs / (1.0 + np.exp(-xs)) * 256), -32768, 32767).astype(np.int16)


def moe_layer(ctx, H: int, I: int, E: int, k: int, shared_I: int, first: int = 0,
              num_local: int | None = None, attach_shared: bool = True, seed: int = 4000):
    """(Moe, shared Mlp or None) with experts [first, first + num_local).
    Every rank that uses the same seed gets the same weights. The router
    shifts are equal across experts, so the expected load is balanced."""
    import myelith_b200 as myl

    nl = E - first if num_local is None else num_local
    rng = np.random.default_rng(seed)
    sh = kbits(H)

    def ints(shape):
        return rng.integers(-127, 128, size=shape, dtype=np.int8)

    Wr = ints((E, H))
    rs = np.full(E, sh + 4, np.uint8)
    Wg, Wu, Wd = ints((E, I, H)), ints((E, I, H)), ints((E, H, I))
    gs = rng.integers(sh - 1, sh + 2, size=(E, I)).astype(np.uint8)
    us = rng.integers(sh - 1, sh + 2, size=(E, I)).astype(np.uint8)
    ds = rng.integers(kbits(I) - 1, kbits(I) + 2, size=(E, H)).astype(np.uint8)
    of = rng.integers(3, 8, size=(E, H)).astype(np.uint8)
    silu = silu_lut()
    shared = None
    if shared_I:
        shared = myl.Mlp(ctx, ints((shared_I, H)), ints((shared_I, H)), ints((H, shared_I)), H, shared_I,
                         rng.integers(sh - 1, sh + 2, size=shared_I).astype(np.uint8),
                         rng.integers(sh - 1, sh + 2, size=shared_I).astype(np.uint8),
                         rng.integers(kbits(shared_I) - 1, kbits(shared_I) + 2, size=H).astype(np.uint8),
                         silu, 8, 7, 7, 7, 6, 8192, 8, rng.integers(3, 8, size=H).astype(np.uint8))
    sl = slice(first, first + nl)
    moe = myl.Moe(ctx, H, I, E, k, Wr, rs, 8, 12, exp_lut14(), 4, 14, Wg[sl], Wu[sl], Wd[sl], gs[sl],
                  us[sl], ds[sl], of[sl], silu, 8, 7, 7, 7, 6, 8192, 8,
                  shared=shared if attach_shared else None, first_expert=first, num_local=nl)
    return moe, shared
