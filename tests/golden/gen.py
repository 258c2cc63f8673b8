"""Seeded tensor generators shared by the fixture script and the tests.

SplitMix64 (INTEGER_LLM/kernels/src/prng.rs:7-15) is counter based: after i
steps from ``seed`` the state is ``seed + i * 0x9E3779B97F4A7C15`` (mod 2^64)
and the output word is the mix of that state. ``stream`` evaluates it for all
i at once with numpy's wrapping uint64 arithmetic.

``int8_tensor`` reproduces ``deterministic_tensor`` of the reference's
golden-vector generator (INTEGER_LLM/tests/golden/generate.py:156-165):
low byte of each word, reinterpreted as a signed byte.
"""
from __future__ import annotations

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)


def stream(seed: int, n: int) -> np.ndarray:
    """The first n SplitMix64 output words from ``seed``."""
    i = np.arange(1, n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + i * GOLDEN
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
    return z ^ (z >> np.uint64(31))


def int8_tensor(seed: int, n: int) -> np.ndarray:
    """generate.py:156 deterministic_tensor: full int8 range [-128, 127]."""
    return (stream(seed, n) & np.uint64(0xFF)).astype(np.uint8).view(np.int8)


def int16_tensor(seed: int, n: int, bits: int = 16) -> np.ndarray:
    """Signed values in [-2^(bits-1), 2^(bits-1)) from bits 24..39 of each word."""
    v = ((stream(seed, n) >> np.uint64(24)) & np.uint64(0xFFFF)).astype(np.uint16).view(np.int16)
    return (v >> np.int16(16 - bits)).astype(np.int16)


def uint8_tensor(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """Values in [lo, hi] (inclusive), for shift tables."""
    span = np.uint64(hi - lo + 1)
    return (np.int64(lo) + (stream(seed, n) % span).astype(np.int64)).astype(np.uint8)


def nominal_shift(K: int, x_bits: int) -> int:
    """A total right shift that keeps outputs mostly inside int16 for full-range
    int8 weights and ``x_bits``-bit activations: log2(sigma_acc / 2^11)."""
    sigma = 73.9 * (2.0 ** (x_bits - 1) / np.sqrt(3.0)) * np.sqrt(K)
    return max(0, int(round(np.log2(sigma / 2048.0))))
