"""Seeded synthetic inputs shared by the GPU path, the CPU oracle and bench.py.

Counter-based generator: value i of stream (seed, stream) is a function of
(seed, stream, i) only, so any slice of a large input can be regenerated
without producing the rest.  Normals come from splitmix64 -> Box-Muller;
bf16 values are the round-to-nearest-even of the fp32 sample (the rounding of
src/mla_compressed_q8_state.c:9-16 for finite inputs).
"""
from __future__ import annotations

import numpy as np

_M = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def _key(seed: int, stream: int) -> np.uint64:
    k = _splitmix64(np.array([(seed & 0xFFFFFFFF) << 32 | (stream & 0xFFFFFFFF)], dtype=np.uint64))
    return k[0]


def uniform01(seed: int, stream: int, n: int, offset: int = 0) -> np.ndarray:
    """n doubles in (0, 1]."""
    with np.errstate(over="ignore"):
        c = _key(seed, stream) + np.arange(offset, offset + n, dtype=np.uint64)
    z = _splitmix64(c)
    return ((z >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)


def normal(seed: int, stream: int, n: int, std: float = 1.0, offset: int = 0) -> np.ndarray:
    """n float32 samples of N(0, std^2)."""
    u1 = uniform01(seed, 2 * stream, n, offset)
    u2 = uniform01(seed, 2 * stream + 1, n, offset)
    r = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return (r * std).astype(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    finite = (u & 0x7F800000) != 0x7F800000
    r = np.where(finite, u + 0x7FFF + ((u >> 16) & 1), u)
    return (r >> 16).astype(np.uint16)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def normal_bf16(seed: int, stream: int, shape, std: float = 1.0) -> np.ndarray:
    """bf16 bit patterns of N(0, std^2) samples, shaped."""
    n = int(np.prod(shape))
    return f32_to_bf16_bits(normal(seed, stream, n, std)).reshape(shape)


def uniform_int8(seed: int, stream: int, shape, lo: int = -127, hi: int = 127) -> np.ndarray:
    n = int(np.prod(shape))
    u = uniform01(seed, stream, n)
    v = np.floor(u * (hi - lo + 1)).astype(np.int64) + lo
    return np.clip(v, lo, hi).astype(np.int8).reshape(shape)


def uniform_f32(seed: int, stream: int, shape, lo: float, hi: float) -> np.ndarray:
    n = int(np.prod(shape))
    return (lo + (hi - lo) * uniform01(seed, stream, n)).astype(np.float32).reshape(shape)


def uniform_ints(seed: int, stream: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers uniform in [lo, hi]."""
    u = uniform01(seed, stream, n)
    return np.minimum(lo + np.floor(u * (hi - lo + 1)).astype(np.int64), hi)


# Stream ids used by the benchmark configurations (seed = configuration index).
S_Q, S_LAT, S_ROPE, S_X, S_WQ, S_WKVA, S_WKVB, S_WO, S_SCALE, S_LEN = range(10)
