"""Seeded synthetic inputs in the reference's native GGUF block layouts.

Distributions follow the benchmark configuration of this build: every fp16
block scale (``d``, and ``dmin`` for Q4_K) is |N(0, 0.02)| cast to fp16; every
other byte (nibbles, Q8_0 quants, Q4_K packed 6-bit scales, Q6_K ql/qh/int8
scales) is uniform random; activations are N(0, 1) fp32.  Byte layouts are
those of csrc/gncx_llm_kernels.cpp:273-297 (packed, little-endian).
"""
from __future__ import annotations

import numpy as np

from .core import BF16, BLOCK, F32, Q4_0, Q4_K, Q6_K, Q8_0, row_bytes


def _scales(rng: np.random.Generator, n: int) -> np.ndarray:
    return np.abs(rng.normal(0.0, 0.02, size=n)).astype(np.float16).view(np.uint8).reshape(n, 2)


def random_weights(ggml_type: int, out_dim: int, in_dim: int, seed: int = 0,
                   rng: np.random.Generator | None = None) -> np.ndarray:
    """uint8 array [out_dim, row_bytes] of random blocks."""
    rng = rng or np.random.default_rng(seed)
    if ggml_type == BF16:
        bits = rng.normal(0, 0.02, size=(out_dim, in_dim)).astype(np.float32).view(np.uint32) >> 16
        return np.ascontiguousarray(bits.astype(np.uint16).view(np.uint8).reshape(out_dim, in_dim * 2))
    if ggml_type == F32:
        return rng.normal(0, 1, size=(out_dim, in_dim)).astype(np.float32).view(np.uint8)
    be, bb = BLOCK[ggml_type]
    nb = in_dim // be
    raw = rng.integers(0, 256, size=(out_dim, nb, bb), dtype=np.uint8)
    flat = raw.reshape(out_dim * nb, bb)
    if ggml_type in (Q4_0, Q8_0):
        flat[:, 0:2] = _scales(rng, flat.shape[0])
    elif ggml_type == Q4_K:
        flat[:, 0:2] = _scales(rng, flat.shape[0])
        flat[:, 2:4] = _scales(rng, flat.shape[0])
    elif ggml_type == Q6_K:
        flat[:, 208:210] = _scales(rng, flat.shape[0])
    return np.ascontiguousarray(raw.reshape(out_dim, nb * bb))


def random_weights_fast(ggml_type: int, out_dim: int, in_dim: int, seed: int = 0) -> np.ndarray:
    """Same distribution, generated in row chunks (for multi-hundred-MB tensors)."""
    rng = np.random.default_rng(seed)
    out = np.empty((out_dim, row_bytes(ggml_type, in_dim)), dtype=np.uint8)
    step = max(1, (64 << 20) // max(1, out.shape[1]))
    for r0 in range(0, out_dim, step):
        r1 = min(out_dim, r0 + step)
        out[r0:r1] = random_weights(ggml_type, r1 - r0, in_dim, rng=rng)
    return out


def random_activations(n: int, seed: int = 0, rows: int | None = None) -> np.ndarray:
    rng = np.random.default_rng(seed)
    shape = (n,) if rows is None else (rows, n)
    return rng.normal(0.0, 1.0, size=shape).astype(np.float32)
