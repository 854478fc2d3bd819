"""Bit packing restated in numpy (oracle; test infrastructure only).

Reference: quantization/utils/binary_packer.py:4-50 (binary_packer),
:53-97 (binary_unpacker); quantization/functions/binary.py:7-10 (sign with
0 -> +1).
"""
from __future__ import annotations

import numpy as np


def sign(x: np.ndarray) -> np.ndarray:
    """STEBinary forward (binary.py:7-10): sign(x), zeros mapped to +1."""
    y = np.sign(x)
    y[y == 0] = 1
    return y


def binary_packer(t: np.ndarray) -> np.ndarray:
    """binary_packer.py:4-50: int8 ±1 [R, C] -> int32 [R, ceil(C/32)].

    Pads with +1 (bit 0), bit = (1 - v) // 2 so -1 -> 1, LSB-first within
    each 32-column word, words are the signed int32 view of the bit pattern.
    """
    if t.dtype != np.int8:
        raise TypeError("Input tensor must be int8.")
    rows, cols = t.shape
    wpr = (cols + 31) // 32
    pad = wpr * 32 - cols
    if pad:
        t = np.concatenate([t, np.ones((rows, pad), dtype=np.int8)], axis=1)
    bits = ((1 - t.astype(np.int64)) // 2).reshape(rows, wpr, 32)
    wts = (np.uint64(1) << np.arange(32, dtype=np.uint64)).astype(np.int64)
    packed = (bits * wts).sum(axis=2)
    return packed.astype(np.uint32).view(np.int32) if packed.dtype != np.int32 else packed


def binary_unpacker(packed: np.ndarray, shape) -> np.ndarray:
    """binary_packer.py:53-97: int32 words -> int8 ±1 of ``shape`` (pad trimmed)."""
    rows, cols = shape
    wpr = (cols + 31) // 32
    if packed.ndim != 2 or packed.shape != (rows, wpr):
        raise ValueError(f"Unsupported packed tensor format {packed.shape}")
    u = packed.astype(np.int64) & 0xFFFFFFFF
    bits = (u[:, :, None] >> np.arange(32, dtype=np.int64)) & 1
    bits = bits.reshape(rows, wpr * 32)[:, :cols]
    return (1 - 2 * bits).astype(np.int8)


def unpack_float(packed: np.ndarray, shape, dtype=np.float64) -> np.ndarray:
    return binary_unpacker(packed, shape).astype(dtype)
