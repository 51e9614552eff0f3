"""numpy restatement of the reference's Q4 record format (test infrastructure).

The checker for the product's on-device quantiser and store repack. It is
pinned against the reference's own quantiser by tests/golden fixtures that
tests/golden/make_golden.py generates by importing the reference.

Format (src/jouleai/storage/q4_store.py:1-10, 23, 40-67): a tensor is
flattened row-major into groups of 64 values; each group gets one fp16 scale
``fp16(max(|g|, 1e-12) / 7)`` computed in fp32; each value is
``clip(round_half_even(v / fp32(scale)), -8, 7)`` stored biased by +8, two per
byte, the even element in the low nibble. A record is
``[scales fp16 x numel/64][packed u8 x numel/2]``.
"""
from __future__ import annotations

import numpy as np

GROUP = 64


def quantize(x: np.ndarray, group: int = GROUP) -> tuple[np.ndarray, np.ndarray]:
    """Restates ``_quantize_tensor`` (q4_store.py:40-55).

    Returns ``(scales uint16 [numel/group], packed uint8 [numel/2])``; the
    uint16 array holds the fp16 bit patterns.
    """
    v = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    n = v.size
    tail = (-n) % group
    if tail:
        v = np.concatenate([v, np.zeros(tail, np.float32)])
    g = v.reshape(-1, group)
    amax = np.abs(g).max(axis=1)
    amax = np.maximum(amax, np.float32(1e-12))
    scale16 = (amax / np.float32(7.0)).astype(np.float16)
    with np.errstate(divide="ignore", invalid="ignore"):
        # a scale that underflows to 0 gives +-inf (clipped) or NaN (cast to 0)
        q = np.rint(g / scale16.astype(np.float32)[:, None])
        q = np.clip(q, -8, 7).astype(np.int8)
    biased = (q.astype(np.int16) + 8).astype(np.uint8).reshape(-1)[:n]
    if tail:
        biased = np.concatenate([biased, np.zeros(tail, np.uint8)])
    packed = (biased[0::2] & 0x0F) | (biased[1::2] << 4)
    return scale16.view(np.uint16).copy(), packed.astype(np.uint8)


def dequantize(scales: np.ndarray, packed: np.ndarray, numel: int,
               group: int = GROUP) -> np.ndarray:
    """Restates ``_dequantize`` (q4_store.py:58-67): fp32 ``(nib - 8) * scale``."""
    p = np.asarray(packed, dtype=np.uint8).reshape(-1)
    vals = np.empty(p.size * 2, np.float32)
    vals[0::2] = (p & 0x0F).astype(np.float32) - 8.0
    vals[1::2] = (p >> 4).astype(np.float32) - 8.0
    s = np.asarray(scales).view(np.float16).astype(np.float32)
    return (vals.reshape(-1, group) * s[:, None]).reshape(-1)[:numel]


def record(x: np.ndarray) -> bytes:
    """One ``experts_q4.bin`` record: scales then packed (q4_store.py:150-152)."""
    s, p = quantize(x)
    return s.tobytes() + p.tobytes()
