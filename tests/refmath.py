"""Small numpy helpers that restate the reference's scalar conventions for tests."""
from fractions import Fraction

import numpy as np


def round_bf16_np(x):
    """round_bf16 (src/tensor.rs:645-652) on a float32 array: RNE, NaN quieted."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    r = np.where(nan, ((b & 0xFFFF0000) | 0x00400000).astype(np.uint32), r)
    return r.view(np.float32)


def f32lit(text):
    """A Rust f32 literal: the decimal correctly rounded to float32 (no double rounding)."""
    exact = Fraction(text)
    cand = np.float32(float(exact))
    best = cand
    for c in (np.nextafter(cand, np.float32(-np.inf)), cand, np.nextafter(cand, np.float32(np.inf))):
        if abs(Fraction(float(c)) - exact) < abs(Fraction(float(best)) - exact):
            best = c
    return np.float32(best)


def bf16_bits(x):
    """float32 (bf16-valued) -> uint16 bf16 bits."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bits_to_f32(b):
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
