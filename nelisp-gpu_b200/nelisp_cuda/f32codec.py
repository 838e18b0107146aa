"""The float32 wire codec of the reference client.

Every float crossing the server boundary is encoded by
`nelisp-gpu--f32-bits' (lisp/nelisp-gpu-compile.el:128-156) and decoded by
`nelisp-gpu--bits-f32' (lisp/nelisp-gpu-run.el:23-36).  This restates both:
IEEE round-to-nearest into normals and subnormals, overflow to a signed
infinity at (2 - 2^-24) * 2^127, FLT_MAX staying finite, zero (of either
sign) to the word 0, and any NaN to the canonical 0x7fc00000.  Vectorised
with numpy, whose float64 -> float32 conversion is that same rounding.
"""
from __future__ import annotations

import numpy as np

CANONICAL_NAN = 0x7FC00000


def f32_bits(x) -> np.ndarray:
    """float(s) -> uint32 bit patterns, as `nelisp-gpu--f32-bits'."""
    a = np.atleast_1d(np.asarray(x, dtype=np.float64))
    with np.errstate(over="ignore"):
        bits = a.astype(np.float32).view(np.uint32).copy()
    bits[a == 0.0] = 0                     # (= x 0.0) holds for -0.0 too
    bits[np.isnan(a)] = CANONICAL_NAN
    return bits


def bits_f32(bits) -> np.ndarray:
    """uint32 bit patterns -> float64 values, as `nelisp-gpu--bits-f32'."""
    b = np.atleast_1d(np.asarray(bits, dtype=np.uint32))
    return b.view(np.float32).astype(np.float64)


def floats_bytes(*vectors) -> bytes:
    """`nelisp-gpu--floats-bytes' (lisp/nelisp-gpu-server.el:45-54)."""
    if not vectors:
        return b""
    return b"".join(f32_bits(v).astype("<u4").tobytes() for v in vectors if len(np.atleast_1d(v)))


def u32_bytes(n: int) -> bytes:
    """`nelisp-gpu--u32-bytes' (lisp/nelisp-gpu-server.el:37-39)."""
    return int(n & 0xFFFFFFFF).to_bytes(4, "little")


def decode_words(buf: bytes, offset_words: int, n: int) -> np.ndarray:
    w = np.frombuffer(buf, dtype="<u4", count=n, offset=4 * offset_words)
    return bits_f32(w)
