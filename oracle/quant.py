"""FP8 e4m3 (``float8_e4m3fn``) codec restated in numpy.  Test infrastructure only.

The reference codec is ``src/linattn/kv/quant.py:76-109``: ``scale = absmax / 448``
(clamped to >= 1e-8), ``codes = (x / scale).to(float8_e4m3fn)`` (round to nearest
even; values past the top of the grid become NaN), ``x_hat = codes * scale``.
The reference groups along the last axis; the build applies the same codec with
one scale per (page, kv head) for the paged KV pool and one per 64 tokens for the
indexer keys.
"""

from __future__ import annotations

import numpy as np

__all__ = ["e4m3_encode", "e4m3_decode", "quantize_fp8", "dequantize_fp8"]


def _e4m3_table() -> np.ndarray:
    """float32 value of every code byte: sign | 4-bit exponent (bias 7) | 3-bit mantissa;
    exponent 0 is subnormal; 0x7F / 0xFF are NaN (no infinities)."""
    vals = np.zeros(256, dtype=np.float32)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            vals[code] = np.nan
        elif e == 0:
            vals[code] = sign * (m / 8.0) * 2.0 ** -6
        else:
            vals[code] = sign * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3_TABLE = _e4m3_table()
_POS = E4M3_TABLE[:0x7F].astype(np.float64)  # codes 0..126, ascending, finite


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(codes, dtype=np.uint8)]


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even onto the e4m3 grid; |x| above the midpoint between 448
    and the (unrepresentable) next step 480 encodes NaN, like torch's cast."""
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    a = np.abs(x)
    # hi = first grid point >= a; lo = the one below it (codes are ascending in value,
    # and a code's parity is its mantissa's last bit, so "even" = even code number)
    hi_code = np.clip(np.searchsorted(_POS, np.minimum(a, 448.0), side="left"), 1, 126)
    lo_code = hi_code - 1
    d_lo = a - _POS[lo_code]
    d_hi = _POS[hi_code] - a
    tie_hi = (d_hi == d_lo) & (hi_code % 2 == 0)
    code = np.where((d_hi < d_lo) | tie_hi, hi_code, lo_code)
    code = np.where(a == 0.0, 0, code)
    code = np.where(a > 448.0, 0x7E, code)  # (448, 464] rounds to 448 (464 is a tie -> even)
    code = np.where(a > 464.0, 0x7F, code)  # past the tie: NaN, as torch's cast
    code = np.where(np.isnan(x), 0x7F, code).astype(np.uint8)
    return np.where(np.signbit(x), code | 0x80, code).astype(np.uint8)


def quantize_fp8(x: np.ndarray, reduce_axes) -> tuple:
    """``scale = max|x| / 448`` over ``reduce_axes`` (clamped to 1e-8), ``codes = e4m3(x / scale)``.

    ``src/linattn/kv/quant.py:90-93``; division in float32 as the reference does.
    Returns ``(codes uint8, scale float32 with reduce_axes kept as size 1)``.
    """
    x32 = np.asarray(x, dtype=np.float32)
    amax = np.max(np.abs(x32), axis=reduce_axes, keepdims=True)
    scale = np.maximum(amax, np.float32(1e-8)) / np.float32(448.0)
    scale = scale.astype(np.float32)
    return e4m3_encode((x32 / scale).astype(np.float32)), scale


def dequantize_fp8(codes: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """``codes.float() * scale`` (``src/linattn/kv/quant.py:96-109``), float32."""
    return (e4m3_decode(codes) * scale).astype(np.float32)
