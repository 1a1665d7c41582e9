"""Number formats of the path, restated in numpy (test infrastructure).

bf16 / fp16 round-to-nearest-even from fp32, and the float8 e4m3fn code book
(1 sign, 4 exponent bits with bias 7, 3 mantissa bits, no infinities, 0x7F =
NaN, largest finite 448) with round-to-nearest-even and saturation to +-448.
"""

from __future__ import annotations

import numpy as np


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); result as float32."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    out[nan] = np.nan
    return out


def round_fp16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def _e4m3_table() -> np.ndarray:
    vals = np.zeros(127, dtype=np.float64)
    for code in range(127):  # 0x00..0x7E, non-negative finite values
        e = code >> 3
        m = code & 7
        vals[code] = (m / 8.0) * 2.0 ** -6 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3_POS = _e4m3_table()
E4M3_MAX = 448.0


def encode_e4m3(x: np.ndarray) -> np.ndarray:
    """float -> e4m3fn byte codes, round-to-nearest-even, saturating to +-448 (NaN -> 0x7F)."""
    v = np.asarray(x, dtype=np.float64)
    sign = (np.signbit(v)).astype(np.uint8) << 7
    a = np.minimum(np.abs(v), E4M3_MAX)
    idx = np.searchsorted(E4M3_POS, a, side="left")  # first table value >= a
    idx = np.clip(idx, 0, 126)
    lo = np.clip(idx - 1, 0, 126)
    d_hi = E4M3_POS[idx] - a
    d_lo = a - E4M3_POS[lo]
    pick_lo = (d_lo < d_hi) | ((d_lo == d_hi) & (lo % 2 == 0) & (lo != idx))
    code = np.where(pick_lo, lo, idx).astype(np.uint8)
    code = code | sign
    code = np.where(np.isnan(v), np.uint8(0x7F), code)
    return code.astype(np.uint8)


def decode_e4m3(code: np.ndarray) -> np.ndarray:
    c = np.asarray(code, dtype=np.uint8)
    mag = c & 0x7F
    out = np.where(mag == 0x7F, np.nan, E4M3_POS[np.minimum(mag, 126)])
    return np.where(c & 0x80, -out, out).astype(np.float32)


def quantize_e4m3_rows(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-output-channel e4m3: scale = max|row| / 448 (1 for a zero row), q = e4m3(w / scale).

    No reference code exists for FP8; this follows the per-channel pattern of the
    integer fake quantizer (stageml/quant_absint.py:47-82, per_channel, channel_dim=0).
    The division is fp32, as on the device.
    """
    w32 = np.asarray(w, dtype=np.float32)
    rows = w32.reshape(-1, w32.shape[-1])
    amax = np.abs(rows).max(axis=1)
    scale = np.where(amax > 0, (amax / np.float32(448.0)).astype(np.float32), np.float32(1.0)).astype(np.float32)
    q = encode_e4m3((rows / scale[:, None]).astype(np.float32))
    return q.reshape(w32.shape), scale.reshape(w32.shape[:-1])


def dequantize_e4m3_rows(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """The dequantized weight q * scale[:, None] (the pattern of quant_dequant, stageml/quant_absint.py:81-82)."""
    return decode_e4m3(q) * np.asarray(scale, dtype=np.float32)[..., None]
