"""NVFP4 codec in numpy.  TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Format (the reference's, ``cirrus/perf/bench_kernels.cu:141-145`` and
``scripts/bench_spark.py:290-296, 400-404``):

* E2M1 codes, 4 bits: bit 3 is the sign, bits 0-2 index the magnitudes
  {0, 0.5, 1, 1.5, 2, 3, 4, 6}.
* one E4M3 (``float8_e4m3fn``) scale byte per 16 consecutive elements of a row;
* one float32 tensor scale;  value = lut[code] * e4m3(scale) * tensor_scale.
* standard packing: ``uint8[N, K/2]``, low nibble = even k.

The reference has no quantiser (its benchmark draws random codes and scales,
``bench_spark.py:284-287, 394-397``).  The quantiser here is the recipe of the
benchmark configuration: block scale = absmax(block / tensor_scale) / 6
rounded to E4M3 (nearest-even, saturating at 448), codes = E2M1 nearest-even
of (w / tensor_scale) / scale, saturating at 6, sign taken from the sign bit
of the quotient; a zero scale gives zero codes.  Every division is one
float32 IEEE division, as in the CUDA quantiser.
"""

from __future__ import annotations

import numpy as np

E2M1_MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
E2M1_LUT = np.concatenate([E2M1_MAG, -E2M1_MAG]).astype(np.float32)  # bench_spark.py:291-292


def _e4m3_table() -> np.ndarray:
    """Magnitudes of the 127 finite non-negative E4M3 codes 0x00..0x7E (ascending)."""
    out = np.zeros(127, dtype=np.float64)
    for c in range(127):
        e, m = c >> 3, c & 7
        out[c] = m * 2.0**-9 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return out


E4M3_MAG = _e4m3_table()


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    """E4M3 bytes -> float32 (0x7F / 0xFF are NaN)."""
    b = np.asarray(b, dtype=np.uint8)
    mag = np.concatenate([E4M3_MAG, [np.nan]])[b & 0x7F]
    return np.where(b & 0x80, -mag, mag).astype(np.float32)


def _rne_to_table(a: np.ndarray, table: np.ndarray) -> np.ndarray:
    """Index of the nearest table entry to each non-negative ``a`` (float64),
    ties to the even index, saturating at the last entry."""
    n = len(table)
    hi = np.clip(np.searchsorted(table, a, side="left"), 1, n - 1)
    lo = hi - 1
    d_lo = a - table[lo]
    d_hi = table[hi] - a
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    idx = np.where(pick_hi, hi, lo)
    return np.where(a >= table[-1], n - 1, idx)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> E4M3 byte, round-to-nearest-even, saturating to +-448."""
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    code = _rne_to_table(np.abs(x), E4M3_MAG).astype(np.uint8)
    return np.where(np.signbit(x), code | 0x80, code).astype(np.uint8)


def e2m1_encode_table(x: np.ndarray) -> np.ndarray:
    """float32 -> E2M1 code (0..15), round-to-nearest-even, saturating to +-6 (table search)."""
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    code = _rne_to_table(np.abs(x), E2M1_MAG.astype(np.float64)).astype(np.uint8)
    return np.where(np.signbit(x), code | 0x8, code).astype(np.uint8)


def e2m1_encode(x: np.ndarray) -> np.ndarray:
    """Same result as ``e2m1_encode_table`` for non-NaN input, by counting the
    rounding boundaries below |x|: a boundary that is a tie belongs to the
    even code (0.25 -> 0, 0.75 -> 1.0, 1.25 -> 1.0, 1.75 -> 2.0, 2.5 -> 2.0,
    3.5 -> 4.0, 5.0 -> 4.0)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x)
    code = ((a > 0.25).astype(np.uint8) + (a >= 0.75) + (a > 1.25) + (a >= 1.75) + (a > 2.5) + (a >= 3.5)
            + (a > 5.0)).astype(np.uint8)
    return np.where(np.signbit(x), code | 0x8, code).astype(np.uint8)


def quantize(w: np.ndarray, tensor_scale: float = 1.0) -> tuple[np.ndarray, np.ndarray]:
    """``w`` float32 [N, K] (K % 16 == 0) -> (codes uint8 [N, K] in 0..15, scales uint8 [N, K/16])."""
    w = np.asarray(w, dtype=np.float32)
    N, K = w.shape
    if K % 16:
        raise ValueError("K must be a multiple of 16")
    wt = (w / np.float32(tensor_scale)).astype(np.float32).reshape(N, K // 16, 16)
    amax = np.abs(wt).max(-1)
    scode = e4m3_encode((amax / np.float32(6.0)).astype(np.float32))
    sval = e4m3_decode(scode)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = (wt / sval[..., None]).astype(np.float32)
    codes = e2m1_encode(np.where(sval[..., None] == 0, np.float32(0.0), q))
    return codes.reshape(N, K), scode


def pack_standard(codes: np.ndarray) -> np.ndarray:
    """[N, K] codes -> [N, K/2] bytes, low nibble = even k (bench_kernels.cu:142)."""
    c = np.asarray(codes, dtype=np.uint8)
    return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)


def unpack_standard(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty((p.shape[0], p.shape[1] * 2), dtype=np.uint8)
    out[:, 0::2] = p & 0xF
    out[:, 1::2] = p >> 4
    return out


def dequantize(codes: np.ndarray, scales: np.ndarray, tensor_scale: float = 1.0) -> np.ndarray:
    """codes [N, K] (0..15), scales [N, K/16] -> float32 [N, K]:
    ``lut[code] * scale * tensor_scale`` (bench_spark.py:400-404), evaluated as
    float32 products in that order."""
    vals = E2M1_LUT[np.asarray(codes, dtype=np.uint8)]
    sc = np.repeat(e4m3_decode(scales), 16, axis=-1)
    return ((vals * sc).astype(np.float32) * np.float32(tensor_scale)).astype(np.float32)


def fake_quant(w: np.ndarray, tensor_scale: float = 1.0) -> np.ndarray:
    """dequantize(quantize(w)): the weights the NVFP4 path computes with."""
    codes, scales = quantize(w, tensor_scale)
    return dequantize(codes, scales, tensor_scale)
