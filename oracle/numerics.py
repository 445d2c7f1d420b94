"""Bit-level number formats used by the GEMV path, restated in numpy (test oracle).

* bf16: round-to-nearest-even of fp32, the rounding torch's ``.to(torch.bfloat16)``
  applies and the one the reference kernels apply before storing
  (kernels/sglang/srt/layers/quantization/w8a16_gemv.py:92-95).
* e4m3 (float8_e4m3fn): decode of all 256 codes; encode = nearest representable value
  with ties to the even code, values above 464 (and inf / nan) -> nan, which is torch's
  float -> float8_e4m3fn conversion that the reference quantiser relies on
  (kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py:463-465).
* e2m1: the 16 NVFP4 codes, code 8 = -0 (w4a16_nvfp4_gemv.py:408-413,
  bench/bench/moe_smallm/refs.py:22-27).
"""

from __future__ import annotations

import numpy as np

E2M1_LEVELS = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
E2M1_LUT = np.concatenate([E2M1_LEVELS, -E2M1_LEVELS]).astype(np.float32)  # code -> value
E4M3_MAX = 448.0
E2M1_MAX = 6.0


# --------------------------------------------------------------------------- bf16
def bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest, ties to even; NaN kept."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint32) & 0xFFFF
    nan = np.isnan(a)
    if nan.any():
        r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint32) & 0xFFFF, r)
    return r.astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


def bf16_round(a: np.ndarray) -> np.ndarray:
    """fp32 (or fp64, narrowed to fp32 first) rounded to bf16, returned as fp32."""
    return bf16_from_bits(bf16_bits(np.asarray(a, dtype=np.float32)))


def bf16_round_from_f64(a: np.ndarray) -> np.ndarray:
    """Round fp64 values straight to bf16 (ties to even), returned as fp32.

    Rounds the fp64 significand to bf16's 8 bits on the fp64 bit pattern, so there is
    no intermediate fp32 rounding.  Exact for the fp32 normal range, which is bf16's.
    """
    a = np.ascontiguousarray(a, dtype=np.float64)
    u = a.view(np.uint64)
    lsb = (u >> np.uint64(45)) & np.uint64(1)
    r = ((u + np.uint64((1 << 44) - 1) + lsb) >> np.uint64(45)) << np.uint64(45)
    out = r.view(np.float64)
    out = np.where(np.isfinite(a), out, a)
    with np.errstate(over="ignore"):
        return out.astype(np.float32)


def ulp_diff_bf16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in bf16 steps between two arrays of bf16-representable values."""

    def ordered(x):
        bits = bf16_bits(np.asarray(x, dtype=np.float32)).astype(np.int32)
        return np.where(bits & 0x8000, -(bits & 0x7FFF), bits)

    return np.abs(ordered(a) - ordered(b))


# --------------------------------------------------------------------------- e4m3
def _e4m3_table() -> np.ndarray:
    codes = np.arange(256, dtype=np.uint32)
    s = (codes >> 7) & 1
    e = (codes >> 3) & 0xF
    m = codes & 7
    mag = np.where(e == 0, m / 8.0 * 2.0**-6, (1.0 + m / 8.0) * 2.0 ** (e.astype(np.float64) - 7))
    mag = np.where((e == 15) & (m == 7), np.nan, mag)
    return np.where(s == 1, -mag, mag).astype(np.float32)


E4M3_TABLE = _e4m3_table()
_POS_CODES = np.arange(0, 127, dtype=np.int64)  # 0x00..0x7E: 0 .. 448, ascending
_POS_VALUES = E4M3_TABLE[:127].astype(np.float64)


def e4m3_to_f32(codes: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(codes, dtype=np.uint8).astype(np.int64)]


def f32_to_e4m3(a: np.ndarray) -> np.ndarray:
    """fp32 -> float8_e4m3fn codes (torch semantics: RNE, |x| > 464 or inf/nan -> nan)."""
    a = np.asarray(a, dtype=np.float32)
    mag = np.abs(a).astype(np.float64)
    neg = np.signbit(a)
    hi = np.searchsorted(_POS_VALUES, mag, side="left").clip(0, 126)
    lo = (hi - 1).clip(0, 126)
    vhi, vlo = _POS_VALUES[hi], _POS_VALUES[lo]
    dhi, dlo = np.abs(vhi - mag), np.abs(mag - vlo)
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (_POS_CODES[hi] % 2 == 0))
    code = np.where(pick_hi, _POS_CODES[hi], _POS_CODES[lo])
    code = np.where(mag == vhi, _POS_CODES[hi], code)
    over = ~np.isfinite(mag) | (mag > 464.0)
    code = np.where(over, 0x7F, code)
    code = np.where(neg, code | 0x80, code)
    return code.astype(np.uint8)


# --------------------------------------------------------------------------- e2m1
def e2m1_to_f32(codes: np.ndarray) -> np.ndarray:
    return E2M1_LUT[np.asarray(codes, dtype=np.uint8).astype(np.int64) & 0xF]


def round_e2m1(a: np.ndarray) -> np.ndarray:
    """|a| in block-scale units -> magnitude code 0..7, nearest level, ties to even code.

    Restates w4a16_nvfp4_gemv.py:416-423: bucketize against the midpoints with exact
    hits rounding down, then bump the three midpoints whose even neighbour is above
    (0.75 -> 1.0, 1.75 -> 2.0, 3.5 -> 4.0).
    """
    a = np.asarray(a, dtype=np.float32)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
    idx = np.searchsorted(mids, a, side="left")
    up = (a == np.float32(0.75)) | (a == np.float32(1.75)) | (a == np.float32(3.5))
    return np.clip(idx + up, 0, 7).astype(np.uint8)
