"""CPU oracle for the block-scaled expert-weight formats of the reference.

TEST INFRASTRUCTURE ONLY.  Only tests/ may import this module; nothing in the
product does.  It restates, in numpy, the reference's CPU definitions of the
quantised formats that its expert GEMMs take (kkontosis/LayerStoRmExpertKernels,
tests/test_reference.py:19-107), the next row of the hot-path scope after the
bf16 layer:

  * FP8 E4M3 with one float32 scale per 128 consecutive elements of a row
    (`ref_fp8_dequant`, test_reference.py:56-73; `ref_dynamic_fp8_quant`,
    test_reference.py:76-107);
  * NVFP4: two E2M1 codes per byte, low nibble first, one scale per 16
    elements (`ref_nvfp4_dequant`, test_reference.py:19-53).

It is pinned against the reference itself: tests/golden/make_golden.py runs
those three functions on seeded inputs and tests/test_oracle_golden.py checks
the functions here against the committed outputs bit for bit.

The reference's CPU quantiser leaves the quantised values in float32 (clamped
to the E4M3 range, not rounded to E4M3 codes).  A device kernel that stores
E4M3 bytes rounds them once more; `e4m3_round` / `e4m3_encode` /
`e4m3_decode` give that step from the OCP 8-bit floating-point format
(E4M3: bias 7, no infinities, S.1111.111 the only NaN, largest finite 448,
subnormals m/8 * 2^-6), rounding to nearest with ties to even.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
FP8_E4M3_MAX = F32(448.0)

# E2M1 code -> value (test_reference.py:33-36): codes 8..15 are the negatives.
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=F32)


def fp8_dequant(values: np.ndarray, scales: np.ndarray, block: int = 128) -> np.ndarray:
    """values [M, N] float32 (E4M3-range numbers), scales [M, ceil(N/block)]
    -> float32 values[r, c] * scales[r, c // block] (test_reference.py:56-73:
    the product of two float32 numbers is exact in double and rounded once to
    float32, which is the float32 product)."""
    v = np.asarray(values, dtype=F32)
    s = np.asarray(scales, dtype=F32)
    cols = np.arange(v.shape[1]) // block
    return (v * s[:, cols]).astype(F32)


def dynamic_fp8_quant(x: np.ndarray, block: int = 128):
    """x [M, K] -> (quantised [M, K] float32, scales [M, ceil(K/block)] float32)
    as test_reference.py:76-107: per row and block, amax = max |x| (exact),
    scale = amax / 448 in double, stored as float32 (1.0 for an all-zero
    block); quantised = clamp(x / scale, -448, 448) with the division in
    float32 by the stored float32 scale."""
    v = np.asarray(x, dtype=F32)
    M, K = v.shape
    nb = (K + block - 1) // block
    scales = np.zeros((M, nb), dtype=F32)
    out = np.zeros((M, K), dtype=F32)
    for b in range(nb):
        blk = v[:, b * block:min((b + 1) * block, K)]
        amax = np.abs(blk).max(axis=1).astype(np.float64)
        sc = np.where(amax > 0, amax / 448.0, 1.0).astype(F32)
        scales[:, b] = sc
        q = (blk / sc[:, None]).astype(F32)
        out[:, b * block:min((b + 1) * block, K)] = np.clip(q, -FP8_E4M3_MAX, FP8_E4M3_MAX)
    return out, scales


def nvfp4_dequant(packed: np.ndarray, scales: np.ndarray, group: int = 16) -> np.ndarray:
    """packed [M, N/2] uint8 (code of column 2i in the low nibble, 2i+1 in the
    high one), scales [M, N/group] -> float32 E2M1 value * scale
    (test_reference.py:19-53)."""
    p = np.asarray(packed, dtype=np.uint8)
    M, half = p.shape
    codes = np.empty((M, 2 * half), dtype=np.uint8)
    codes[:, 0::2] = p & 0x0F
    codes[:, 1::2] = p >> 4
    s = np.asarray(scales, dtype=F32)
    cols = np.arange(2 * half) // group
    return (E2M1_VALUES[codes] * s[:, cols]).astype(F32)


# ---------------------------------------------------------------------------
# E4M3 codes (OCP 8-bit floating point, E4M3 variant)
# ---------------------------------------------------------------------------

def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    """uint8 E4M3 codes -> float32 values (NaN for S.1111.111)."""
    c = np.asarray(codes, dtype=np.uint8).astype(np.int32)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 0x7
    mag = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * 2.0 ** (e - 7))
    val = sign * mag
    val = np.where((e == 15) & (m == 7), np.nan, val)
    return val.astype(F32)


_FINITE_CODES = np.array([c for c in range(128) if c != 0x7F], dtype=np.uint8)
_FINITE_VALUES = e4m3_decode(_FINITE_CODES).astype(np.float64)  # ascending, 0 .. 448


def e4m3_encode(x: np.ndarray, saturate: bool = True) -> np.ndarray:
    """float32 -> uint8 E4M3 code, round to nearest, ties to the even code
    (even mantissa).  Magnitudes past 448 saturate to 448 (saturate=True) or
    become NaN (0x7F with the sign); NaN stays NaN."""
    v = np.asarray(x, dtype=np.float64)
    a = np.abs(v)
    # index of the largest finite magnitude <= a, then pick the nearer of it
    # and the next one; on a tie the even code (even mantissa bit 0) wins
    lo = np.clip(np.searchsorted(_FINITE_VALUES, a, side="right") - 1, 0, len(_FINITE_VALUES) - 1)
    hi = np.minimum(lo + 1, len(_FINITE_VALUES) - 1)
    dlo = a - _FINITE_VALUES[lo]
    dhi = _FINITE_VALUES[hi] - a
    take_hi = (dhi < dlo) | ((dhi == dlo) & (hi != lo) & (_FINITE_CODES[hi] % 2 == 0))
    code = np.where(take_hi, _FINITE_CODES[hi], _FINITE_CODES[lo]).astype(np.uint8)
    # past the largest finite value: saturate, or NaN when the value rounds beyond 448
    over = a > 448.0
    if not saturate:
        # past 448 + half an ulp (the tie at 464 goes to 448, the even code)
        # a value rounds to the next binade, which E4M3 lacks: NaN
        code = np.where(a > 464.0, np.uint8(0x7F), code)
    else:
        code = np.where(over, np.uint8(0x7E), code)
    code = np.where(np.isnan(v), np.uint8(0x7F), code)
    sign = np.where(np.signbit(v), np.uint8(0x80), np.uint8(0))
    return (code | sign).astype(np.uint8)


def e4m3_round(x: np.ndarray, saturate: bool = True) -> np.ndarray:
    """float32 -> the float32 value of its E4M3 code (e4m3_encode, decoded)."""
    return e4m3_decode(e4m3_encode(x, saturate))
