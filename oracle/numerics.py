"""Rounding helpers of the oracle (numpy, bit-level).

bf16: round-to-nearest-even of the fp32 bit pattern (the conversion torch and
CUDA's cvt.rn.bf16.f32 perform). fp16: numpy's IEEE half conversion (RTNE).
fp8 e4m3 ("fn": no infinities, max 448): RTNE with saturation to +-448, the
conversion of cvt.rn.satfinite.e4m3x2.f32 that Triton uses for fp32->e4m3.
"""
from __future__ import annotations

import numpy as np


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(x))


def f16_to_f32(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def round_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def _e4m3_table() -> np.ndarray:
    vals = np.zeros(256, np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            vals[b] = np.nan
        elif e == 0:
            vals[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            vals[b] = s * (1 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3 = _e4m3_table()
_POS = E4M3[:0x7F]  # 0x00..0x7E, increasing, 0 .. 448


def e4m3_to_f32(bits: np.ndarray) -> np.ndarray:
    return E4M3[bits.astype(np.uint8)]


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32)
    a = np.abs(x).astype(np.float64)
    sign = (np.signbit(x)).astype(np.uint8) << 7
    a = np.minimum(a, 448.0)
    hi = np.searchsorted(_POS, a, side="left").clip(0, 0x7E)  # first >= a
    lo = np.maximum(hi - 1, 0)
    dlo = a - _POS[lo]
    dhi = _POS[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(a == _POS[hi], hi, code).astype(np.uint8)
    out = code | sign
    out = np.where(np.isnan(x), np.uint8(0x7F), out)
    return out.astype(np.uint8)


# per-dtype (raw numpy dtype, to_f32, from_f32, round_f32)
DTYPES = {
    "bf16": (np.uint16, bf16_to_f32, f32_to_bf16, round_bf16),
    "f16": (np.uint16, f16_to_f32, f32_to_f16, round_f16),
    "f32": (np.float32, lambda b: b.view(np.float32), lambda x: np.asarray(x, np.float32),
            lambda x: np.asarray(x, np.float32)),
    "fp8": (np.uint8, e4m3_to_f32, f32_to_e4m3, lambda x: e4m3_to_f32(f32_to_e4m3(x))),
}
