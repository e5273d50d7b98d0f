"""Bit-level rounding helpers for the CPU oracle (numpy only).

bf16 / fp16 / fp8-e4m3fn rounding as performed by the reference's storage dtypes:
the NKI kernels round probabilities to bf16 (attention_const_max.py:318-327),
shifted scores to fp16 (attention_const_max.py:311-327), the softmax bound c to
bf16 (ring_attention_const_max_fwd.py:585-591) and ROW-quantised activations to
OCP e4m3fn (adaln_quant_torch.py:33-36, adaln_quant.py:472-537).
"""

from __future__ import annotations

import numpy as np

FP8_E4M3FN_MAX = 448.0  # adaln_quant_torch.py:27
FP8_E4M3_MAX = 240.0  # adaln_quant_torch.py:28


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even), returned as float32."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    bias = 0x7FFF + ((u >> 16) & 1)
    r = ((u + bias) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32)
    # NaN stays NaN (never produced by the oracle's inputs).
    return np.where(np.isnan(a), a, out)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bfloat16 bit patterns (round-to-nearest-even)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    """uint16 bfloat16 bit patterns -> float32."""
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


def fp16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to IEEE fp16 (numpy's native RNE), returned as float32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def e4m3fn_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to OCP fp8 e4m3fn, saturating at +-448, returned as float32.

    e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa bits; normals from 2^-6, subnormal
    spacing 2^-9, largest finite 448, no infinities. Round-to-nearest-even. Values
    beyond 448 saturate (the quantiser never produces them: codes are y / (amax/448)).
    """
    a = np.asarray(x, dtype=np.float32).astype(np.float64)
    m = np.abs(a)
    _, ex = np.frexp(np.where(m > 0, m, 1.0))
    # floor(log2(m)) = ex - 1; spacing of the binade is 2^(floor-3); subnormal spacing 2^-9.
    e = np.maximum(ex - 1, -6)
    spacing = np.ldexp(1.0, (e - 3).astype(np.int64))
    q = np.rint(m / spacing) * spacing
    q = np.minimum(q, FP8_E4M3FN_MAX)
    return np.copysign(q, a).astype(np.float32)


def e4m3fn_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint8 e4m3fn bit patterns (round-to-nearest-even, saturating)."""
    q = e4m3fn_round(x).astype(np.float64)
    sign = (q < 0) | ((q == 0) & np.signbit(q))
    m = np.abs(q)
    out = np.zeros(m.shape, dtype=np.uint8)
    nz = m > 0
    _, ex = np.frexp(np.where(nz, m, 1.0))
    e = ex - 1
    normal = nz & (e >= -6)
    sub = nz & (e < -6)
    frac = np.where(normal, m / np.ldexp(1.0, e) - 1.0, 0.0)
    man = np.rint(frac * 8).astype(np.int64)
    out = np.where(normal, ((e + 7) << 3) | man, out)
    out = np.where(sub, np.rint(m / 2.0 ** -9).astype(np.int64), out)
    out = out.astype(np.uint8) | (sign.astype(np.uint8) << 7)
    return out


def e4m3fn_from_bits(b: np.ndarray) -> np.ndarray:
    """uint8 e4m3fn bit patterns -> float32 (0x7F/0xFF decode as NaN)."""
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.ldexp(1.0, e - 7))
    val = np.where((e == 0xF) & (m == 0x7), np.nan, val)
    return (sign * val).astype(np.float32)
