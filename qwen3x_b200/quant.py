"""Host-side block formats and quantizers for synthetic inputs (numpy).

The packed formats are model.bin's (q8.h:10-15, q4.h:29-42):
  Q8_0: {fp16 scale, int8[32]}            34 bytes per 32 weights
  Q4_0: {fp16 scale, u8[16]}              18 bytes per 32 weights; byte i holds
        element i (low nibble) and element i + 16 (high nibble); value = n - 8.

Encoders:
  quantize_q8_0        scripts/pack_weights.py:299-318 arithmetic (d = max|w|/127,
                       q = round-half-away(w * (1/d)), clipped to +-127) -- this is
                       also the synthetic-input encoder of the benchmark configs.
  quantize_q4_0        the benchmark configs' Q4_0 encoder: d = max|w|/8,
                       q = clamp(round(w/d) + 8, 0, 15).
  quantize_q4_0_ggml   scripts/pack_weights.py:321-343 (ggml): d = signed max/-8,
                       q = min(15, trunc(w/d + 8.5)).
All produce valid blocks for the same decode rule; the kernels do not care
which encoder made them.
"""
from __future__ import annotations

import numpy as np

BLOCK = 32
Q8_DTYPE = np.dtype([("scale", "<u2"), ("values", "i1", (BLOCK,))])
Q4_DTYPE = np.dtype([("scale", "<u2"), ("values", "u1", (BLOCK // 2,))])
assert Q8_DTYPE.itemsize == 34 and Q4_DTYPE.itemsize == 18

BF16, Q8_0, Q4_0 = 0, 1, 2


def gaussian(shape, seed: int, std: float = 1.0) -> np.ndarray:
    """Seeded N(0, std^2) FP32 samples (numpy PCG64 `default_rng(seed)`)."""
    rng = np.random.default_rng(seed)
    out = rng.standard_normal(size=shape, dtype=np.float32)
    if std != 1.0:
        out *= np.float32(std)
    return out


def _blocks(values: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float32)
    if v.shape[-1] % BLOCK:
        raise ValueError("last dimension must be a multiple of 32")
    if not np.isfinite(v).all():
        raise ValueError("non-finite weight")
    return v.reshape(-1, BLOCK)


def _round_half_away(x: np.ndarray) -> np.ndarray:
    return np.copysign(np.floor(np.abs(x) + np.float32(0.5)), x)


def _inverse(scale: np.ndarray) -> np.ndarray:
    inv = np.zeros_like(scale)
    np.divide(np.float32(1.0), scale, out=inv, where=scale != 0)
    return inv


def quantize_q8_0(values: np.ndarray) -> np.ndarray:
    """FP32 [..., K] -> Q8_0 blocks (uint8 bytes, shape [..., K/32*34])."""
    v = _blocks(values)
    scale = np.max(np.abs(v), axis=1) / np.float32(127.0)
    q = np.clip(_round_half_away(v * _inverse(scale)[:, None]), -127, 127).astype(np.int8)
    blocks = np.empty(v.shape[0], dtype=Q8_DTYPE)
    blocks["scale"] = scale.astype("<f2").view("<u2")
    blocks["values"] = q
    return blocks.view(np.uint8).reshape(*values.shape[:-1], -1)


def _pack_q4(scale: np.ndarray, q: np.ndarray, shape) -> np.ndarray:
    q = q.astype(np.uint8)
    blocks = np.empty(q.shape[0], dtype=Q4_DTYPE)
    blocks["scale"] = scale.astype("<f2").view("<u2")
    blocks["values"] = q[:, :16] | (q[:, 16:] << 4)
    return blocks.view(np.uint8).reshape(*shape[:-1], -1)


def quantize_q4_0(values: np.ndarray) -> np.ndarray:
    """Benchmark-config Q4_0 encoder: d = max|w|/8, q = clamp(round(w/d)+8, 0, 15)."""
    v = _blocks(values)
    scale = np.max(np.abs(v), axis=1) / np.float32(8.0)
    q = np.clip(_round_half_away(v * _inverse(scale)[:, None]) + 8, 0, 15)
    return _pack_q4(scale, q, values.shape)


def quantize_q4_0_ggml(values: np.ndarray) -> np.ndarray:
    """ggml Q4_0 (scripts/pack_weights.py:321-343) applied to FP32 values."""
    v = _blocks(values)
    largest = np.argmax(np.abs(v), axis=1)
    scale = v[np.arange(v.shape[0]), largest] / np.float32(-8.0)
    q = np.minimum(15, np.trunc(v * _inverse(scale)[:, None] + np.float32(8.5)))
    return _pack_q4(scale, q, values.shape)


def quantize(values: np.ndarray, mtype: int) -> np.ndarray:
    if mtype == Q8_0:
        return quantize_q8_0(values)
    if mtype == Q4_0:
        return quantize_q4_0(values)
    if mtype == BF16:
        return to_bf16_bits(values).view(np.uint8).reshape(*values.shape[:-1], -1)
    raise ValueError(mtype)


def to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """FP32 -> BF16 bits by truncation (the reference packer's source format)."""
    return (np.ascontiguousarray(values, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def dequantize(packed: np.ndarray, mtype: int, rows: int, cols: int) -> np.ndarray:
    """Packed bytes -> FP32 [rows, cols] (value = f16(d) * q, exact in FP32)."""
    raw = np.ascontiguousarray(packed).reshape(-1).view(np.uint8)
    if mtype == Q8_0:
        b = raw.view(Q8_DTYPE)
        d = b["scale"].view("<f2").astype(np.float32)
        return (d[:, None] * b["values"].astype(np.float32)).reshape(rows, cols)
    if mtype == Q4_0:
        b = raw.view(Q4_DTYPE)
        d = b["scale"].view("<f2").astype(np.float32)
        lo = (b["values"] & 15).astype(np.float32) - 8
        hi = (b["values"] >> 4).astype(np.float32) - 8
        return (d[:, None] * np.concatenate([lo, hi], axis=1)).reshape(rows, cols)
    if mtype == BF16:
        return bf16_to_f32(raw.view("<u2")).reshape(rows, cols)
    raise ValueError(mtype)


def packed_row_bytes(mtype: int, cols: int) -> int:
    if mtype == Q8_0:
        return cols // BLOCK * 34
    if mtype == Q4_0:
        return cols // BLOCK * 18
    return cols * 2
