"""MLX affine quantization format helpers (host side, numpy / torch).

Format (MLX ``mx.quantize(..., mode="affine")``, as stored in Runnel's
checkpoints and produced by ``fuse_routed_gate_up``):

* codes: ``uint32`` words holding ``32 // bits`` codes each, code ``j`` of a
  word in bits ``[bits*j, bits*(j+1))`` (LSB first);
* ``scales`` and ``biases``: bf16, one per ``group_size`` consecutive inputs of
  a row; the dequantised weight is ``scale * code + bias``.

bf16 values on the host are carried as ``uint16`` bit patterns in numpy.
"""
from __future__ import annotations

import numpy as np

GROUP_SIZE = 64


def f32_to_bf16_bits(a) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns; inf/nan pass through."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    special = (u & 0x7F800000) == 0x7F800000
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(special, (u >> 16).astype(np.uint16), rounded)


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """Pack integer codes ``[..., K]`` into uint32 words ``[..., K*bits/32]``."""
    if bits not in (4, 8):
        raise ValueError("bits must be 4 or 8")
    per = 32 // bits
    c = np.ascontiguousarray(codes, dtype=np.uint32)
    if c.shape[-1] % per:
        raise ValueError(f"last dimension must be a multiple of {per}")
    c = c.reshape(*c.shape[:-1], c.shape[-1] // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    return np.bitwise_or.reduce(c << shifts, axis=-1).astype(np.uint32)


def unpack_codes(words: np.ndarray, bits: int) -> np.ndarray:
    """Inverse of :func:`pack_codes`: ``[..., W]`` uint32 -> ``[..., W*32/bits]`` uint8."""
    per = 32 // bits
    w = np.ascontiguousarray(words, dtype=np.uint32)
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    mask = np.uint32((1 << bits) - 1)
    out = (w[..., None] >> shifts) & mask
    return out.reshape(*w.shape[:-1], w.shape[-1] * per).astype(np.uint8)


def dequantize(words, scales_bf16, biases_bf16, bits: int, group: int = GROUP_SIZE) -> np.ndarray:
    """fp32 weights ``scale * code + bias`` for inspection and small references."""
    q = unpack_codes(words, bits).astype(np.float32)
    s = bf16_bits_to_f32(scales_bf16)
    b = bf16_bits_to_f32(biases_bf16)
    q = q.reshape(*q.shape[:-1], q.shape[-1] // group, group)
    return (q * s[..., None] + b[..., None]).reshape(*q.shape[:-2], -1)


def quantize(w: np.ndarray, bits: int, group: int = GROUP_SIZE):
    """Affine-quantize fp32 rows ``[..., K]`` per ``group`` (min/max, as MLX does).

    Returns ``(words uint32, scales bf16 bits, biases bf16 bits)``.  Scale is
    ``(max - min) / (2^bits - 1)`` and bias is the group minimum, both
    rounded to bf16; codes are ``round((w - bias) / scale)`` clipped to range.
    """
    w = np.asarray(w, dtype=np.float32)
    K = w.shape[-1]
    if K % group:
        raise ValueError("last dimension must be a multiple of the group size")
    g = w.reshape(*w.shape[:-1], K // group, group)
    lo = g.min(axis=-1)
    hi = g.max(axis=-1)
    n = (1 << bits) - 1
    scale = np.maximum((hi - lo) / n, 1e-8)
    s_bits = f32_to_bf16_bits(scale)
    b_bits = f32_to_bf16_bits(lo)
    s = bf16_bits_to_f32(s_bits)
    b = bf16_bits_to_f32(b_bits)
    q = np.clip(np.rint((g - b[..., None]) / s[..., None]), 0, n).astype(np.uint32)
    return pack_codes(q.reshape(w.shape), bits), s_bits, b_bits
