"""TEST INFRASTRUCTURE ONLY (the checker, never the product): numpy restatement of the int4 kernel layout.

Follows the reference's runtime/python/src/jeff_runtime/engine/int4.py:
- pack_int4 / unpack_int4 (:183-200): the folder layout, uint8 (out, in / 2), low nibble first, each q + 8;
- pack_kernel / unpack_kernel (:233-262): int32 words (in / 8, columns), input 8i + j of column c in bits 4j .. 4j + 3
  of word (i, c); columns padded to a multiple of 64 with q = 0 and scale 1;
- dequantize (:203-208): bf16(fp32(q) * fp32(s)), one rounding.
The group-128-with-zero format extends these with zeros (group, column) and bf16(fp32(u - z) * fp32(s)).

bfloat16 values are held as uint16 bit patterns; `to_bf16_bits` rounds float32 to nearest even, the IEEE rule
torch and the CUDA conversion intrinsics use."""

from __future__ import annotations

import numpy as np

WORD = 8
COLUMNS = 64


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return ((u >> 16) & 0xFFFF).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def pack_int4(q: np.ndarray) -> np.ndarray:
    """int8 (out, in) in [-8, 7] -> uint8 (out, in / 2), low nibble first, q + 8."""
    s = (q.astype(np.int16) + 8).astype(np.uint8)
    return (s[:, 0::2] | (s[:, 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    lo = (packed & 0xF).astype(np.int8) - 8
    hi = (packed >> 4).astype(np.int8) - 8
    return np.stack([lo, hi], -1).reshape(packed.shape[0], packed.shape[1] * 2)


def pack_kernel(u: np.ndarray, scale_bits: np.ndarray, zero_bits: np.ndarray | None
                ) -> tuple[np.ndarray, np.ndarray, np.ndarray | None]:
    """Unsigned integers u (out, in) in [0, 15] and per-group scale (and zero) bit patterns (out, in / group) ->
    (words int32 (in / 8, columns), scales uint16 (in / group, columns), zeros or None)."""
    out, inputs = u.shape
    columns = -(-out // COLUMNS) * COLUMNS
    stored = np.full((columns, inputs), 8, dtype=np.uint32)
    stored[:out] = u
    stored = stored.T                                  # (in, columns)
    words = np.zeros((inputs // WORD, columns), dtype=np.uint32)
    for j in range(WORD):
        words |= stored[j::WORD] << np.uint32(4 * j)
    groups = scale_bits.shape[1]
    s = np.full((columns, groups), 0x3F80, dtype=np.uint16)   # bf16 1.0
    s[:out] = scale_bits
    z = None
    if zero_bits is not None:
        z = np.full((columns, groups), 0x4100, dtype=np.uint16)  # bf16 8.0
        z[:out] = zero_bits
        z = np.ascontiguousarray(z.T)
    return words.view(np.int32), np.ascontiguousarray(s.T), z


def unpack_kernel(words: np.ndarray, out: int) -> np.ndarray:
    """words (in / 8, columns) -> u (out, in) uint8 in [0, 15]."""
    w = words.view(np.uint32)
    nib = np.stack([(w >> np.uint32(4 * j)) & 0xF for j in range(WORD)], axis=1)   # (in/8, 8, columns)
    return nib.reshape(-1, w.shape[1]).T[:out].astype(np.uint8)


def dequantize(u: np.ndarray, scale_bits: np.ndarray, zero_bits: np.ndarray | None, group: int) -> np.ndarray:
    """bf16 bit patterns (out, in) of bf16(fp32(u - z) * fp32(s)), z = 8 when there are no zeros."""
    out, inputs = u.shape
    s = bf16_to_f32(scale_bits)
    z = np.full(s.shape, 8.0, dtype=np.float32) if zero_bits is None else bf16_to_f32(zero_bits)
    q = u.astype(np.float32).reshape(out, inputs // group, group) - z[..., None]
    return to_bf16_bits((q * s[..., None]).reshape(out, inputs).astype(np.float32))


def dequantize_kernel_layout(words: np.ndarray, scale_bits: np.ndarray, zero_bits: np.ndarray | None,
                             group: int) -> np.ndarray:
    """The kernel layout dequantised to bf16 bits (columns, in): what a device dequantiser must produce, padding
    columns included."""
    columns = words.shape[1]
    u = unpack_kernel(words, columns)
    z = None if zero_bits is None else np.ascontiguousarray(zero_bits.T)
    return dequantize(u, np.ascontiguousarray(scale_bits.T), z, group)
