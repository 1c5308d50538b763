"""The int4 weight formats of the decision hot path, host side (load time only).

Two formats are held, both in the reference's kernel word layout (reference
runtime/python/src/jeff_runtime/engine/int4.py:215-262, `KernelInt4`, `pack_kernel`, `unpack_kernel`):

- words: int32 (K / 8, columns); word i of column c holds the 4-bit integers of inputs 8i .. 8i + 7, input 8i + j in
  bits 4j .. 4j + 3, stored unsigned (u = q + 8 for the symmetric format);
- scales: bfloat16 (K / G, columns), the scale of inputs Gg .. Gg + G - 1 of column c at (g, c);
- zeros: bfloat16 (K / G, columns) or None, an integer-valued zero point per group;
- columns: the outputs rounded up to a multiple of 64; padding columns hold weight 0 (u = 8, scale 1, zero 8).

"int4-g64" (group 64, symmetric, no zero: the reference's only format, int4.py:1-18) dequantises to
bf16(fp32(u - 8) * fp32(s)), exactly `int4.dequantize` (int4.py:203-208). "int4-g128z" (group 128, asymmetric u4
with a bf16 zero point per group: the benchmark configuration) dequantises to bf16(fp32(u - z) * fp32(s)); u - z is a
small integer, so the product is exact in float32 before its single rounding, the same rule as the symmetric format.
The device kernels apply the same formula; `tests/` checks them bit for bit against the CPU oracle."""

from __future__ import annotations

from dataclasses import dataclass

import torch

from jeff_b200.constants import KERNEL_COLUMNS, WORD

LOW, HIGH = -8, 7


@dataclass(frozen=True)
class PackedInt4:
    """One fused group's integers in the kernel layout (module docstring). `out`: the real outputs."""
    words: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor | None
    group: int
    out: int

    @property
    def columns(self) -> int:
        return int(self.words.shape[1])

    @property
    def inputs(self) -> int:
        return int(self.words.shape[0]) * WORD

    def nbytes(self) -> int:
        total = self.words.numel() * 4 + self.scales.numel() * 2
        return total + (self.zeros.numel() * 2 if self.zeros is not None else 0)

    def to(self, device: str | torch.device) -> "PackedInt4":
        return PackedInt4(self.words.to(device), self.scales.to(device),
                          None if self.zeros is None else self.zeros.to(device), self.group, self.out)


def quantize_symmetric(w: torch.Tensor, group: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """Round to nearest, symmetric: scale bf16(max |w| / 7) per group (1 for an all-zero group), integers
    round(w / s) clamped to [-8, 7] (the reference's `quantize.round_to_nearest`, quantize.py:259-267, with the group
    as a parameter). Returns int8 integers (out, in) and bf16 scales (out, in / group)."""
    groups = w.float().reshape(w.shape[0], -1, group)
    top = groups.abs().amax(-1)
    scales = torch.where(top == 0, torch.ones_like(top), top / HIGH).to(torch.bfloat16).float()
    q = torch.clamp(torch.round(groups / scales[..., None]), LOW, HIGH).reshape(w.shape)
    return q.to(torch.int8), scales.to(torch.bfloat16)


def quantize_asymmetric(w: torch.Tensor, group: int = 128) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Round to nearest, asymmetric u4: per group s = bf16((max - min) / 15) (1 when max == min), zero
    z = clamp(round(-min / s), 0, 15), u = clamp(round(w / s) + z, 0, 15). Returns uint8 integers u (out, in), bf16
    scales and bf16 zeros (out, in / group)."""
    groups = w.float().reshape(w.shape[0], -1, group)
    lo, hi = groups.amin(-1), groups.amax(-1)
    span = hi - lo
    scales = torch.where(span == 0, torch.ones_like(span), span / 15).to(torch.bfloat16).float()
    zeros = torch.clamp(torch.round(-lo / scales), 0, 15)
    u = torch.clamp(torch.round(groups / scales[..., None]) + zeros[..., None], 0, 15).reshape(w.shape)
    return u.to(torch.uint8), scales.to(torch.bfloat16), zeros.to(torch.bfloat16)


def pack_kernel(u: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None, group: int) -> PackedInt4:
    """Unsigned 4-bit integers u (out, in) in [0, 15] with their scales (and zeros) (out, in / group) in the kernel
    layout. For the symmetric format pass u = q + 8 and zeros None. The word layout is the reference's
    (int4.py:233-255): columns padded to a multiple of 64 with zero weights."""
    out, inputs = u.shape
    if inputs % group or group % WORD or group not in (64, 128):
        raise ValueError(f"pack_kernel: inputs ({inputs}) must be a multiple of the group, and the group 64 or 128; "
                         f"got group {group}")
    if int(u.min()) < 0 or int(u.max()) > 15:
        raise ValueError(f"pack_kernel: integers from {int(u.min())} to {int(u.max())}; 4-bit storage holds 0..15")
    if scales.dtype != torch.bfloat16 or tuple(scales.shape) != (out, inputs // group):
        raise ValueError(f"pack_kernel: scales must be bfloat16 ({out}, {inputs // group}); got {scales.dtype} "
                         f"{tuple(scales.shape)}")
    if zeros is not None and (zeros.dtype != torch.bfloat16 or zeros.shape != scales.shape):
        raise ValueError("pack_kernel: zeros must be bfloat16 with the scales' shape")
    columns = -(-out // KERNEL_COLUMNS) * KERNEL_COLUMNS
    stored = torch.full((columns, inputs), 8, dtype=torch.int64)
    stored[:out] = u.to(torch.int64)
    stored = stored.T.contiguous()                       # (in, columns)
    words = torch.zeros(inputs // WORD, columns, dtype=torch.int64)
    for j in range(WORD):
        words |= stored[j::WORD] << (4 * j)
    words = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)
    padded_s = torch.ones(columns, inputs // group, dtype=torch.bfloat16)
    padded_s[:out] = scales
    padded_z = None
    if zeros is not None:
        padded_z = torch.full((columns, inputs // group), 8.0, dtype=torch.bfloat16)
        padded_z[:out] = zeros
        padded_z = padded_z.T.contiguous()
    return PackedInt4(words, padded_s.T.contiguous(), padded_z, group, out)


def unpack_kernel(packed: PackedInt4) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """pack_kernel's inverse: u (out, in) uint8, scales and zeros (out, in / group), padding columns dropped."""
    words = packed.words.to(torch.int64) & 0xFFFFFFFF
    nib = torch.stack([(words >> (4 * j)) & 0xF for j in range(WORD)], dim=1)   # (in/8, 8, columns)
    u = nib.reshape(-1, words.shape[1]).T[:packed.out].to(torch.uint8).contiguous()
    zeros = None if packed.zeros is None else packed.zeros.T[:packed.out].contiguous()
    return u, packed.scales.T[:packed.out].contiguous(), zeros


def dequantize(u: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None, group: int) -> torch.Tensor:
    """bf16(fp32(u - z) * fp32(s)) per weight (z = 8 without zeros): one rounding, as the kernels compute it."""
    out, inputs = u.shape
    z = torch.full_like(scales, 8.0, dtype=torch.float32) if zeros is None else zeros.float()
    q = u.to(torch.float32).reshape(out, inputs // group, group) - z[..., None]
    return (q * scales.float()[..., None]).reshape(out, inputs).to(torch.bfloat16)


def quantize_pack(w: torch.Tensor, fmt: str) -> tuple[PackedInt4, torch.Tensor]:
    """Quantise a float matrix (out, in) in format "g64" (symmetric, the reference's int4-g64) or "g128z"
    (asymmetric with zeros) and pack it; also returns the dequantised bf16 weights (the matrix the model holds)."""
    if fmt == "g64":
        q, s = quantize_symmetric(w, 64)
        u = (q.to(torch.int16) + 8).to(torch.uint8)
        return pack_kernel(u, s, None, 64), dequantize(u, s, None, 64)
    if fmt == "g128z":
        u, s, z = quantize_asymmetric(w, 128)
        return pack_kernel(u, s, z, 128), dequantize(u, s, z, 128)
    raise ValueError(f"Unknown int4 format {fmt!r}; expected 'g64' or 'g128z'")
