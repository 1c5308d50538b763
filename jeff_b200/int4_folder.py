"""The reference's INT4 base folder read straight into this library's kernel layout (load time, host side).

An INT4 base folder (the reference's runtime/python/src/jeff_runtime/engine/int4.py:1-18) keeps each matrix of the
text decoder in int4.safetensors as `<name>.qweight`, uint8 (out, in / 2), two 4-bit integers per byte with the
input of even index in the low nibble, each stored as q + 8, and `<name>.scales`, bfloat16 (out, in / 64): the
symmetric "int4-g64" format. The reference reads the integers back into bfloat16 weights bf16(q * s) for its
standard path (int4.py:341-359, load_int4_state_dict) and, for its fast path, checks a fused group's bfloat16
weights against its integers and packs them into its kernel layout (int4.py:264-277). This module goes from the
stored bytes to the kernel layout directly, one fused group at a time: no bfloat16 copy of the matrices is made.

read_int4_file applies the reference's checks to the file (int4.py:280-323): its sha256 must be the one the base's
record names, it must hold exactly a qweight and a scales tensor for each expected matrix, of the right dtypes and
shapes, with finite positive scales; anything else is an EngineError naming the problem, as in the reference.
write_int4_file writes the same layout (for fixtures and for bases quantised here)."""

from __future__ import annotations

import hashlib
from collections.abc import Mapping, Sequence
from pathlib import Path

import torch

from jeff_b200.int4 import HIGH, LOW, PackedInt4, pack_kernel
from jeff_b200.prefix_pool import EngineError

INT4_FILE = "int4.safetensors"
GROUP = 64


def file_sha256(path: Path) -> str:
    with Path(path).open("rb") as stream:
        return hashlib.file_digest(stream, "sha256").hexdigest()


def unpack_folder(qweight: torch.Tensor) -> torch.Tensor:
    """uint8 (out, in / 2), low nibble first -> the stored integers u = q + 8 as uint8 (out, in)."""
    lo = qweight & 0xF
    hi = qweight >> 4
    return torch.stack([lo, hi], dim=-1).reshape(qweight.shape[0], -1)


def pack_folder(u: torch.Tensor) -> torch.Tensor:
    """unpack_folder's inverse: stored integers u (out, in) in [0, 15] -> uint8 (out, in / 2)."""
    if u.shape[1] % 2:
        raise ValueError(f"pack_folder: {u.shape[1]} inputs; the folder stores two per byte")
    pairs = u.to(torch.uint8).reshape(u.shape[0], -1, 2)
    return (pairs[..., 0] | (pairs[..., 1] << 4)).contiguous()


def _check_matrix(name: str, shape: tuple[int, int], qweight: torch.Tensor, scales: torch.Tensor) -> None:
    out, inputs = shape
    if qweight.dtype != torch.uint8:
        raise EngineError(f"{INT4_FILE}: {name}.qweight is {qweight.dtype}; it must be uint8, two 4-bit integers per "
                          f"byte stored as q + 8 (so every integer is in [{LOW}, {HIGH}])")
    if tuple(qweight.shape) != (out, inputs // 2):
        raise EngineError(f"{INT4_FILE}: {name}.qweight has shape {tuple(qweight.shape)}; the {out} x {inputs} "
                          f"matrix needs ({out}, {inputs // 2})")
    if scales.dtype != torch.bfloat16:
        raise EngineError(f"{INT4_FILE}: {name}.scales is {scales.dtype}; it must be bfloat16")
    if tuple(scales.shape) != (out, inputs // GROUP):
        raise EngineError(f"{INT4_FILE}: {name}.scales has shape {tuple(scales.shape)}; the {out} x {inputs} matrix "
                          f"needs ({out}, {inputs // GROUP}), one scale per {GROUP} inputs")
    if not bool(torch.isfinite(scales).all()) or not bool((scales > 0).all()):
        raise EngineError(f"{INT4_FILE}: {name}.scales holds a scale that is not finite and positive")


def read_int4_file(folder: Path, matrices: Mapping[str, tuple[int, int]], int4_sha256: str
                   ) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
    """{matrix name: (qweight, scales)} from `folder`/int4.safetensors, every tensor checked (module docstring):
    `matrices` maps each expected matrix name to its (out, in); `int4_sha256` is the digest the base's record
    gives for the file."""
    from safetensors.torch import load_file

    path = Path(folder) / INT4_FILE
    if not path.is_file():
        raise EngineError(f"{folder} is an INT4 base but has no {INT4_FILE}")
    digest = file_sha256(path)
    if digest != int4_sha256:
        raise EngineError(f"{path} has sha256 {digest}, but the record names {int4_sha256}: the file is not the one "
                          "this INT4 base was made with")
    packed = load_file(str(path))
    wanted = {f"{name}.{part}" for name in matrices for part in ("qweight", "scales")}
    absent = sorted(wanted - set(packed))
    if absent:
        raise EngineError(f"{path} lacks {len(absent)} tensors ({', '.join(absent[:3])}"
                          f"{', ...' if len(absent) > 3 else ''}): each INT4 matrix needs its qweight and scales")
    surplus = sorted(set(packed) - wanted)
    if surplus:
        raise EngineError(f"{path} holds {len(surplus)} tensors that are not an INT4 matrix's qweight or scales "
                          f"({', '.join(surplus[:3])}{', ...' if len(surplus) > 3 else ''})")
    found = {}
    for name, shape in matrices.items():
        qweight, scales = packed[f"{name}.qweight"], packed[f"{name}.scales"]
        _check_matrix(name, shape, qweight, scales)
        found[name] = (qweight, scales)
    return found


def write_int4_file(folder: Path, matrices: Mapping[str, tuple[torch.Tensor, torch.Tensor]]) -> str:
    """Write {name: (q int8 (out, in) in [-8, 7], scales bfloat16 (out, in / 64))} as `folder`/int4.safetensors in
    the folder layout; returns the file's sha256 (what the base's record holds)."""
    from safetensors.torch import save_file

    tensors = {}
    for name, (q, scales) in matrices.items():
        if int(q.min()) < LOW or int(q.max()) > HIGH:
            raise ValueError(f"{name}: integers from {int(q.min())} to {int(q.max())}; int4-g64 holds {LOW}..{HIGH}")
        tensors[f"{name}.qweight"] = pack_folder((q.to(torch.int16) + 8).to(torch.uint8))
        tensors[f"{name}.scales"] = scales.to(torch.bfloat16).contiguous()
    path = Path(folder) / INT4_FILE
    Path(folder).mkdir(parents=True, exist_ok=True)
    save_file(tensors, str(path))
    return file_sha256(path)


def pack_group(found: Mapping[str, tuple[torch.Tensor, torch.Tensor]], names: Sequence[str]) -> PackedInt4:
    """One fused group (matrices reading the same input, concatenated along the output in `names` order) in the
    kernel layout, from the stored bytes: the same words and scales the reference's fast path packs from its
    checked bfloat16 copy (int4.py:264-277, pack_kernel), with no bfloat16 weights made on the way."""
    u = torch.cat([unpack_folder(found[name][0]) for name in names])
    scales = torch.cat([found[name][1] for name in names])
    return pack_kernel(u, scales, None, GROUP)


def kernel_groups(found: Mapping[str, tuple[torch.Tensor, torch.Tensor]],
                  groups: Mapping[str, Sequence[str]]) -> dict[str, PackedInt4]:
    """Every fused group {group key: its matrix names} of a read file in the kernel layout."""
    return {key: pack_group(found, names) for key, names in groups.items()}
