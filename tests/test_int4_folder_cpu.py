"""The INT4 base folder read straight into the kernel layout (jeff_b200.int4_folder), on the CPU: the folder's byte
layout against the golden vectors the reference's own code produced (tests/golden/make_golden.py: pack_int4 of the
same integers), a fused group's kernel words and scales equal to the reference's pack_kernel output for those
integers, a written file read back, and each of the reference's refusals (engine/int4.py:280-323)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from jeff_b200 import int4, int4_folder
from jeff_b200.prefix_pool import EngineError


@pytest.fixture(scope="module")
def g4() -> dict[str, np.ndarray]:
    return dict(np.load(GOLDEN / "int4_golden.npz"))


def bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def test_folder_bytes_match_the_reference(g4) -> None:
    u = (torch.from_numpy(g4["q"]).to(torch.int16) + 8).to(torch.uint8)
    assert np.array_equal(int4_folder.pack_folder(u).numpy(), g4["folder"])
    assert torch.equal(int4_folder.unpack_folder(torch.from_numpy(g4["folder"])), u)


def test_a_group_from_the_bytes_equals_the_reference_kernel_layout(g4) -> None:
    found = {"m": (torch.from_numpy(g4["folder"]), bf16(g4["scales"]))}
    packed = int4_folder.pack_group(found, ["m"])
    assert np.array_equal(packed.words.numpy(), g4["words"])
    assert np.array_equal(packed.scales.view(torch.int16).numpy().view(np.uint16), g4["kscales"])
    assert packed.zeros is None and packed.group == 64 and packed.out == 128
    deq = int4.dequantize(*int4.unpack_kernel(packed)[:2], None, 64)
    assert np.array_equal(deq.view(torch.int16).numpy().view(np.uint16), g4["deq"])


def _matrices(g: torch.Generator) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
    out = {}
    shapes = {"layers.0.q_proj": (96, 128), "layers.0.k_proj": (32, 128), "layers.0.o_proj": (128, 64)}
    for name, (o, i) in shapes.items():
        q = torch.randint(-8, 8, (o, i), generator=g, dtype=torch.int8)
        s = (torch.rand(o, i // 64, generator=g) * 0.01 + 1e-3).to(torch.bfloat16)
        out[name] = (q, s)
    return out


def test_a_written_file_reads_back_into_fused_groups(tmp_path) -> None:
    mats = _matrices(torch.Generator().manual_seed(3))
    digest = int4_folder.write_int4_file(tmp_path, mats)
    shapes = {name: tuple(q.shape) for name, (q, _) in mats.items()}
    found = int4_folder.read_int4_file(tmp_path, shapes, digest)
    groups = int4_folder.kernel_groups(found, {"qk": ["layers.0.q_proj", "layers.0.k_proj"], "o": ["layers.0.o_proj"]})
    q = torch.cat([mats["layers.0.q_proj"][0], mats["layers.0.k_proj"][0]])
    s = torch.cat([mats["layers.0.q_proj"][1], mats["layers.0.k_proj"][1]])
    want = int4.pack_kernel((q.to(torch.int16) + 8).to(torch.uint8), s, None, 64)
    assert torch.equal(groups["qk"].words, want.words) and torch.equal(groups["qk"].scales, want.scales)
    assert groups["qk"].out == 128 and groups["qk"].columns == 128 and groups["o"].columns == 128


def test_the_reference_refusals(tmp_path) -> None:
    g = torch.Generator().manual_seed(4)
    mats = _matrices(g)
    digest = int4_folder.write_int4_file(tmp_path, mats)
    shapes = {name: tuple(q.shape) for name, (q, _) in mats.items()}
    with pytest.raises(EngineError, match="has no int4.safetensors"):
        int4_folder.read_int4_file(tmp_path / "elsewhere", shapes, digest)
    with pytest.raises(EngineError, match="is not the one this INT4 base was made with"):
        int4_folder.read_int4_file(tmp_path, shapes, "0" * 64)
    with pytest.raises(EngineError, match="lacks 2 tensors"):
        int4_folder.read_int4_file(tmp_path, {**shapes, "layers.0.v_proj": (32, 128)}, digest)
    with pytest.raises(EngineError, match="holds 2 tensors that are not"):
        int4_folder.read_int4_file(tmp_path, {k: v for k, v in shapes.items() if k != "layers.0.o_proj"}, digest)
    with pytest.raises(EngineError, match=r"needs \(96, 128\)"):
        int4_folder.read_int4_file(tmp_path, {**shapes, "layers.0.q_proj": (96, 256)}, digest)
    bad = dict(mats)
    bad["layers.0.k_proj"] = (bad["layers.0.k_proj"][0], -bad["layers.0.k_proj"][1])
    digest = int4_folder.write_int4_file(tmp_path, bad)
    with pytest.raises(EngineError, match="not finite and positive"):
        int4_folder.read_int4_file(tmp_path, shapes, digest)
    with pytest.raises(ValueError, match="int4-g64 holds"):
        int4_folder.write_int4_file(tmp_path, {"m": (torch.full((2, 64), 9, dtype=torch.int8),
                                                     torch.ones(2, 1, dtype=torch.bfloat16))})
