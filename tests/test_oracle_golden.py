"""The CPU oracle (oracle/) and the product's host-side int4 packer (jeff_b200.int4) against the golden vectors the
reference's own code produced (tests/golden/make_golden.py). CPU only."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from jeff_b200 import int4 as prod_int4
from jeff_b200 import synthetic
from oracle import int4_ref, model_ref


@pytest.fixture(scope="module")
def g4() -> dict[str, np.ndarray]:
    return dict(np.load(GOLDEN / "int4_golden.npz"))


def to_torch_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def test_oracle_pack_kernel_matches_the_reference(g4: dict[str, np.ndarray]) -> None:
    q = g4["q"]
    words, scales, zeros = int4_ref.pack_kernel((q.astype(np.int16) + 8).astype(np.uint8), g4["scales"], None)
    assert zeros is None
    assert np.array_equal(words, g4["words"])
    assert np.array_equal(scales, g4["kscales"])
    assert int(words[0, 0]) & 0xFFFFFFFF == 0xFED98710     # the reference's known-answer word
    w70, s70, _ = int4_ref.pack_kernel((g4["q70"].astype(np.int16) + 8).astype(np.uint8), g4["s70"], None)
    assert np.array_equal(w70, g4["words70"]) and np.array_equal(s70, g4["kscales70"])
    assert (w70[:, 70:].view(np.uint32) == 0x88888888).all()    # padding columns: every nibble 0 + 8
    assert (s70[:, 70:] == 0x3F80).all()                        # with scale 1
    assert np.array_equal(int4_ref.unpack_kernel(g4["words"], 128).astype(np.int16) - 8, q)


def test_oracle_folder_layout_and_dequantize_match_the_reference(g4: dict[str, np.ndarray]) -> None:
    assert np.array_equal(int4_ref.pack_int4(g4["q"]), g4["folder"])
    assert np.array_equal(int4_ref.unpack_int4(g4["folder"]), g4["q"])
    u = (g4["q"].astype(np.int16) + 8).astype(np.uint8)
    assert np.array_equal(int4_ref.dequantize(u, g4["scales"], None, 64), g4["deq"])
    u7 = np.full((1, 64), 15, dtype=np.uint8)
    assert np.array_equal(int4_ref.dequantize(u7, np.array([[0x3F81]], dtype=np.uint16), None, 64), g4["deq7"])


def test_product_packer_matches_the_reference(g4: dict[str, np.ndarray]) -> None:
    q = torch.from_numpy(g4["q"])
    u = (q.to(torch.int16) + 8).to(torch.uint8)
    packed = prod_int4.pack_kernel(u, to_torch_bf16(g4["scales"]), None, 64)
    assert np.array_equal(packed.words.numpy(), g4["words"])
    assert np.array_equal(packed.scales.view(torch.int16).numpy().view(np.uint16), g4["kscales"])
    back_u, back_s, back_z = prod_int4.unpack_kernel(packed)
    assert torch.equal(back_u, u) and back_z is None
    deq = prod_int4.dequantize(u, to_torch_bf16(g4["scales"]), None, 64)
    assert np.array_equal(deq.view(torch.int16).numpy().view(np.uint16), g4["deq"])
    rq, rs = prod_int4.quantize_symmetric(torch.from_numpy(g4["w_rtn"]), 64)
    assert np.array_equal(rq.numpy(), g4["q_rtn"])
    assert np.array_equal(rs.view(torch.int16).numpy().view(np.uint16), g4["s_rtn"])


def test_group128_zero_format_round_trips_and_matches_the_oracle() -> None:
    w = synthetic.normal(5, "g128z", (200, 512), 0.02)
    u, s, z = prod_int4.quantize_asymmetric(w, 128)
    packed = prod_int4.pack_kernel(u, s, z, 128)
    assert packed.words.shape == (64, 256) and packed.zeros is not None and packed.zeros.shape == (4, 256)
    bu, bs, bz = prod_int4.unpack_kernel(packed)
    assert torch.equal(bu, u) and torch.equal(bs, s) and bz is not None and torch.equal(bz, z)
    sb = s.view(torch.int16).numpy().view(np.uint16)
    zb = z.view(torch.int16).numpy().view(np.uint16)
    words, scales, zeros = int4_ref.pack_kernel(u.numpy(), sb, zb)
    assert np.array_equal(words, packed.words.numpy())
    assert zeros is not None and np.array_equal(zeros, packed.zeros.view(torch.int16).numpy().view(np.uint16))
    deq = prod_int4.dequantize(u, s, z, 128).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(deq, int4_ref.dequantize(u.numpy(), sb, zb, 128))
    # padding columns dequantise to exactly zero, and the whole layout to the oracle's
    full = int4_ref.dequantize_kernel_layout(words, scales, zeros, 128)
    assert np.array_equal(full[:200], deq) and not int4_ref.bf16_to_f32(full[200:]).any()
    # quantisation error: within one step per weight (the integer zero point can clip an extreme by up to a step),
    # plus the output's bf16 rounding
    err = (prod_int4.dequantize(u, s, z, 128).float() - w).abs().reshape(200, 4, 128)
    assert bool((err <= s.float()[..., None] + w.abs().reshape(200, 4, 128) * 2**-8).all())


def test_prefix_pool_layout_matches_the_reference() -> None:
    from jeff_b200.prefix_pool import FAST_PATH_SHAPES, pool_pages, prefix_pool_mb_for, prefixes_held

    ref = json.loads((GOLDEN / "pool_layout.json").read_text())
    s = FAST_PATH_SHAPES
    got = {"page_bytes": s.page_bytes, "state_pages": s.state_pages, "heads_per_page": s.heads_per_page,
           "conv_pages": s.conv_pages, "layers_per_conv_page": s.layers_per_conv_page, "fixed_pages": s.fixed_pages}
    assert got == {k: ref[k] for k in got}
    assert {t: s.pages_per_prefix(int(t)) for t in ref["pages_per_prefix"]} == ref["pages_per_prefix"]
    assert pool_pages(8192) == ref["pool_pages_8192"]
    assert prefixes_held(8192, 1000) == ref["prefixes_held_8192_1000"]
    assert {r: prefix_pool_mb_for(int(r)) for r in ref["prefix_pool_mb_for"]} == ref["prefix_pool_mb_for"]


def test_oracle_scan_matches_the_standard_path_chunked_scan() -> None:
    """The oracle's token-by-token rule against transformers' chunked torch_chunk_gated_delta_rule (the reference's
    standard path) from the same initial state: float32 both, so within float32 summation-order noise."""
    d = np.load(GOLDEN / "gdn_scan_golden.npz")
    q, k, v, beta = (to_torch_bf16(d[n]).float() for n in ("q", "k", "v", "beta"))
    o, s = model_ref.gdn_scan(q, k, v, torch.from_numpy(d["g"]), beta, torch.from_numpy(d["h0"]))
    torch.testing.assert_close(o, torch.from_numpy(d["o"]), rtol=1e-4, atol=2e-5)
    torch.testing.assert_close(s, torch.from_numpy(d["s"]), rtol=1e-4, atol=2e-5)


@pytest.fixture(scope="module")
def golden_model():
    meta = json.loads((GOLDEN / "model_golden.json").read_text())
    spec = synthetic.ModelSpec(layers=meta["layers"], vocab=meta["vocab"], fmt=meta["fmt"], seed=meta["seed"],
                               norm_noise=meta["norm_noise"])
    model = synthetic.make_model(spec)
    adapters = [synthetic.make_adapter(model, i, seed=meta["seed"] + i) for i in meta["adapters"]]
    return model, adapters, dict(np.load(GOLDEN / "model_golden.npz"))


def test_synthetic_weights_regenerate_bit_for_bit(golden_model) -> None:
    import zlib

    model, _, g = golden_model
    got = {}
    for layer in model.layers:
        for grp in layer.groups.values():
            got[grp.names[0]] = zlib.crc32(grp.W.contiguous().view(torch.int16).numpy().tobytes())
    assert got == dict(zip(g["crc_names"].tolist(), g["crc_values"].tolist()))


def _rows(model, adapters, g, split: bool):
    heads = [synthetic.base_head(model)] + [(a.readout, a.temperature) for a in adapters]
    ids = g["ids"].tolist()
    rows_out, off = [], 0
    prefixes = []
    for adapter, plen, nlen, count in g["rows"].tolist():
        row_ids = ids[off:off + plen + nlen]
        off += plen + nlen
        lora = None if adapter == 0 else adapters[adapter - 1].lora
        readout, temp = heads[adapter]
        empty = model_ref.PrefixState.empty(sum(k == "linear_attention" for k in model.kinds),
                                            sum(k == "full_attention" for k in model.kinds))
        if split:
            prefixes.append((row_ids[:plen], lora, readout, temp))
            rows_out.append(model_ref.RowIn(row_ids[plen:], lora, readout, temp, count, empty))
        else:
            rows_out.append(model_ref.RowIn(row_ids, lora, readout, temp, count, empty))
    return rows_out, prefixes


@pytest.mark.parametrize("exact", [True, False])
def test_oracle_forward_matches_the_transformers_standard_path(golden_model, exact: bool) -> None:
    """Prefix pass then decision pass (the fast path's split) against the whole prompt through transformers'
    Qwen3_5Model + DecisionModel's readout, float32. exact=True (no intermediate rounding): float32 noise only.
    exact=False (the fast path's bfloat16 rounding points) against the float32 standard path: the gap between the
    reference's two paths, about 1% norm-wise per layer (measured 0.96%, 1.7%, 2.4% after layers 1-3), so within 5e-2
    per layer here; probabilities within 1e-2 absolute (measured 6.5e-3). The hot path's own bar (2e-2 per layer) is
    held between the CUDA path and this oracle, which round at the same points (tests/test_forward_gpu.py)."""
    model, adapters, g = golden_model
    rows, prefixes = _rows(model, adapters, g, split=True)
    for row, (pids, lora, readout, temp) in zip(rows, prefixes, strict=True):
        if pids:
            pre = model_ref.run_pass(model, [model_ref.RowIn(pids, lora, readout, temp, 2, row.prefix)], exact=exact,
                                     want_prefix=True)
            assert pre.prefix_out is not None
            row.prefix = pre.prefix_out[0]
    out = model_ref.run_pass(model, rows, exact=exact)
    probs = torch.stack(out.probs)
    want = torch.from_numpy(g["probs"])
    layers = len(model.layers)
    if exact:
        torch.testing.assert_close(probs, want, rtol=1e-4, atol=2e-6)
        for li in range(layers - 1):
            got = torch.stack([out.layer_last[li][i] for i in range(len(rows))])
            torch.testing.assert_close(got, torch.from_numpy(g["hidden_last"][:, li]), rtol=1e-4, atol=1e-4)
        # transformers records the last layer's output after the final norm
        torch.testing.assert_close(torch.stack(out.hidden), torch.from_numpy(g["hidden_last"][:, -1]), rtol=1e-4,
                                   atol=1e-4)
    else:
        assert float((probs - want).abs().max()) < 1e-2
        for li in range(layers - 1):
            got = torch.stack([out.layer_last[li][i] for i in range(len(rows))])
            assert model_ref.rel_error(got, torch.from_numpy(g["hidden_last"][:, li])) < 5e-2
        assert model_ref.rel_error(torch.stack(out.hidden), torch.from_numpy(g["hidden_last"][:, -1])) < 5e-2
