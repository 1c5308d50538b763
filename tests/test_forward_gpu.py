"""The whole batched forward on the GPU (prefix pass into the pool, then the decision pass, CUDA graphs) against
the CPU oracle and the reference's own golden outputs (B200 only).

Acceptance bar (the hot path's), held where it is meaningful:
- per-layer activations within a relative 2e-2 (norm-wise, over each row's tokens) of the oracle, which rounds to bf16
  at the same points, layer by layer on the oracle's inputs and prefix states (teacher-forced);
- label probabilities within 1e-2 absolute of the oracle's when the last layer, the final norm and the readout run on
  the oracle's input to the last layer;
- the chained pass (24 layers from the GPU's own prefix pass): bf16 arithmetic of two implementations with the same
  rounding points drifts apart from summation order alone (measured on the CPU: the oracle against itself with
  exact instead of float32 product sums moves probabilities by up to 9.4e-3 on this model; the GPU's chunked scan
  also rounds its state operands to bf16, as fla's chunk kernel that the reference runs does), so the chained pass is
  checked on its outputs over all 64 calls: probabilities within 5e-2 and the chosen option identical on at least 56
  (these random-weight models give flat option distributions, where near-ties are common; the test prints the
  spread and the agreement)."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from jeff_b200 import synthetic
from jeff_b200.batched_path import BatchedPath, Row
from jeff_b200.fast_path import FastPath
from oracle import model_ref

pytestmark = pytest.mark.gpu

CHAIN_TOL = 2.5e-2   # twice the largest summation-order drift measured between two float32 oracles
THRESHOLD = 0.8


def check_decisions(got: list[float], want: torch.Tensor, count: int, tol: float, bound: float | None = None) -> bool:
    """Probabilities within `bound` (default tol); the decision and the abstention identical unless within 2 tol of
    a tie (returns whether the call counted as decided, i.e. was not such a near-tie)."""
    g = torch.tensor(got[:count])
    w = want[:count]
    assert float((g - w).abs().max()) < (tol if bound is None else bound)
    top = torch.topk(w, min(2, count)).values
    if count > 1 and float(top[0] - top[1]) < 2 * tol:
        return False
    gd = model_ref.decision(g, count, THRESHOLD)
    wd = model_ref.decision(w, count, THRESHOLD)
    assert gd[0] == wd[0]
    if abs(wd[1] - THRESHOLD) > 2 * tol:
        assert gd[2] == wd[2]
    return True


@pytest.fixture(scope="module")
def golden():
    meta = json.loads((GOLDEN / "model_golden.json").read_text())
    spec = synthetic.ModelSpec(layers=meta["layers"], vocab=meta["vocab"], fmt=meta["fmt"], seed=meta["seed"],
                               norm_noise=meta["norm_noise"])
    model = synthetic.make_model(spec)
    adapters = [synthetic.make_adapter(model, i, seed=meta["seed"] + i) for i in meta["adapters"]]
    return model, adapters, dict(np.load(GOLDEN / "model_golden.npz"))


def test_forward_matches_the_reference_golden_outputs(golden) -> None:
    """The 4-layer model at the real layer dimensions, whose probabilities the reference's transformers path
    computed (float32) from the whole prompt: the GPU's prefix pass + decision pass within 1e-2 of them, and within
    1e-2 of the bf16 oracle with the same split."""
    model, adapters, g = golden
    fast = FastPath(model, max_adapters=2, pool_pages_count=400, base_readout=synthetic.base_head(model))
    index = [0] + [fast.add_adapter(a) for a in adapters]
    ids = g["ids"].tolist()
    texts, keys, rows, off = {}, [], [], 0
    for i, (adapter, plen, nlen, count) in enumerate(g["rows"].tolist()):
        row_ids = ids[off:off + plen + nlen]
        off += plen + nlen
        text = f"golden prefix {i}"
        texts[text] = row_ids[:plen]
        keys.append((index[adapter], text))
        rows.append((row_ids[plen:], count))
    path = BatchedPath(fast, tokenize=lambda t: texts[t], max_tokens=1024, max_rows_per_pass=8)
    slots, _ = path.ensure_prefixes(keys, max_tokens=8192)
    try:
        probs, tokens, _ = path.decide([(keys[i][0], slots[i], Row(keys[i][1], rows[i][0], rows[i][1]))
                                        for i in range(len(rows))])
    finally:
        path.pool.unpin(slots)
    for i, (adapter, plen, nlen, count) in enumerate(g["rows"].tolist()):
        assert tokens[i] == plen + nlen
        want = torch.from_numpy(g["probs"][i])
        assert float((torch.tensor(probs[i]) - want[:count]).abs().max()) < 1e-2, f"row {i} vs the reference"


@pytest.fixture(scope="module")
def cfg4():
    """The benchmark model (24 layers, int4 group 128 with zeros, norm weights perturbed so every norm weight
    matters), 16 adapters, and its batched path with the 64 x 128 pass run once."""
    model = synthetic.make_model(synthetic.ModelSpec(norm_noise=0.1))
    adapters = [synthetic.make_adapter(model, i, seed=1000 + i) for i in range(1, 17)]
    fast = FastPath(model, max_adapters=16, pool_pages_count=2 + 24 * 70,
                    base_readout=synthetic.base_head(model))
    for a in adapters:
        fast.add_adapter(a)
    rows = synthetic.make_cfg4_rows(seed=4)
    texts = {f"prefix {a}": p for a, p in zip(rows.adapters, rows.prefixes)}
    path = BatchedPath(fast, tokenize=lambda t: texts[t], max_tokens=64 * 128, max_rows_per_pass=64)
    index = [fast.index(f"adapter-{a}") for a in rows.adapters]
    keys = [(index[i], f"prefix {rows.adapters[i]}") for i in range(64)]
    slots, _ = path.ensure_prefixes(keys, max_tokens=8192)
    part = [(index[i], slots[i], Row(keys[i][1], rows.new_ids[i], rows.counts[i])) for i in range(64)]
    return model, adapters, fast, path, rows, part, slots


def oracle_rows(model, adapters, rows, picks: list[int]) -> list:
    empty = model_ref.PrefixState.empty(18, 6)
    out = []
    for i in picks:
        ad = adapters[rows.adapters[i] - 1]
        pre = model_ref.run_pass(model, [model_ref.RowIn(rows.prefixes[i], ad.lora, ad.readout, ad.temperature, 2,
                                                         empty)], want_prefix=True)
        assert pre.prefix_out is not None
        out.append(model_ref.RowIn(rows.new_ids[i], ad.lora, ad.readout, ad.temperature, rows.counts[i],
                                   pre.prefix_out[0]))
    return out


def test_cfg4_layers_match_the_oracle_layer_by_layer(cfg4) -> None:
    """Layer-local parity on the benchmark model: four rows' oracle prefix states are written into pool slots, and
    every GPU layer runs on the oracle's input to that layer; its output residual stream (each row's 128 tokens x
    1024) is within 2e-2 of the oracle's (norm-wise). Chained through 24 layers, two bf16 implementations drift
    apart by more than that from summation order alone (the oracle against itself with exact instead of float32
    product sums: 1.8% after 6 layers), so the chain is checked on its outputs (the next test)."""
    model, adapters, fast, path, rows, part, slots = cfg4
    picks = [0, 21, 42, 63]
    refs = oracle_rows(model, adapters, rows, picks)
    ref = model_ref.run_pass(model, refs, keep_all=True)
    assert ref.layer_all is not None
    fresh, staged = [], []
    try:
        for j, i in enumerate(picks):
            st = refs[j].prefix
            slot = path.pool.reserve(part[i][0], f"oracle prefix {i}", st.length)
            path.pool.pin([slot])      # so that the next reservation cannot evict it
            fresh.append(slot)
            kv = torch.stack([torch.stack([k, v]) for k, v in zip(st.keys, st.values)])
            path.pool.write(slot, torch.stack(st.conv).cuda(), torch.stack(st.state).cuda(), kv.cuda())
            staged.append((part[i][0], slot, part[i][2]))
        lengths = [512] * len(picks)
        ids = torch.tensor([t for i in picks for t in rows.new_ids[i]])
        x_in = model.embed[ids].cuda()
        worst = []
        for li in range(len(model.layers)):
            got = path.layer_pass(li, x_in, len(picks), 128, staged, lengths).float().cpu()
            want = ref.layer_all[li]
            errs = [model_ref.rel_error(got[j * 128:(j + 1) * 128], want[j * 128:(j + 1) * 128])
                    for j in range(len(picks))]
            worst.append(max(errs))
            x_in = want.to(torch.bfloat16).cuda()
        assert max(worst) < 2e-2, f"per-layer worst relative errors {[round(w, 4) for w in worst]}"
    finally:
        path.pool.unpin(fresh)
        for slot in fresh:
            path.pool.release(slot)


def test_cfg4_last_layer_and_readout_match_the_oracle(cfg4) -> None:
    """The last layer, the final norm and the readout on the oracle's input to the last layer (and its prefix
    state): probabilities within 1e-2 of the oracle's, the same decision and abstention."""
    model, adapters, fast, path, rows, part, slots = cfg4
    picks = [0, 21, 42, 63]
    refs = oracle_rows(model, adapters, rows, picks)
    ref = model_ref.run_pass(model, refs, keep_all=True)
    assert ref.layer_all is not None
    fresh, staged = [], []
    try:
        for j, i in enumerate(picks):
            st = refs[j].prefix
            slot = path.pool.reserve(part[i][0], f"oracle prefix {i}", st.length)
            path.pool.pin([slot])
            fresh.append(slot)
            kv = torch.stack([torch.stack([k, v]) for k, v in zip(st.keys, st.values)])
            path.pool.write(slot, torch.stack(st.conv).cuda(), torch.stack(st.state).cuda(), kv.cuda())
            staged.append((part[i][0], slot, part[i][2]))
        last_layer = len(model.layers) - 1
        x_in = ref.layer_all[last_layer - 1].to(torch.bfloat16).cuda()
        probs = path.last_layer_readout(x_in, len(picks), 128, staged, [512] * len(picks)).cpu()
        for j, i in enumerate(picks):
            check_decisions(probs[j].tolist(), ref.probs[j], rows.counts[i], 1e-2)
    finally:
        path.pool.unpin(fresh)
        for slot in fresh:
            path.pool.release(slot)


def test_cfg4_chained_pass_matches_the_oracle_on_every_call(cfg4) -> None:
    """All 64 calls of the benchmark pass, chained (GPU prefix passes, GPU decision pass) against the chained oracle
    (its own prefix passes, once per distinct prefix): probabilities within CHAIN_TOL, decisions identical except
    near-ties (module docstring)."""
    model, adapters, fast, path, rows, part, slots = cfg4
    lengths = [path.pool.length(s) for s in slots]
    probs, _ = path.run_pass(64, 128, part, lengths)
    empty = model_ref.PrefixState.empty(18, 6)
    prefix_of: dict[int, model_ref.PrefixState] = {}
    for a in sorted(set(rows.adapters)):
        i = rows.adapters.index(a)
        ad = adapters[a - 1]
        pre = model_ref.run_pass(model, [model_ref.RowIn(rows.prefixes[i], ad.lora, ad.readout, ad.temperature, 2,
                                                         empty)], want_prefix=True)
        assert pre.prefix_out is not None
        prefix_of[a] = pre.prefix_out[0]
    ref_rows = [model_ref.RowIn(rows.new_ids[i], adapters[rows.adapters[i] - 1].lora,
                                adapters[rows.adapters[i] - 1].readout, adapters[rows.adapters[i] - 1].temperature,
                                rows.counts[i], prefix_of[rows.adapters[i]]) for i in range(64)]
    ref = model_ref.run_pass(model, ref_rows)
    diffs, agree, outcome_same, clear, clear_same, abstained, gaps = [], 0, 0, 0, 0, 0, []
    for i in range(64):
        c = rows.counts[i]
        g, w = torch.tensor(probs[i][:c].tolist()), ref.probs[i][:c]
        diffs.append(float((g - w).abs().max()))
        agree += int(torch.argmax(g) == torch.argmax(w))
        # the Decision outcome (decision.py:87-113): the chosen option, or an abstention below the threshold
        gd, wd = model_ref.decision(g, c, THRESHOLD), model_ref.decision(w, c, THRESHOLD)
        same = (gd[2] and wd[2]) or (not gd[2] and not wd[2] and gd[0] == wd[0])
        outcome_same += int(same)
        abstained += int(wd[2])
        if torch.argmax(g) != torch.argmax(w):
            srt = torch.sort(w.double() / w.double().sum(), descending=True).values
            gaps.append(round(float(srt[0] - srt[1]), 4))
        top = torch.topk(w.double() / w.double().sum(), min(2, c)).values
        near = abs(wd[1] - THRESHOLD) < CHAIN_TOL or (not wd[2] and c > 1 and float(top[0] - top[1]) < CHAIN_TOL)
        if not near:
            clear += 1
            clear_same += int(same)
    print(f"chained pass: max |dp| {max(diffs):.4f}, mean {sum(diffs) / 64:.4f}, argmax agreement {agree}/64, "
          f"decision/abstain outcome identical on {outcome_same}/64 ({clear_same}/{clear} away from the threshold "
          f"and from ties; the oracle abstains on {abstained}); top-2 gaps where the argmax differs: {gaps}")
    assert max(diffs) < 5e-2
    assert agree >= 56, f"argmax agrees on {agree} of 64 calls"
    assert clear_same == clear, f"decision outcome differs on {clear - clear_same} calls away from threshold and ties"


def test_cfg4_graph_replays_are_deterministic_and_well_formed(cfg4) -> None:
    """Two replays of the recorded graph give the same bits, the eager pass the same bits as the graph, every row's
    probabilities sum to 1 over its options (within 1e-4, the reference's SUM_TOLERANCE) and are zero past them."""
    model, adapters, fast, path, rows, part, slots = cfg4
    lengths = [path.pool.length(s) for s in slots]
    first, _ = path.run_pass(64, 128, part, lengths)
    first = first.copy()
    second, _ = path.run_pass(64, 128, part, lengths)
    assert np.array_equal(first, second)
    eager, _ = path.trace_pass(64, 128, part, lengths)
    assert np.array_equal(eager.cpu().numpy(), first)
    for i in range(64):
        c = rows.counts[i]
        assert abs(float(first[i, :c].sum()) - 1.0) < 1e-4
        assert not first[i, c:].any()


def test_decide_groups_rows_by_bucket_and_keeps_order(cfg4) -> None:
    """Rows of mixed lengths (buckets 32, 64, 128) through decide(): each row's probabilities equal those of the same
    row alone in a B = 1 pass of its bucket."""
    model, adapters, fast, path, rows, part, slots = cfg4
    mixed = []
    for j, (adapter, slot, row) in enumerate(part[:6]):
        cut = (20, 50, 128, 33, 64, 1)[j]
        mixed.append((adapter, slot, Row(row.prefix_text, row.new_ids[:cut], row.count)))
    together, tokens, timing = path.decide(mixed)
    assert timing["passes"] == 3 and sorted(set(timing["bucket"])) == [32, 64, 128]
    for j, item in enumerate(mixed):
        alone, _, _ = path.decide([item])
        np.testing.assert_allclose(together[j], alone[0], rtol=0, atol=2e-3)
        assert tokens[j] == 512 + len(item[2].new_ids)
