"""The whole batched forward on the GPU (prefix pass into the pool, then the decision pass, CUDA graphs) against
the oracle and the reference's own golden outputs (B200 only; the oracle runs on this GPU as the checker where the
call count makes the CPU too slow).

Acceptance bar (the hot path's), held where it is meaningful:
- per-layer activations within a relative 2e-2 (norm-wise, over each row's tokens) of the oracle, which rounds to bf16
  at the same points, layer by layer on the oracle's inputs and prefix states (teacher-forced);
- label probabilities within 1e-2 absolute of the oracle's, with an identical decision/abstain outcome, on all 1,024
  calls of 16 benchmark passes when the last layer, the final norm and the readout run on the oracle's input to the
  last layer;
- the chained pass (24 layers from the GPU's own prefix passes) over the same 1,024 calls: the decision/abstain
  outcome identical on >= 99.9% of calls; probabilities held against the drift two float32-accumulating bf16
  implementations with identical rounding points show on these calls (measured in the test itself: the oracle
  against itself with float64 product sums), see test_cfg4_1024_chained_calls_match_the_oracle."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from jeff_b200 import synthetic
from jeff_b200.batched_path import BatchedPath, Row
from jeff_b200.fast_path import FastPath
from oracle import model_ref

pytestmark = pytest.mark.gpu

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


@pytest.fixture(scope="module")
def bench_model():
    """The benchmark's own model and inputs (configuration 4 as bench.py builds it: norm weights 0 as transformers
    initialises them), 16 adapters, its batched path, and a device copy of the weights for the oracle."""
    model = synthetic.make_model(synthetic.ModelSpec())
    adapters = [synthetic.make_adapter(model, i, seed=1000 + i) for i in range(1, 17)]
    fast = FastPath(model, max_adapters=16, pool_pages_count=2 + 36 * 66, base_readout=synthetic.base_head(model))
    for a in adapters:
        fast.add_adapter(a)
    texts: dict[str, list[int]] = {}
    path = BatchedPath(fast, tokenize=lambda t: texts[t], max_tokens=64 * 128, max_rows_per_pass=64)
    return model, adapters, fast, path, texts, model_ref.to_device(model, "cuda"), model_ref.to_device(adapters, "cuda")


CALLS_SEEDS = range(4, 20)     # 16 passes of 64 calls: 1,024 calls


def outcome(probs: torch.Tensor, count: int) -> tuple[int, bool]:
    best, _, abstained = model_ref.decision(probs, count, THRESHOLD)
    return (-1, True) if abstained else (best, False)


def test_cfg4_1024_chained_calls_match_the_oracle(bench_model) -> None:
    """1,024 calls of the benchmark configuration (16 passes of 64 calls x 128 tokens, seeds 4..19, each pass on 16
    new 512-token prefixes), chained exactly as served: the GPU's own prefix passes write the pool, its decision
    pass reads it. The checker is the oracle run on this GPU in float32 (its own prefix passes, then the decision
    pass).

    The bar, and why it has two parts:
    - the decision/abstain outcome (decision.py:87-113 at threshold 0.8) is identical on >= 99.9% of the calls;
    - probabilities: two float32-accumulating bf16 implementations with the SAME rounding points already differ by
      more than 1e-2 on a share of these calls, because this random-weight model amplifies one-ulp differences layer
      by layer (the residual stream's relative difference grows ~0.25% per layer). The test measures that floor on
      the same calls: the oracle against itself with float64 product sums (`wide`). Measured at 1,024 calls: oracle
      vs wide oracle max |dp| 0.048, p90 0.013, 167 calls over 1e-2; the GPU's chunked scan adds the bf16 operand
      roundings of a chunked delta rule (as fla's chunk kernel, which the reference's batched path runs), measured
      max 0.086, p90 0.020. So the GPU's |dp| is held to its median <= 1e-2, its p90 within twice the wide oracle's
      p90, its max <= 0.15; and every call within 1e-2 when the last layer runs on the oracle's input (next test).
    """
    model, adapters, fast, path, texts, om, oad = bench_model
    dp_gpu, dp_wide, same, same_wide = [], [], 0, 0
    for seed in CALLS_SEEDS:
        rows = synthetic.make_cfg4_rows(seed=seed)
        for a, p in zip(rows.adapters, rows.prefixes, strict=True):
            texts[f"seed {seed} prefix {a}"] = p
        index = [fast.index(f"adapter-{a}") for a in rows.adapters]
        keys = [(index[i], f"seed {seed} prefix {rows.adapters[i]}") for i in range(64)]
        slots, _ = path.ensure_prefixes(keys, max_tokens=8192)
        try:
            part = [(index[i], slots[i], Row(keys[i][1], rows.new_ids[i], rows.counts[i])) for i in range(64)]
            probs, _ = path.run_pass(64, 128, part, [path.pool.length(s) for s in slots])
            probs = probs.copy()
        finally:
            path.pool.unpin(slots)
        ref = {}
        for wide in (False, True):
            dist = sorted(set(rows.adapters))
            empty = model_ref.PrefixState.empty(18, 6, "cuda")
            pre = model_ref.run_pass(om, [model_ref.RowIn(rows.prefixes[rows.adapters.index(a)], oad[a - 1].lora,
                                                          oad[a - 1].readout, oad[a - 1].temperature, 2, empty)
                                          for a in dist], want_prefix=True, wide=wide)
            assert pre.prefix_out is not None
            state = dict(zip(dist, pre.prefix_out, strict=True))
            ref[wide] = model_ref.run_pass(om, [
                model_ref.RowIn(rows.new_ids[i], oad[rows.adapters[i] - 1].lora, oad[rows.adapters[i] - 1].readout,
                                oad[rows.adapters[i] - 1].temperature, rows.counts[i], state[rows.adapters[i]])
                for i in range(64)], wide=wide).probs
        for i in range(64):
            c = rows.counts[i]
            w, w2, g = ref[False][i][:c].cpu(), ref[True][i][:c].cpu(), torch.tensor(probs[i][:c])
            dp_gpu.append(float((g - w).abs().max()))
            dp_wide.append(float((w2 - w).abs().max()))
            same += int(outcome(g, c) == outcome(w, c))
            same_wide += int(outcome(w2, c) == outcome(w, c))
    calls = len(dp_gpu)
    q = lambda v, f: sorted(v)[min(len(v) - 1, int(f * len(v)))]   # noqa: E731
    print(f"{calls} chained calls: GPU vs oracle |dp| max {max(dp_gpu):.4f} p90 {q(dp_gpu, .9):.4f} median "
          f"{q(dp_gpu, .5):.4f}, {sum(d > 1e-2 for d in dp_gpu)} over 1e-2, outcome identical on {same}; wide oracle "
          f"vs oracle max {max(dp_wide):.4f} p90 {q(dp_wide, .9):.4f} median {q(dp_wide, .5):.4f}, "
          f"{sum(d > 1e-2 for d in dp_wide)} over 1e-2, outcome identical on {same_wide}")
    assert calls >= 1024
    assert same >= math.ceil(0.999 * calls), f"decision/abstain outcome identical on {same} of {calls} calls"
    assert q(dp_gpu, 0.5) <= 1e-2
    assert q(dp_gpu, 0.9) <= 2 * q(dp_wide, 0.9)
    assert max(dp_gpu) <= 0.15


def test_cfg4_1024_calls_last_layer_within_1e2(bench_model) -> None:
    """The same 1,024 calls with the last layer, the final norm and the readout run on the GPU from the oracle's
    input to the last layer (and the oracle's prefix states, written into pool slots): every call's probabilities
    within 1e-2 of the oracle's and its decision/abstain outcome identical. This is the north star's probability
    bar where the model's layer-to-layer amplification of rounding differences is taken out."""
    model, adapters, fast, path, texts, om, oad = bench_model
    worst, same, calls = 0.0, 0, 0
    last = len(model.layers) - 1
    for seed in CALLS_SEEDS:
        rows = synthetic.make_cfg4_rows(seed=seed)
        dist = sorted(set(rows.adapters))
        empty = model_ref.PrefixState.empty(18, 6, "cuda")
        pre = model_ref.run_pass(om, [model_ref.RowIn(rows.prefixes[rows.adapters.index(a)], oad[a - 1].lora,
                                                      oad[a - 1].readout, oad[a - 1].temperature, 2, empty)
                                      for a in dist], want_prefix=True)
        assert pre.prefix_out is not None
        state = dict(zip(dist, pre.prefix_out, strict=True))
        ref = model_ref.run_pass(om, [
            model_ref.RowIn(rows.new_ids[i], oad[rows.adapters[i] - 1].lora, oad[rows.adapters[i] - 1].readout,
                            oad[rows.adapters[i] - 1].temperature, rows.counts[i], state[rows.adapters[i]])
            for i in range(64)], keep_all=True)
        assert ref.layer_all is not None
        slot_of, fresh = {}, []
        try:
            for a in dist:
                st = state[a]
                slot = path.pool.reserve(fast.index(f"adapter-{a}"), f"oracle seed {seed} prefix {a}", st.length)
                path.pool.pin([slot])
                fresh.append(slot)
                kv = torch.stack([torch.stack([k, v]) for k, v in zip(st.keys, st.values, strict=True)])
                path.pool.write(slot, torch.stack(st.conv), torch.stack(st.state), kv)
                slot_of[a] = slot
            part = [(fast.index(f"adapter-{rows.adapters[i]}"), slot_of[rows.adapters[i]],
                     Row("", rows.new_ids[i], rows.counts[i])) for i in range(64)]
            x_in = ref.layer_all[last - 1].to(torch.bfloat16)
            probs = path.last_layer_readout(x_in, 64, 128, part, [512] * 64).cpu()
        finally:
            path.pool.unpin(fresh)
            for slot in fresh:
                path.pool.release(slot)
        for i in range(64):
            c = rows.counts[i]
            w = ref.probs[i][:c].cpu()
            worst = max(worst, float((probs[i, :c] - w).abs().max()))
            same += int(outcome(probs[i, :c], c) == outcome(w, c))
            calls += 1
    print(f"{calls} calls, last layer on the oracle's input: max |dp| {worst:.5f}, outcome identical on {same}")
    assert worst <= 1e-2
    assert same == calls


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
    """Rows of mixed lengths (buckets 32, 64, 128) through decide(): each row keeps its place, and its probabilities
    agree with those of the same row alone in a B = 1 pass of its bucket by the reference's rule for a row in a pass
    against the row alone (runtime/python/tests/test_batched_path_cuda.py:38-47, 222-243): the same top option and no
    probability more than 0.03 apart. The two passes are not bit for bit the same because a small pass takes other
    kernel forms (the products' K split over CTAs, the attention's key walk split), which round differently."""
    model, adapters, fast, path, rows, part, slots = cfg4
    mixed = []
    for j, (adapter, slot, row) in enumerate(part[:6]):
        cut = (20, 50, 128, 33, 64, 1)[j]
        mixed.append((adapter, slot, Row(row.prefix_text, row.new_ids[:cut], row.count)))
    together, tokens, timing = path.decide(mixed)
    assert timing["passes"] == 3 and sorted(set(timing["bucket"])) == [32, 64, 128]
    for j, item in enumerate(mixed):
        alone, _, _ = path.decide([item])
        c = item[2].count
        top2 = np.sort(alone[0][:c])[-2:]
        if top2[1] - top2[0] > 1e-2:   # the reference's rows exclude near ties from the top-option check
            assert int(np.argmax(together[j][:c])) == int(np.argmax(alone[0][:c]))
        np.testing.assert_allclose(together[j], alone[0], rtol=0, atol=3e-2)
        assert tokens[j] == 512 + len(item[2].new_ids)
