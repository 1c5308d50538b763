"""B200Engine end to end on a B200: prepare, predict_many over groups of two adapters and the base (prefix passes
for new prefixes, cached prefixes on the second call, decision passes), against the CPU oracle of the same rows
(prefix pass, then the decision pass from the prefix's state). A 4-layer synthetic model run as two chained passes
(the prefix pass's states feed the decision pass), so bf16 summation-order drift accumulates over eight layer
applications: probabilities are held to 2e-2 here (the teacher-forced tests of test_forward_gpu.py hold the 1e-2
bar), and decisions and abstentions (threshold 0.8) must agree except at a near-tie."""

from __future__ import annotations

import pytest
import torch

from jeff_b200 import synthetic
from jeff_b200.engine import BASE_ADAPTER, B200Engine, EngineResult, NotInstalled, make_decision
from oracle import model_ref

pytestmark = pytest.mark.gpu

VOCAB = 4096
PROB_TOL = 2e-2


@pytest.fixture(scope="module")
def setup():
    torch.cuda.set_device(0)
    model = synthetic.make_model(synthetic.ModelSpec(layers=4, vocab=VOCAB, fmt="g128z", seed=31, norm_noise=0.1))
    adapters = {f"jeff.test.a{i}": synthetic.make_adapter(model, i, seed=60 + i) for i in (1, 2)}
    g = torch.Generator().manual_seed(32)
    texts = {f"prefix {j}": torch.randint(0, VOCAB, (int(n),), generator=g).tolist()
             for j, n in enumerate((40, 77, 3))}
    engine = B200Engine(model, max_adapters=2, pool_pages_count=2 + 3 * 70, tokenize=lambda t: texts[t],
                        max_batch_rows=16)
    for adapter_id, weights in adapters.items():
        engine.add_adapter(adapter_id, weights)
    return model, adapters, texts, engine, g


def oracle_probs(model, adapter, texts, row) -> torch.Tensor:
    gdn = sum(k == "linear_attention" for k in model.kinds)
    empty = model_ref.PrefixState.empty(gdn, len(model.kinds) - gdn)
    if adapter is None:
        lora, readout, temperature = {}, *synthetic.base_head(model)
    else:
        lora, readout, temperature = adapter.lora, adapter.readout, adapter.temperature
    pre = model_ref.run_pass(model, [model_ref.RowIn(texts[row["prefix_text"]], lora, readout, temperature, 2, empty)],
                             want_prefix=True)
    out = model_ref.run_pass(model, [model_ref.RowIn(row["new_ids"], lora, readout, temperature, row["count"],
                                                     pre.prefix_out[0])])
    return out.probs[0][:row["count"]]


def test_engine_groups_match_the_oracle(setup) -> None:
    model, adapters, texts, engine, g = setup
    groups_rows = {
        "jeff.test.a1": [("prefix 0", 20, 5), ("prefix 1", 33, 2)],
        "jeff.test.a2": [("prefix 0", 7, 9)],
        BASE_ADAPTER: [("prefix 2", 64, 3)],
    }
    groups, spec = [], []
    for adapter_id, rows in groups_rows.items():
        dict_rows = [{"prefix_text": p, "new_ids": torch.randint(0, VOCAB, (n,), generator=g).tolist(), "count": c}
                     for p, n, c in rows]
        groups.append((adapter_id, engine.prepare(adapter_id, dict_rows)))
        spec.append((adapter_id, dict_rows))
    for attempt in range(2):   # the second call finds every prefix cached
        results = engine.predict_many(groups)
        assert all(isinstance(r, EngineResult) for r in results)
        if attempt == 0:
            assert results[0].timing["prefix_misses"] == 4
        else:
            assert results[0].timing["prefix_hits"] == 4 and results[0].timing["prefix_misses"] == 0
        for (adapter_id, rows), result in zip(spec, results, strict=True):
            adapter = None if adapter_id == BASE_ADAPTER else adapters[adapter_id]
            for row, got, tokens in zip(rows, result.probabilities, result.input_tokens, strict=True):
                want = oracle_probs(model, adapter, texts, row)
                diff = float((torch.tensor(got) - want).abs().max())
                assert diff < PROB_TOL, f"{adapter_id}: |p - p_oracle| = {diff}"
                assert tokens == len(texts[row["prefix_text"]]) + len(row["new_ids"])
                mine, theirs = make_decision(got, 0.8), make_decision(want.tolist(), 0.8)
                top2 = sorted(want.tolist())[-2:] if len(want) > 1 else [0.0, 1.0]
                if top2[1] - top2[0] > 2e-2 and abs(theirs.confidence - 0.8) > 2e-2:
                    assert (mine.value, mine.abstained) == (theirs.value, theirs.abstained)


def test_engine_refuses_rows_prepared_before_a_reload(setup) -> None:
    model, adapters, texts, engine, g = setup
    row = {"prefix_text": "prefix 1", "new_ids": [1, 2, 3], "count": 4}
    prepared = engine.prepare("jeff.test.a2", [row])
    engine.remove_adapter("jeff.test.a2")
    engine.add_adapter("jeff.test.a2", adapters["jeff.test.a2"])
    [result] = engine.predict_many([("jeff.test.a2", prepared)])
    assert isinstance(result, NotInstalled)
    [result] = engine.predict_many([("jeff.test.a2", engine.prepare("jeff.test.a2", [row]))])
    assert isinstance(result, EngineResult) and abs(sum(result.probabilities[0]) - 1) < 1e-4
