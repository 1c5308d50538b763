"""B200Engine's host logic on the CPU: the ServingEngine contract of the reference (packages/python/src/jeff/engine.py
and LocalEngine's fast backend, runtime/python/src/jeff_runtime/local_engine.py:295-622), with the GPU passes
replaced by a fake batched path over a real PrefixPool held in host memory. The same behaviours the reference's
engine tests check: adapter add/remove errors and capacity, typed request errors, generations (rows prepared before
a reload are refused), runs of distinct prefixes, pins released, per-group results and timing; and the decision
step's checks (decision.py:68-113)."""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any

import pytest
import torch

from jeff_b200 import constants as C
from jeff_b200.engine import (BASE_ADAPTER, B200Engine, EngineResult, InputTooLong, InvalidRequest, NotInstalled,
                              Prepared, TooManyLabels, checked_probabilities, make_decision)
from jeff_b200.prefix_pool import EngineError, PrefixPool


@dataclass
class FakeAdapter:
    name: str
    max_options: int | None = None


@dataclass
class FakeFast:
    prefixes: PrefixPool
    max_adapters: int
    adapter_index: dict[Any, int] = field(default_factory=lambda: {None: 0})

    def add_adapter(self, adapter: FakeAdapter) -> int:
        if adapter.name.endswith("broken"):
            raise ValueError("bad shapes")
        free = [r for r in range(1, self.max_adapters + 1) if r not in self.adapter_index.values()]
        self.adapter_index[adapter.name] = free[0]
        self.prefixes.forget_adapter(free[0])
        return free[0]

    def remove_adapter(self, name: str) -> None:
        index = self.adapter_index.pop(name)
        self.prefixes.forget_adapter(index)

    def index(self, name: str | None) -> int:
        return self.adapter_index[name]


class FakeBatched:
    """ensure_prefixes on the real pool (reserve + pin, lengths from a fake tokenizer: one token per character);
    decide answers option i of a row with probability proportional to i + 1."""

    def __init__(self, pool: PrefixPool) -> None:
        self.pool = pool
        self.calls: list[list[tuple[int, int, Any]]] = []

    def ensure_prefixes(self, rows, max_tokens):
        slots, misses = [], 0
        for adapter, text in rows:
            slot = self.pool.lookup(adapter, text)
            if slot is None:
                slot = self.pool.reserve(adapter, text, len(text))
                misses += 1
            self.pool.pin([slot])
            slots.append(slot)
        return slots, {"prefix_ms": 1.0, "prefix_misses": misses, "prefix_hits": len(rows) - misses,
                       "prefix_shared": 0, "prefix_passes": 1 if misses else 0}

    def decide(self, rows):
        self.calls.append(list(rows))
        values = []
        for _, _, row in rows:
            w = [i + 1.0 for i in range(row.count)]
            values.append([x / sum(w) for x in w])
        tokens = [self.pool.length(slot) + len(row.new_ids) for _, slot, row in rows]
        return values, tokens, {"passes": 1, "batch_rows": [len(rows)] * len(rows),
                                "bucket": [32] * len(rows), "adapters_in_pass": [1] * len(rows)}


def make_engine(max_adapters: int = 3, pages: int = 2 + 3 * 80, max_tokens: int = 8192) -> B200Engine:
    pool = PrefixPool(pages, "cpu")
    fast = FakeFast(pool, max_adapters)
    return B200Engine(paths=(fast, FakeBatched(pool)), max_adapters=max_adapters, max_tokens=max_tokens)


def row(prefix: str, n: int = 5, count: int = 3) -> dict[str, Any]:
    return {"prefix_text": prefix, "new_ids": list(range(n)), "count": count}


def test_adapters_add_remove_and_their_errors() -> None:
    eng = make_engine(max_adapters=2)
    assert eng.installed() == {BASE_ADAPTER}
    eng.add_adapter("jeff.a.one", FakeAdapter("x"))
    eng.add_adapter("jeff.a.two", FakeAdapter("y", max_options=4))
    assert eng.installed() == {BASE_ADAPTER, "jeff.a.one", "jeff.a.two"}
    with pytest.raises(EngineError, match="already loaded"):
        eng.add_adapter("jeff.a.one", FakeAdapter("x"))
    with pytest.raises(EngineError, match="at most 2 adapters"):
        eng.add_adapter("jeff.a.three", FakeAdapter("z"))
    with pytest.raises(EngineError, match="base model"):
        eng.add_adapter(BASE_ADAPTER, FakeAdapter("b"))
    with pytest.raises(EngineError, match="base model"):
        eng.remove_adapter(BASE_ADAPTER)
    eng.remove_adapter("jeff.a.one")
    with pytest.raises(EngineError, match="not loaded"):
        eng.remove_adapter("jeff.a.one")
    with pytest.raises(EngineError, match="rejected"):
        eng.add_adapter("jeff.a.broken", FakeAdapter("broken"))
    assert eng.installed() == {BASE_ADAPTER, "jeff.a.two"}
    with pytest.raises(EngineError, match="no loader"):
        eng.add_adapter("jeff.a.path", "/nowhere/adapter")


def test_prepare_refuses_with_the_typed_errors() -> None:
    eng = make_engine()
    eng.add_adapter("jeff.a.small", FakeAdapter("s", max_options=4))
    with pytest.raises(NotInstalled, match="jeff.a.other is not installed"):
        eng.prepare("jeff.a.other", [row("p")])
    with pytest.raises(InvalidRequest, match="missing new_ids"):
        eng.prepare("jeff.a.small", [{"prefix_text": "p", "count": 2}])
    with pytest.raises(TooManyLabels, match="at most 4"):
        eng.prepare("jeff.a.small", [row("p", count=5)])
    with pytest.raises(InputTooLong, match="token limit"):
        eng.prepare("jeff.a.small", [row("p", n=max(C.NEW_BUCKETS) + 1)])
    with pytest.raises(InvalidRequest, match="no new tokens"):
        eng.prepare(BASE_ADAPTER, [row("p", n=0)])
    prepared = eng.prepare("jeff.a.small", [row("p"), row("q", count=4)])
    assert prepared.route == "fast" and len(prepared.items) == 2 and prepared.items[1].count == 4
    eng.check(BASE_ADAPTER, [row("p", count=C.READOUT_ROWS)])


def test_predict_many_results_timing_and_generations() -> None:
    eng = make_engine()
    eng.add_adapter("jeff.a.one", FakeAdapter("x"))
    eng.add_adapter("jeff.a.two", FakeAdapter("y"))
    g1 = eng.prepare("jeff.a.one", [row("shared prefix", 3, 2), row("other", 7, 4)])
    g2 = eng.prepare("jeff.a.two", [row("shared prefix", 2, 3)])
    g3 = eng.prepare(BASE_ADAPTER, [row("base prefix", 1, 2)])
    out = eng.predict_many([("jeff.a.one", g1), ("jeff.a.two", g2), (BASE_ADAPTER, g3)])
    assert all(isinstance(r, EngineResult) for r in out)
    assert [len(p) for p in out[0].probabilities] == [2, 4] and len(out[1].probabilities[0]) == 3
    assert out[0].input_tokens == [len("shared prefix") + 3, len("other") + 7]
    assert out[0].row_timing["new_tokens"] == [3, 7] and out[2].row_timing["new_tokens"] == [1]
    assert out[0].timing["path"] == "fast" and out[0].timing["prefix_misses"] == 4
    assert out[0].timing["format"] == "int4-g128z"
    assert not eng.fast.prefixes._pinned, "every pin of the call is released"
    # prepared before a reload: refused, the other groups still run
    eng.remove_adapter("jeff.a.two")
    eng.add_adapter("jeff.a.two", FakeAdapter("y"))
    out = eng.predict_many([("jeff.a.one", g1), ("jeff.a.two", g2)])
    assert isinstance(out[0], EngineResult)
    assert isinstance(out[1], NotInstalled) and "loaded again" in str(out[1])
    with pytest.raises(EngineError, match="did not make"):
        eng.predict_many([("jeff.a.one", Prepared(g1.rows, g1.items, "standard", g1.generation))])
    # predict raises the group's typed error
    assert eng.predict(BASE_ADAPTER, [row("z", 2, 2)]).probabilities[0] == pytest.approx([1 / 3, 2 / 3])


def test_token_limit_is_the_groups_typed_error() -> None:
    eng = make_engine(max_tokens=12)
    prepared = eng.prepare(BASE_ADAPTER, [row("0123456789", 5, 2)])
    [result] = eng.predict_many([(BASE_ADAPTER, prepared)])
    assert isinstance(result, InputTooLong)
    assert not eng.fast.prefixes._pinned


def test_rows_run_in_runs_of_distinct_prefixes_the_pool_holds() -> None:
    eng = make_engine()
    eng._prefixes_at_once = 2
    rows = [row(p) for p in ("a", "b", "a", "c", "d", "c", "e")]
    eng.predict_many([(BASE_ADAPTER, eng.prepare(BASE_ADAPTER, rows))])
    runs = [[r.prefix_text for _, _, r in call] for call in eng.batched.calls]
    assert runs == [["a", "b", "a"], ["c", "d", "c"], ["e"]]


def test_prepared_join_and_part() -> None:
    a = Prepared([{"i": 0}, {"i": 1}], ["x", "y"], "fast", 3)
    b = Prepared([{"i": 2}], ["z"], "fast", 3)
    joined = Prepared.join([a, b])
    assert [r["i"] for r in joined.rows] == [0, 1, 2] and joined.items == ["x", "y", "z"]
    assert joined.part(1, 3).items == ["y", "z"] and joined.part(0, 3) is joined
    with pytest.raises(EngineError, match="several routes"):
        Prepared.join([a, Prepared([{"i": 3}], ["w"], "fast", 4)])
    with pytest.raises(EngineError, match="items for"):
        Prepared([{"i": 0}], ["a", "b"])


def test_decision_step_checks_and_abstains() -> None:
    assert checked_probabilities([0.25, 0.75], 2, "f") == [0.25, 0.75]
    with pytest.raises(EngineError, match="2 probabilities for 3 options"):
        checked_probabilities([0.5, 0.5], 3, "f")
    with pytest.raises(EngineError, match="finite number"):
        checked_probabilities([math.nan, 1.0], 2, "f")
    with pytest.raises(EngineError, match="sum"):
        checked_probabilities([0.5, 0.6], 2, "f")
    d = make_decision([0.1, 0.85, 0.05], 0.8)
    assert (d.value, d.abstained) == (1, False) and d.confidence == pytest.approx(0.85)
    assert make_decision([0.3, 0.7], 0.8).abstained
    assert not make_decision([0.3, 0.7], None).abstained
    assert make_decision([0.5, 0.5], 0.8).value == 0   # a tie takes the first option
    probs = torch.softmax(torch.randn(7, generator=torch.Generator().manual_seed(1)), 0).tolist()
    assert make_decision(probs, 0.8).value == max(range(7), key=probs.__getitem__)


def test_the_fast_path_refuses_more_adapters_than_the_product_gathers() -> None:
    from jeff_b200.fast_path import MAX_ADAPTERS, FastPath

    with pytest.raises(ValueError, match="at most 255 adapters"):
        FastPath(None, max_adapters=MAX_ADAPTERS + 1)   # type: ignore[arg-type]
    with pytest.raises(ValueError, match="at least one adapter"):
        FastPath(None, max_adapters=0)   # type: ignore[arg-type]
