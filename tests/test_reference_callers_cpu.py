"""The reference's own callers driving B200Engine (CPU): its Scheduler and its Jeff client, unmodified, imported from
the reference's packages (skipped where no checkout is on the path), over the engine with its GPU passes replaced by
test_engine_cpu's fake batched path on a real PrefixPool.

- Scheduler (runtime/python/src/jeff_runtime/scheduler.py): requests are prepared on submit (typed errors of
  prepare() are delivered as they are, :148-152), gathered into one predict_many call (:309-320), and each group's
  result is sorted into probabilities or a typed failure by `isinstance(result, JeffError)` (:340). A group whose
  adapter was reloaded after it was prepared gets NotInstalled from predict_many; the scheduler must hand that error,
  the reference's own class, to the request's callback.
- Jeff client (packages/python/src/jeff/client.py:151-169): binds a function from a manifest catalogue (the
  reference's test fixture), builds rows, calls predict, and makes Decisions; a typed error predict raises reaches
  the caller as the reference's class.

The tail test runs test_engine_cpu.py again in a child process with JEFF_B200_LOCAL_TYPES=1, where the reference's
packages stay off the path: the engine's stand-in types must pass the same tests."""

from __future__ import annotations

import json
import os
import subprocess
import sys
import threading
from pathlib import Path
from typing import Any

import pytest

from conftest import REFERENCE, ROOT
from jeff_b200 import errors
from jeff_b200.batched_path import Row
from test_engine_cpu import FakeAdapter, FakeBatched, FakeFast

pytestmark = pytest.mark.skipif(not errors.REFERENCE_TYPES, reason="the reference's jeff package is not importable")

CATALOGUE = REFERENCE / "packages" / "python" / "tests" / "fixtures" / "catalogue"


def make_engine(max_tokens: int = 8192, **options: Any):
    from jeff_b200.engine import B200Engine
    from jeff_b200.prefix_pool import PrefixPool

    pool = PrefixPool(2 + 3 * 80, "cpu")
    return B200Engine(paths=(FakeFast(pool, 3), FakeBatched(pool)), max_adapters=3, max_tokens=max_tokens, **options)


def row(prefix: str, n: int = 5, count: int = 3) -> dict[str, Any]:
    return {"prefix_text": prefix, "new_ids": list(range(n)), "count": count}


class Outcomes:
    """on_done callbacks that record what each request got, and wait for all of them."""

    def __init__(self, count: int) -> None:
        self.got: dict[str, Any] = {}
        self.count = count
        self.all_in = threading.Event()

    def callback(self, name: str):
        def done(value: Any) -> None:
            self.got[name] = value
            if len(self.got) == self.count:
                self.all_in.set()
        return done


def test_the_reference_scheduler_sorts_results_and_typed_errors() -> None:
    from jeff.engine import EngineResult
    from jeff.errors import JeffError, NotInstalled, TooManyLabels
    from jeff_runtime.scheduler import Scheduler, Settings

    eng = make_engine()
    eng.add_adapter("jeff.a.one", FakeAdapter("x", max_options=4))
    eng.add_adapter("jeff.a.two", FakeAdapter("y"))
    scheduler = Scheduler(eng, Settings(window_ms=5.0, max_batch_rows=64, queue_limit_rows=256))
    out = Outcomes(4)
    scheduler.submit("jeff.a.one", [row("shared", 3, 2), row("other", 7, 4)], None, out.callback("ok"))
    scheduler.submit("jeff.a.two", [row("stale", 2, 3)], None, out.callback("stale"))
    scheduler.submit("jeff.a.one", [row("big", 2, 5)], None, out.callback("labels"))          # prepare refuses
    scheduler.submit("jeff.a.none", [row("p")], None, out.callback("missing"))               # prepare refuses
    # reloaded after "stale" was prepared: predict_many answers that group with NotInstalled
    reloaded = threading.Event()
    scheduler.change(lambda: (eng.remove_adapter("jeff.a.two"), eng.add_adapter("jeff.a.two", FakeAdapter("y"))),
                     lambda error: reloaded.set())
    scheduler.start()
    try:
        assert out.all_in.wait(30), f"only {sorted(out.got)} answered"
    finally:
        scheduler.stop()
    assert reloaded.is_set()
    ok = out.got["ok"]
    assert isinstance(ok, EngineResult) and [len(p) for p in ok.probabilities] == [2, 4]
    assert ok.input_tokens == [len("shared") + 3, len("other") + 7] and ok.timing["path"] == "fast"
    assert isinstance(out.got["stale"], NotInstalled) and "loaded again" in str(out.got["stale"])
    assert isinstance(out.got["labels"], TooManyLabels)
    assert isinstance(out.got["missing"], NotInstalled)
    assert all(isinstance(v, JeffError) for k, v in out.got.items() if k != "ok")
    assert not eng.fast.prefixes._pinned


def prepare_binding_row(adapter_id: str, item: dict[str, Any]) -> Row:
    """A stand-in for the reference's tokenizer-based preparer (prepare.prepare_rows): the question's instructions
    and option keys as the prefix text, the request state's characters as the new token ids."""
    question = item["question"]
    criteria = list(question.get("criteria") or {})
    state = json.dumps(item["state"], sort_keys=True)
    return Row(f"{question['instructions']} | {' '.join(criteria)}", [ord(c) % 251 for c in state][:128],
               max(len(criteria), 1))


def test_the_reference_jeff_client_decides_and_raises_typed_errors() -> None:
    from jeff.catalogue import Catalogue
    from jeff.client import Call, Jeff
    from jeff.decision import Decision
    from jeff.errors import TooManyLabels

    if not CATALOGUE.is_dir():
        pytest.skip("the reference's test catalogue is not in this checkout")
    eng = make_engine(preparer=prepare_binding_row, base_format={"format": "bf16"})
    eng.add_adapter("jeff.safety.spam", FakeAdapter("s"))
    jeff = Jeff(eng, Catalogue.from_dir(CATALOGUE))
    [decision] = jeff.decide([Call("spam.message_type", "Win a prize now", {"channel": "email"})])
    assert isinstance(decision, Decision)
    # the fake answers option i with weight i + 1: 3 options -> 1/6, 2/6, 3/6; below the 0.7 calibration threshold
    assert decision.probabilities == pytest.approx({"legitimate": 1 / 6, "spam": 2 / 6, "phishing": 3 / 6})
    assert decision.confidence == pytest.approx(0.5) and decision.value == "phishing"
    bound = jeff.function("spam.message_type", context={"channel": "sms"})
    assert len(bound.many(["a", "b", "c"])) == 3
    eng.remove_adapter("jeff.safety.spam")
    eng.add_adapter("jeff.safety.spam", FakeAdapter("s", max_options=2))
    with pytest.raises(TooManyLabels, match="at most 2"):
        jeff.decide([Call("spam.message_type", "hello", {"channel": "email"})])
    assert not eng.fast.prefixes._pinned


def test_the_engine_tests_pass_with_the_stand_in_types() -> None:
    env = dict(os.environ, JEFF_B200_LOCAL_TYPES="1")
    probe = subprocess.run([sys.executable, "-c", "import jeff_b200.errors as e; print(e.REFERENCE_TYPES)"],
                           cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert probe.stdout.strip() == "False", probe.stderr
    res = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider",
                          str(Path(__file__).with_name("test_engine_cpu.py"))],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
