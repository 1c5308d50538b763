"""The engine the reference's callers talk to, on the B200 path.

B200Engine implements the reference's ServingEngine protocol (packages/python/src/jeff/engine.py:158-208): the same
attributes (backend, base_checkpoint, max_adapters, base_format, base_max_options) and methods (installed, check,
prepare, predict_many, predict, add_adapter, remove_adapter), with the behaviour of LocalEngine's fast backend
(runtime/python/src/jeff_runtime/local_engine.py:295-622): adapter generations so rows prepared before a reload are
refused, runs of at most as many distinct prefixes as the pool surely holds, each run's prefixes made sure of and
pinned, the token limit checked, the batched passes, and per-group results with the call's timing and per-row
timing. The result and request types (EngineResult, Prepared) and the typed errors come from jeff_b200.errors: the
reference's own jeff.engine and jeff.errors classes whenever its client package is importable, so the reference's
Scheduler and Jeff client dispatch on this engine's results and errors unchanged (tests/test_reference_callers_cpu.py
drives both over this engine), else stand-ins with the same names, fields and messages.

What differs, and why: the reference's prepare() renders each row through the adapter's chat template and splits it
with its tokenizer (prepare.prepare_rows, prepare.py:366-392). No tokenizer or prompt layout exists offline, so this
engine takes rows that are already split: {"prefix_text": str, "new_ids": [int, ...], "count": int} (the fields of
the reference's prepare.Row), or any row through a `preparer` callable given at construction that returns a Row.
New prefixes are tokenised by the `tokenize` callable (prefix text -> token ids), as BatchedPath.ensure_prefixes
does. Adapters are added as AdapterWeights (or a path handed to a `loader` callable).

checked_probabilities and make_decision restate the decision step of the reference's client
(packages/python/src/jeff/decision.py:68-113) for choice questions: the argmax option, its probability as the
confidence, abstention below the calibration threshold."""

from __future__ import annotations

import dataclasses
import itertools
import math
import threading
import time
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from jeff_b200 import constants as C
from jeff_b200.errors import (BASE_ADAPTER, REFERENCE_TYPES, EngineError, EngineResult, InputTooLong, InvalidRequest,
                              JeffError, NotInstalled, Prepared, TooManyLabels)
from jeff_b200.prefix_pool import RESERVED_PAGES

SUM_TOLERANCE = 1e-4
TOO_LONG_MESSAGE = "no input was truncated"
ROW_TIMING = ("pass_rows", "bucket", "adapters_in_pass")
CALL_COUNTERS = ("passes", "prefix_ms", "prefix_misses", "prefix_hits", "prefix_shared", "prefix_passes")


# ---------------------------------------------------------------- the decision step (jeff/decision.py)


@dataclass(frozen=True)
class Decision:
    value: int
    confidence: float
    abstained: bool
    probabilities: list[float]


def checked_probabilities(probabilities: Sequence[float], option_count: int, name: str) -> list[float]:
    """The engine reply check of decision.py:68-84: refused (EngineError) for the wrong count, a value that is not a
    finite number in [0, 1], or a sum more than SUM_TOLERANCE from 1; a valid reply divided by its sum."""
    if len(probabilities) != option_count:
        raise EngineError(f"{name}: the engine returned {len(probabilities)} probabilities for {option_count} options")
    offending = [p for p in probabilities if not (math.isfinite(p) and 0 <= p <= 1)]
    if offending:
        raise EngineError(f"{name}: the engine returned invalid probabilities {list(probabilities)}; expected each to "
                          f"be a finite number from 0 to 1, which {offending} are not")
    total = sum(probabilities)
    if abs(total - 1) > SUM_TOLERANCE:
        raise EngineError(f"{name}: the engine returned invalid probabilities {list(probabilities)}; expected their "
                          f"sum to be within {SUM_TOLERANCE} of 1, got {total}")
    return [p / total for p in probabilities]


def make_decision(probabilities: Sequence[float], threshold: float | None, name: str = "decision") -> Decision:
    """A choice question's Decision (decision.py:87-113): the most probable option (the first on a tie), its
    probability as the confidence, abstained when calibrated (threshold not None) and the confidence is below it."""
    normalised = checked_probabilities(probabilities, len(probabilities), name)
    best = max(range(len(normalised)), key=normalised.__getitem__)
    confidence = normalised[best]
    return Decision(best, confidence, threshold is not None and confidence < threshold, normalised)


# ---------------------------------------------------------------- the engine


def _row_of(row: dict[str, Any], number: int) -> Any:
    from jeff_b200.batched_path import Row

    missing = [name for name in ("prefix_text", "new_ids", "count") if name not in row]
    if missing:
        raise InvalidRequest(f"Row {number}: missing {', '.join(missing)} (this engine takes rows split into "
                             "prefix_text, new_ids and count, or a preparer)")
    new_ids = [int(t) for t in row["new_ids"]]
    count = int(row["count"])
    if not isinstance(row["prefix_text"], str):
        raise InvalidRequest(f"Row {number}: prefix_text must be a string")
    if not 1 <= count <= C.READOUT_ROWS:
        raise InvalidRequest(f"Row {number}: {count} options; a question has 1 to {C.READOUT_ROWS}")
    return Row(row["prefix_text"], new_ids, count)


class B200Engine:
    """ServingEngine on the B200 batched path. Build it with the base's weights (or hand it a prebuilt
    (FastPath, BatchedPath) pair as `paths`), then add adapters. predict_many is called from one thread (the GPU
    thread); prepare and check from any."""

    backend = "fast"

    def __init__(self, model: Any = None, *, max_adapters: int = 8, prefix_pool_mb: int | None = None,
                 pool_pages_count: int | None = None, max_tokens: int = 8192, max_batch_rows: int = 64,
                 tokenize: Callable[[str], list[int]] | None = None,
                 preparer: Callable[[str, dict[str, Any]], Any] | None = None,
                 loader: Callable[[Path], Any] | None = None, base_checkpoint: str = "synthetic",
                 base_format: dict[str, str] | None = None, base_max_options: int = C.READOUT_ROWS,
                 paths: tuple[Any, Any] | None = None, device: Any = None) -> None:
        if paths is None:
            from jeff_b200 import synthetic
            from jeff_b200.batched_path import BatchedPath
            from jeff_b200.fast_path import FastPath

            if model is None:
                raise EngineError("B200Engine needs the base's weights (model) or prebuilt paths")
            fast = FastPath(model, max_adapters=max_adapters, prefix_pool_mb=prefix_pool_mb,
                            pool_pages_count=pool_pages_count, device=device if device is not None else "cuda",
                            base_readout=synthetic.base_head(model))
            batched = BatchedPath(fast, tokenize=tokenize, max_rows_per_pass=max_batch_rows)
        else:
            fast, batched = paths
        self.fast, self.batched = fast, batched
        self.max_adapters = max_adapters
        self.max_tokens = max_tokens
        self.base_checkpoint = base_checkpoint
        self.base_format = dict(base_format or {"format": "int4-g128z", "format_id": base_checkpoint})
        self._base_max_options = base_max_options
        self.preparer, self.loader = preparer, loader
        pool = fast.prefixes
        per_prefix = pool.shapes.pages_per_prefix(C.LONGEST_PREFIX_TOKENS)
        self._prefixes_at_once = max(1, (pool.pages - RESERVED_PAGES) // per_prefix)
        self._adapters_lock = threading.Lock()
        self._adapters: dict[str, Any] = {}
        self._max_options: dict[str, int] = {}
        self._generations: dict[str, int] = {BASE_ADAPTER: 0}
        self._loads = itertools.count(1)

    # ------------------------------------------------------------ adapters

    def installed(self, refresh: bool = False) -> set[str]:
        with self._adapters_lock:
            return {BASE_ADAPTER, *self._adapters}

    @property
    def base_max_options(self) -> int:
        return self._base_max_options

    def add_adapter(self, adapter_id: str, path: Any) -> None:
        """Load an adapter beside the others (local_engine.py:414-441): refused for the base's id, an id already
        loaded, or past max_adapters; `path` is AdapterWeights, or a path given to the loader."""
        if adapter_id == BASE_ADAPTER:
            raise EngineError(f"{BASE_ADAPTER!r} is the base model, always served; it cannot be added as an adapter")
        with self._adapters_lock:
            if adapter_id in self._adapters:
                raise EngineError(f"{adapter_id} is already loaded in this engine")
            if self.max_adapters is not None and len(self._adapters) >= self.max_adapters:
                raise EngineError(f"This engine holds at most {self.max_adapters} adapters (--max-adapters "
                                  f"{self.max_adapters}) and {len(self._adapters)} are loaded; remove one first, or "
                                  "restart the engine with a larger --max-adapters")
        weights = path
        if isinstance(path, (str, Path)):
            if self.loader is None:
                raise EngineError(f"{adapter_id}: this engine has no loader for adapter folders ({path})")
            weights = self.loader(Path(path))
        weights = dataclasses.replace(weights, name=adapter_id)
        limit = int(getattr(weights, "max_options", None) or self._base_max_options)
        try:
            self.fast.add_adapter(weights)
        except Exception as error:
            raise EngineError(f"{adapter_id}: the fast path rejected this adapter: {error}") from error
        with self._adapters_lock:
            self._max_options[adapter_id] = limit
            self._generations[adapter_id] = next(self._loads)
            self._adapters[adapter_id] = path

    def remove_adapter(self, adapter_id: str) -> None:
        if adapter_id == BASE_ADAPTER:
            raise EngineError(f"{BASE_ADAPTER!r} is the base model, always served; it cannot be removed")
        with self._adapters_lock:
            if adapter_id not in self._adapters:
                raise EngineError(f"{adapter_id} is not loaded in this engine (loaded: {sorted(self._adapters)})")
        self.fast.remove_adapter(adapter_id)
        with self._adapters_lock:
            del self._adapters[adapter_id]
            del self._max_options[adapter_id]
            del self._generations[adapter_id]

    # ------------------------------------------------------------ requests

    def _limit(self, adapter_id: str) -> int:
        if adapter_id == BASE_ADAPTER:
            return self._base_max_options
        if adapter_id not in self._adapters:
            raise NotInstalled(adapter_id, f"this engine serves {sorted(self._adapters) or 'no adapters'}")
        return self._max_options[adapter_id]

    def check(self, adapter_id: str, rows: list[dict[str, Any]]) -> None:
        self.prepare(adapter_id, rows)

    def prepare(self, adapter_id: str, rows: list[dict[str, Any]]) -> Prepared:
        """Validate and split a request without touching the GPU (local_engine.py:327-396): NotInstalled for an
        adapter not loaded, InvalidRequest for a row that cannot be read, TooManyLabels past the adapter's option
        limit, InputTooLong for more new tokens than the largest bucket or the token limit."""
        with self._adapters_lock:
            limit = self._limit(adapter_id)
            generation = self._generations[adapter_id]
        items = []
        for number, row in enumerate(rows):
            item = self.preparer(adapter_id, row) if self.preparer is not None else _row_of(row, number)
            if item.count > limit:
                raise TooManyLabels(f"A choice question has {item.count} options, but this model handles at most "
                                    f"{limit} ({adapter_id} was trained on questions of up to {limit} options). "
                                    "Shortlist the options first, or split the question.")
            if len(item.new_ids) > max(C.NEW_BUCKETS) or len(item.new_ids) > self.max_tokens:
                raise InputTooLong(f"Question branch exceeds the {self.max_tokens}-token limit; {TOO_LONG_MESSAGE}.")
            if not item.new_ids:
                raise InvalidRequest(f"Row {number}: no new tokens")
            items.append(item)
        return Prepared(list(rows), items, "fast", generation)

    def predict(self, adapter_id: str, rows: list[dict[str, Any]]) -> EngineResult:
        [result] = self.predict_many([(adapter_id, self.prepare(adapter_id, rows))])
        if isinstance(result, JeffError):
            raise result
        return result

    def predict_many(self, groups: list[tuple[str, Prepared]]) -> list[EngineResult | JeffError]:
        """One result per (adapter id, prepared rows) group, in order (local_engine.py:469-516): a group whose
        adapter was removed or loaded again since it was prepared gets NotInstalled; the other groups run together
        on the batched path, sharing one outcome (a typed failure is every group's)."""
        results: list[EngineResult | JeffError | None] = [None] * len(groups)
        with self._adapters_lock:
            generations = dict(self._generations)
        for i, (adapter_id, prepared) in enumerate(groups):
            if prepared.generation is None or prepared.route != "fast":
                raise EngineError(f"{adapter_id}: predict_many was given rows this engine's prepare() did not make")
            if generations.get(adapter_id) != prepared.generation:
                results[i] = NotInstalled(adapter_id, "was unloaded or loaded again after this request arrived, so it "
                                                      "was prepared for the adapter as it was then; send it again")
        live = [i for i in range(len(groups)) if results[i] is None]
        if live:
            try:
                outcome: list[EngineResult] | JeffError = self._fast_many([groups[i] for i in live])
            except JeffError as error:
                outcome = error
            except ValueError as error:
                if TOO_LONG_MESSAGE not in str(error):
                    raise
                outcome = InputTooLong(str(error))
            for n, i in enumerate(live):
                results[i] = outcome if isinstance(outcome, JeffError) else outcome[n]
        return results  # type: ignore[return-value]

    def _runs(self, rows: list[tuple[int, Any]]) -> list[list[tuple[int, Any]]]:
        """The rows cut, in order, into runs of at most _prefixes_at_once distinct (adapter row, prefix text)."""
        runs: list[list[tuple[int, Any]]] = []
        keys: set[tuple[int, str]] = set()
        for index, row in rows:
            key = (index, row.prefix_text)
            if not runs or (key not in keys and len(keys) == self._prefixes_at_once):
                runs.append([])
                keys = set()
            keys.add(key)
            runs[-1].append((index, row))
        return runs

    def _fast_run(self, rows: list[tuple[int, Any]]) -> tuple[list[list[float]], list[int], dict[str, Any]]:
        batched, pool = self.batched, self.fast.prefixes
        slots, prefix_timing = batched.ensure_prefixes([(index, row.prefix_text) for index, row in rows],
                                                       self.max_tokens)
        try:
            for (_, row), slot in zip(rows, slots, strict=True):
                if pool.length(slot) + len(row.new_ids) > self.max_tokens:
                    raise ValueError(f"Question branch exceeds the {self.max_tokens}-token limit; "
                                     f"{TOO_LONG_MESSAGE}.")
            values, tokens, pass_timing = batched.decide([(index, slot, row)
                                                          for (index, row), slot in zip(rows, slots, strict=True)])
        finally:
            pool.unpin(slots)
        return values, tokens, {**prefix_timing, "passes": pass_timing["passes"],
                                "pass_rows": pass_timing["batch_rows"], "bucket": pass_timing["bucket"],
                                "adapters_in_pass": pass_timing["adapters_in_pass"]}

    def _fast_many(self, groups: list[tuple[str, Prepared]]) -> list[EngineResult]:
        """Every fast group of a predict_many call: the rows of all groups in order, cut into runs the pool holds
        (_runs), each run's prefixes made sure of and its passes run; then each group gets its rows' slice of the
        per-row lists, and the call-wide counters and wall time that every group of the call shares (the reference's
        timing contract: local_engine.py:469-516)."""
        started = time.perf_counter()
        rows = [(self.fast.index(None if adapter_id == BASE_ADAPTER else adapter_id), item)
                for adapter_id, prepared in groups for item in prepared.items or []]
        done = [self._fast_run(run) for run in self._runs(rows)]
        values = list(itertools.chain.from_iterable(d[0] for d in done))
        tokens = list(itertools.chain.from_iterable(d[1] for d in done))
        per_row = {name: list(itertools.chain.from_iterable(d[2][name] for d in done)) for name in ROW_TIMING}
        shared: dict[str, Any] = {"path": "fast", "model_ms": round((time.perf_counter() - started) * 1000, 3)}
        shared.update({name: sum(d[2][name] for d in done) for name in CALL_COUNTERS})
        shared.update(self.base_format)
        edges = list(itertools.accumulate((len(p.rows) for _, p in groups), initial=0))
        out = []
        for (_, prepared), lo, hi in zip(groups, edges, edges[1:], strict=False):
            row_timing = {name: per_row[name][lo:hi] for name in ROW_TIMING}
            row_timing["new_tokens"] = [len(item.new_ids) for item in prepared.items or []]
            out.append(EngineResult([[float(p) for p in v] for v in values[lo:hi]], dict(shared),
                                    [int(t) for t in tokens[lo:hi]], row_timing))
        return out
