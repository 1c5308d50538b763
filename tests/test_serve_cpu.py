"""The configuration 5 serving harness on the CPU, against a fake engine on a virtual clock: the call stream's
distributions, the sticky routing of (adapter, prefix) to replicas, and the micro-batching rule of the reference
scheduler (runtime/python/src/jeff_runtime/scheduler.py, Scheduler._gather): a batch closes window_ms after its
oldest waiting call arrived or once max_batch_rows calls wait, takes calls in arrival order, and is sent as one
group per adapter; latency runs from arrival to the end of the engine call."""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import pytest

from jeff_b200 import serve_bench as sb


class VirtualClock:
    def __init__(self) -> None:
        self.t = 0.0

    def clock(self) -> float:
        return self.t

    def sleep(self, seconds: float) -> None:
        self.t += max(seconds, 1e-9)


@dataclass
class FakeResult:
    probabilities: list
    timing: dict


@dataclass
class FakeEngine:
    clock: VirtualClock
    service_s: float = 0.010
    calls: list = field(default_factory=list)

    def prepare(self, adapter: str, rows: list[dict]) -> list[dict]:
        return rows

    def predict_many(self, groups):
        groups = [(adapter, getattr(rows, "rows", rows)) for adapter, rows in groups]
        self.calls.append([(adapter, len(rows)) for adapter, rows in groups])
        self.clock.t += self.service_s
        return [FakeResult([[0.5, 0.5]] * len(rows), {"prefix_misses": 0, "passes": len(groups)})
                for _, rows in groups]


def stream(arrivals, adapters=None) -> sb.Calls:
    n = len(arrivals)
    adapters = adapters if adapters is not None else [1] * n
    return sb.Calls(np.asarray(arrivals, dtype=np.float64), np.asarray(adapters), np.zeros(n, dtype=np.int64),
                    [np.array([1, 2, 3])] * n, np.full(n, 2))


def test_a_batch_closes_one_window_after_its_oldest_call() -> None:
    vc = VirtualClock()
    engine = FakeEngine(vc)
    calls = stream([0.0, 0.0005, 0.002])
    served = sb.serve(engine, calls, window_ms=1.0, clock=vc.clock, sleep=vc.sleep)
    assert served.batch_rows == [2, 1]
    lat = sb.latency_ms(calls, served)
    # the first batch closes at 1 ms and runs 10 ms; the third call waited through it and runs next
    assert lat == pytest.approx([11.0, 10.5, 19.0], abs=1e-3)


def test_a_full_batch_does_not_wait_for_the_window_and_takes_arrival_order() -> None:
    vc = VirtualClock()
    engine = FakeEngine(vc, service_s=0.001)
    calls = stream([0.0] * 100, adapters=[1 + i % 3 for i in range(100)])
    served = sb.serve(engine, calls, window_ms=50.0, max_batch_rows=64, clock=vc.clock, sleep=vc.sleep)
    assert served.batch_rows == [64, 36]
    # the 36 left over still wait for their window (50 ms after their arrival at 0), then run 1 ms
    assert served.done[0] == pytest.approx(0.001) and served.done[99] == pytest.approx(0.051)
    # one group per adapter, in order of first appearance, rows of the batch split among them
    assert engine.calls[0] == [("adapter-1", 22), ("adapter-2", 21), ("adapter-3", 21)]


def test_an_idle_server_sleeps_until_the_next_arrival() -> None:
    vc = VirtualClock()
    engine = FakeEngine(vc, service_s=0.002)
    calls = stream([1.0, 5.0])
    served = sb.serve(engine, calls, window_ms=1.0, clock=vc.clock, sleep=vc.sleep)
    assert served.batches == 2
    assert sb.latency_ms(calls, served) == pytest.approx([3.0, 3.0], abs=1e-3)
    assert served.elapsed == pytest.approx(5.003)


def test_the_call_stream_follows_configuration_5() -> None:
    calls = sb.make_calls(20000, 1000.0)
    lengths = np.array([len(ids) for ids in calls.new_ids])
    assert lengths.min() >= 1 and lengths.max() <= 1024
    assert abs(lengths.mean() - 96) < 4
    assert abs(np.diff(calls.arrival).mean() - 1e-3) < 5e-5 and np.all(np.diff(calls.arrival) >= 0)
    freq = np.bincount(calls.adapter, minlength=33)[1:] / len(calls)
    assert freq[0] == pytest.approx(sb.zipf_weights(32, 1.1)[0], abs=0.01) and freq[0] > 5 * freq[-1]
    assert set(np.unique(calls.prefix)) == set(range(64))
    assert calls.count.min() >= 2 and calls.count.max() <= 32
    again = sb.make_calls(20000, 1000.0)
    assert np.array_equal(again.adapter, calls.adapter) and np.array_equal(again.new_ids[7], calls.new_ids[7])
    assert np.all(sb.make_calls(10, math.inf).arrival == 0)


def test_routing_keeps_each_binding_on_one_replica_and_spreads_them() -> None:
    calls = sb.make_calls(5000, 1.0)
    shares = sb.route(calls.adapter, calls.prefix, 8)
    assert sorted(i for share in shares for i in share) == list(range(len(calls)))
    owner = {}
    for r, share in enumerate(shares):
        for i in share:
            key = (int(calls.adapter[i]), int(calls.prefix[i]))
            assert owner.setdefault(key, r) == r
    bindings = np.bincount(list(owner.values()), minlength=8)
    assert bindings.min() > 0.6 * bindings.mean()
    assert sb.route(calls.adapter, calls.prefix, 1) == [list(range(len(calls)))]


def test_prepared_calls_are_joined_per_adapter() -> None:
    from jeff_b200.engine import Prepared

    vc = VirtualClock()
    engine = FakeEngine(vc, service_s=0.001)
    calls = stream([0.0] * 5, adapters=[2, 1, 2, 2, 1])
    ready = [Prepared([{"call": i}], [f"item {i}"], "fast", 7) for i in range(5)]
    sb.serve(engine, calls, window_ms=1.0, clock=vc.clock, sleep=vc.sleep, prepared=ready)
    assert engine.calls == [[("adapter-2", 3), ("adapter-1", 2)]]
