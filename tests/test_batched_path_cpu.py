"""BatchedPath's host logic on the CPU, with the GPU passes replaced by a stand-in: decide() groups rows by new-token
bucket (the smallest of 32 ... 1024 holding the row), cuts each bucket into passes of at most max_rows(N) rows, runs
each at the smallest batch bucket holding its rows (the reference's batched_path.py:528-562), hands every pass to
run_passes in one call, and returns each row's probabilities (cut to its option count), input tokens and timing in
the rows' own order."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np

from jeff_b200 import constants as C
from jeff_b200.batched_path import BatchedPath, Row, max_rows


def fake_path(prefix_len: int = 10, rows_cap: int = 64, max_tokens: int = C.MAX_PASS_TOKENS):
    calls: list[list[tuple[int, int, list[int]]]] = []

    def run_passes(passes):
        calls.append([(b, n, [row.new_ids[0] for _, _, row in part]) for b, n, part, _ in passes])
        out = []
        for b, n, part, lengths in passes:
            assert len(part) <= b and all(length == prefix_len for length in lengths)
            probs = np.zeros((b, C.READOUT_ROWS), dtype=np.float32)
            for j, (_, _, row) in enumerate(part):
                probs[j] = row.new_ids[0] + np.arange(C.READOUT_ROWS) / 1000.0   # identifies the row and option
            out.append((probs, 1.5))
        return out

    path = SimpleNamespace(_check=lambda rows: [prefix_len] * len(rows), run_passes=run_passes,
                           ws=SimpleNamespace(rows=rows_cap), max_tokens=max_tokens, batch_buckets=C.BATCH_BUCKETS)
    return path, calls


def rows_of(lengths: list[int], count: int = 3) -> list[tuple[int, int, Row]]:
    # the first token id names the row, so a result can be traced back to its row
    return [(1 + i % 2, 5, Row("p", [i] + [7] * (n - 1), count)) for i, n in enumerate(lengths)]


def test_decide_groups_by_bucket_and_answers_in_row_order() -> None:
    path, calls = fake_path()
    lengths = [20, 100, 33, 1, 64, 65, 500, 32]
    results, tokens, timing = BatchedPath.decide(path, rows_of(lengths))
    assert len(calls) == 1                                     # every pass in one run_passes call
    assert [(b, n, ids) for b, n, ids in calls[0]] == [(4, 32, [0, 3, 7]), (2, 64, [2, 4]), (2, 128, [1, 5]),
                                                       (1, 512, [6])]
    for i, probs in enumerate(results):
        assert len(probs) == 3 and probs[0] == i and abs(probs[2] - (i + 0.002)) < 1e-6
    assert tokens == [10 + n for n in lengths]
    assert timing["passes"] == 4 and timing["model_ms"] == 6.0
    assert timing["bucket"] == [32, 128, 64, 32, 64, 128, 512, 32]
    assert timing["batch_rows"] == [3, 2, 2, 3, 2, 2, 1, 3]
    assert timing["adapters_in_pass"] == [2, 1, 1, 2, 1, 1, 1, 2]


def test_decide_cuts_a_bucket_into_passes_of_at_most_max_rows() -> None:
    assert max_rows(1024) == C.MAX_PASS_TOKENS // 1024
    path, calls = fake_path()
    n_rows = max_rows(1024) + 3
    results, _, timing = BatchedPath.decide(path, rows_of([1000] * n_rows))
    assert [(b, n, len(ids)) for b, n, ids in calls[0]] == [(max_rows(1024), 1024, max_rows(1024)), (4, 1024, 3)]
    assert [r[0] for r in results] == list(range(n_rows))
    path, calls = fake_path(rows_cap=8)                        # a smaller workspace caps the passes too
    BatchedPath.decide(path, rows_of([30] * 20))
    assert [(b, len(ids)) for b, _, ids in calls[0]] == [(8, 8), (8, 8), (4, 4)]


def test_a_path_with_the_configuration_5_batch_buckets_pads_to_them() -> None:
    """batch_buckets (1, 8, 16, 32, 64), the serving configuration's graph buckets: 5 rows of one new-token bucket run
    as one pass of 8 rows, 20 as one of 32; a bucket list that does not run from 1 to 64 is refused."""
    import pytest

    path, calls = fake_path()
    path.batch_buckets = (1, 8, 16, 32, 64)
    BatchedPath.decide(path, rows_of([20] * 5))
    BatchedPath.decide(path, rows_of([20] * 20))
    assert [b for b, _, _ in calls[0]] == [8] and [b for b, _, _ in calls[1]] == [32]
    with pytest.raises(ValueError, match="from 1 to 64"):
        BatchedPath(SimpleNamespace(), batch_buckets=(8, 16, 64))   # type: ignore[arg-type]
