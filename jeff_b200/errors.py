"""The result, request and error types the reference's callers dispatch on.

The reference's scheduler sorts a group's outcome with `isinstance(result, jeff.errors.JeffError)`
(runtime/python/src/jeff_runtime/scheduler.py:340) and its client raises the typed errors it is handed
(packages/python/src/jeff/client.py:151-169). So when the reference's client package `jeff` is importable, every name
here IS the reference's own class (jeff.errors, jeff.engine): B200Engine's results and errors then pass those checks
unchanged. Without the package (the GPU box carries only this repository) the same names are defined here with the
reference's fields, base classes and messages, so the engine and its tests behave the same either way.

REFERENCE_TYPES tells which of the two is in use."""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass, field
from typing import Any

BASE_ADAPTER = "base"

try:  # the reference's own types, when its client package is on the path
    from jeff.engine import EngineResult, Prepared
    from jeff.errors import EngineError, InputTooLong, InvalidRequest, JeffError, NotInstalled, TooManyLabels

    REFERENCE_TYPES = True
except ImportError:
    REFERENCE_TYPES = False

    class JeffError(Exception):  # type: ignore[no-redef]
        """Root of the typed errors; a group's result is either an EngineResult or one of these."""

        request_id: str | None = None

    class EngineError(JeffError):  # type: ignore[no-redef]
        """The engine cannot serve a request as configured, or broke its own contract."""

    class InvalidRequest(JeffError):  # type: ignore[no-redef]
        """A row the engine cannot read."""

    class InputTooLong(JeffError):  # type: ignore[no-redef]
        """A request longer than the engine's token limit; refused, never truncated."""

    class TooManyLabels(JeffError):  # type: ignore[no-redef]
        """More options than the adapter was trained on."""

    class NotInstalled(JeffError):  # type: ignore[no-redef]
        def __init__(self, function_id: str, why: str = "") -> None:
            adapter = function_id.rsplit(".", 1)[0] if function_id.count(".") >= 3 else function_id
            super().__init__(f"{function_id} is not installed{(': ' + why) if why else ''}. Install it with: jeff "
                             f"pull {adapter}")
            self.function_id = function_id

    @dataclass(frozen=True)
    class EngineResult:  # type: ignore[no-redef]
        """Per row its option probabilities; the group's timing; per row its input tokens and its own timing lists."""

        probabilities: list[list[float]]
        timing: dict[str, Any] = field(default_factory=dict)
        input_tokens: list[int] | None = None
        row_timing: dict[str, list[Any]] | None = None

    @dataclass(frozen=True)
    class Prepared:  # type: ignore[no-redef]
        """A request's checked rows, one prepared item per row, the route that runs them and the adapter load they
        were prepared for."""

        rows: list[dict[str, Any]]
        items: list[Any] | None = None
        route: str | None = None
        generation: Any = None

        def __post_init__(self) -> None:
            if self.items is not None and len(self.items) != len(self.rows):
                raise EngineError(f"Prepared has {len(self.items)} items for {len(self.rows)} rows")

        def part(self, start: int, stop: int) -> Prepared:
            if (start, stop) == (0, len(self.rows)):
                return self
            items = None if self.items is None else self.items[start:stop]
            return Prepared(self.rows[start:stop], items, self.route, self.generation)

        @staticmethod
        def join(parts: Sequence[Prepared]) -> Prepared:
            if len(parts) == 1:
                return parts[0]
            kinds = {(p.route, p.generation) for p in parts}
            if len(kinds) > 1:
                raise EngineError(f"Prepared.join was given parts of several routes or generations "
                                  f"{sorted(map(str, kinds))}")
            with_items = [p.items is not None for p in parts]
            if any(with_items) and not all(with_items):
                raise EngineError("Prepared.join was given parts with items and parts without")
            items = [it for p in parts for it in p.items] if all(with_items) else None  # type: ignore[union-attr]
            route, generation = kinds.pop()
            return Prepared([r for p in parts for r in p.rows], items, route, generation)


__all__ = ["BASE_ADAPTER", "EngineError", "EngineResult", "InputTooLong", "InvalidRequest", "JeffError",
           "NotInstalled", "Prepared", "REFERENCE_TYPES", "TooManyLabels"]
