"""Phases group compile steps so a caller can stop, print or trace at a boundary.

Same surface as the reference's gnnc/pipeline/phase.py:50-246 (PhasePipeline,
CallablePhase, PhaseNotReached; add_callable_phase, extend, names, find, run
with stop_before / stop_after / print_ir_before / print_ir_after / emit), so
`--trace` and `--stop-*` keep working for the B200 target. The MLIR-only
StagePhase (a lazily built Lighthouse PipelineDriver) has no counterpart: the
B200 phases are Python callables over an fx graph and a kernel program.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from collections.abc import Callable
from typing import Any, TypeVar


class PhaseNotReached(Exception):
    """A requested phase isn't in this pipeline, or the stop excluded it."""


class Phase(ABC):
    """A named pipeline phase; `passes` is the step list `--trace` reports."""

    def __init__(self, name: str) -> None:
        self.name = name

    @property
    @abstractmethod
    def passes(self) -> list[str]: ...

    @abstractmethod
    def run(self, module: Any, get_context: Callable[[], Any]) -> Any: ...


class CallablePhase(Phase):
    """A phase that is a single callable; `passes` is supplied at construction."""

    def __init__(self, name: str, fn: Callable[[Any], Any], passes: tuple[str, ...] = ()) -> None:
        super().__init__(name)
        self._fn = fn
        self._passes = list(passes)

    @property
    def passes(self) -> list[str]:
        return self._passes

    def run(self, module: Any, get_context: Callable[[], Any]) -> Any:
        return self._fn(module)


_P = TypeVar("_P", bound=Phase)


class PhasePipeline:
    """An ordered list of phases plus the `run` that folds a module through them."""

    def __init__(self) -> None:
        self._phases: list[Phase] = []

    def add_callable_phase(
        self, name: str, fn: Callable[[Any], Any], passes: tuple[str, ...] = ()
    ) -> CallablePhase:
        return self._append(CallablePhase(name, fn, passes))

    def _append(self, phase: _P) -> _P:
        if self.find(phase.name) is not None:
            raise ValueError(f"duplicate phase name {phase.name!r}")
        self._phases.append(phase)
        return phase

    def extend(self, other: PhasePipeline) -> None:
        for phase in other._phases:
            if self.find(phase.name) is not None:
                raise ValueError(f"duplicate phase name {phase.name!r}")
        self._phases.extend(other._phases)

    def names(self) -> list[str]:
        return [phase.name for phase in self._phases]

    def find(self, name: str) -> Phase | None:
        return next((phase for phase in self._phases if phase.name == name), None)

    def run(
        self,
        module: Any,
        get_context: Callable[[], Any] = lambda: None,
        *,
        stop_before: str | None = None,
        stop_after: str | None = None,
        print_ir_before: frozenset[str] = frozenset(),
        print_ir_after: frozenset[str] = frozenset(),
        emit: Callable[[str], None] = print,
    ) -> tuple[Any, list[tuple[str, tuple[str, ...]]]]:
        """Fold `module` through the phases; returns (module, [(phase, passes), ...])."""
        if stop_before and stop_after:
            raise ValueError("stop_before and stop_after are mutually exclusive")
        names = self.names()
        referenced = {n for n in (stop_before, stop_after) if n}
        referenced |= set(print_ir_before) | set(print_ir_after)
        unknown = referenced - set(names)
        if unknown:
            raise PhaseNotReached(f"unknown phase(s) {sorted(unknown)}; phases: {names}")
        end = len(self._phases)
        if stop_before:
            end = names.index(stop_before)
        elif stop_after:
            end = names.index(stop_after) + 1
        missed = (set(print_ir_before) | set(print_ir_after)) - set(names[:end])
        if missed:
            raise PhaseNotReached(f"can't print at phase(s) {sorted(missed)}; the stop excludes them")
        trace: list[tuple[str, tuple[str, ...]]] = []
        for phase in self._phases[:end]:
            if phase.name in print_ir_before:
                emit(f"// -----// IR before {phase.name} //----- //\n{module}")
            module = phase.run(module, get_context)
            trace.append((phase.name, tuple(phase.passes)))
            if phase.name in print_ir_after:
                emit(f"// -----// IR after {phase.name} //----- //\n{module}")
        return module, trace
