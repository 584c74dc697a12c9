"""Named compile phases: a caller can halt, dump or trace at any phase boundary.

Public surface kept from the reference's gnnc/pipeline/phase.py:50-246 so that
`gnnc-bench --trace`, `--stop-before/--stop-after` and `--print-ir-*` behave the
same for the B200 target: `PhasePipeline` (`add_callable_phase`, `extend`,
`names`, `find`, `run`), `CallablePhase`, `PhaseNotReached`, and `run`'s
keyword arguments and `(module, [(phase, passes), ...])` result. The
reference's MLIR-only StagePhase (a Lighthouse pass driver) has no counterpart:
every B200 phase is a Python callable over an fx graph or a kernel program.

Implementation. A pipeline keeps its phases in order plus a name -> position
map. `run` first turns its arguments into a `_Schedule` (how many phases run,
and for each of them whether to dump the module before / after it), checking
every named phase against the position map in one pass, and only then folds
the module through the scheduled phases. Nothing runs if any argument is bad.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from collections.abc import Callable, Iterable
from dataclasses import dataclass
from typing import Any

Trace = list[tuple[str, tuple[str, ...]]]


class PhaseNotReached(Exception):
    """A phase named in a request is not in the pipeline, or the stop point
    leaves it out so the request can never be honoured."""


class Phase(ABC):
    """One named step of a pipeline; `passes` lists what `--trace` reports for it."""

    def __init__(self, name: str) -> None:
        self.name = name

    @property
    @abstractmethod
    def passes(self) -> list[str]: ...

    @abstractmethod
    def run(self, module: Any, get_context: Callable[[], Any]) -> Any: ...


class CallablePhase(Phase):
    """A phase backed by a single function `module -> module`."""

    def __init__(self, name: str, fn: Callable[[Any], Any], passes: tuple[str, ...] = ()) -> None:
        super().__init__(name)
        self._fn = fn
        self._passes = list(passes)

    @property
    def passes(self) -> list[str]:
        return self._passes

    def run(self, module: Any, get_context: Callable[[], Any]) -> Any:
        return self._fn(module)


@dataclass(frozen=True)
class _Schedule:
    """What one `run` call does: phases [0, count) run; `dump_before[i]` /
    `dump_after[i]` say whether the module is printed around phase i."""

    count: int
    dump_before: tuple[bool, ...]
    dump_after: tuple[bool, ...]


def _banner(when: str, phase: str, module: Any) -> str:
    return f"// ---- IR {when} phase '{phase}' ---- //\n{module}"


class PhasePipeline:
    """Phases in execution order, addressable by name."""

    def __init__(self) -> None:
        self._order: list[Phase] = []
        self._index: dict[str, int] = {}

    # -- building ------------------------------------------------------------

    def _adopt(self, phases: Iterable[Phase]) -> None:
        incoming = list(phases)
        names = [p.name for p in incoming]
        clash = {n for n in names if n in self._index or names.count(n) > 1}
        if clash:
            raise ValueError(f"phase name(s) already in the pipeline: {sorted(clash)}")
        for p in incoming:
            self._index[p.name] = len(self._order)
            self._order.append(p)

    def add_callable_phase(
        self, name: str, fn: Callable[[Any], Any], passes: tuple[str, ...] = ()
    ) -> CallablePhase:
        phase = CallablePhase(name, fn, passes)
        self._adopt([phase])
        return phase

    def extend(self, other: PhasePipeline) -> None:
        """Append every phase of `other`, keeping its order (all or none)."""
        self._adopt(other._order)

    # -- queries -------------------------------------------------------------

    def names(self) -> list[str]:
        return [p.name for p in self._order]

    def find(self, name: str) -> Phase | None:
        at = self._index.get(name)
        return None if at is None else self._order[at]

    # -- running -------------------------------------------------------------

    def _schedule(self, stop_before, stop_after, print_before, print_after) -> _Schedule:
        if stop_before and stop_after:
            raise ValueError("give stop_before or stop_after, not both")
        wanted = {n for n in (stop_before, stop_after) if n} | set(print_before) | set(print_after)
        absent = sorted(n for n in wanted if n not in self._index)
        if absent:
            raise PhaseNotReached(f"no phase named {absent} in this pipeline {self.names()}")
        if stop_before:
            count = self._index[stop_before]
        elif stop_after:
            count = self._index[stop_after] + 1
        else:
            count = len(self._order)
        cut = sorted(n for n in set(print_before) | set(print_after) if self._index[n] >= count)
        if cut:
            raise PhaseNotReached(f"phase(s) {cut} would be printed but the stop point skips them")
        ran = self._order[:count]
        return _Schedule(
            count,
            tuple(p.name in print_before for p in ran),
            tuple(p.name in print_after for p in ran),
        )

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
    ) -> tuple[Any, Trace]:
        """Pass `module` through the phases up to the stop point.

        Returns the final module and the trace [(phase name, passes), ...] of
        the phases that ran. Raises PhaseNotReached for an unknown phase name
        or a print request past the stop, ValueError for two stops."""
        sched = self._schedule(stop_before, stop_after, print_ir_before, print_ir_after)
        trace: Trace = []
        for i in range(sched.count):
            phase = self._order[i]
            if sched.dump_before[i]:
                emit(_banner("before", phase.name, module))
            module = phase.run(module, get_context)
            trace.append((phase.name, tuple(phase.passes)))
            if sched.dump_after[i]:
                emit(_banner("after", phase.name, module))
        return module, trace
