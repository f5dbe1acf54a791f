"""Execution tracing: which primitives ran, which candidates were considered.

Every executed ``einshard``/``einfft``/... call records an :class:`ExecutionPlan`
and publishes it through :func:`set_last_plan`, so callers (and tests) can ask
``last_plan()``, ``last_candidates()`` and ``last_alternatives()`` what the last
call on this process did.  Interface of ``src/torch_einshard/symbolic.py:386-445``.

Beyond the reference, :class:`ExecutionPlan` can carry per-step device timings
(``EINSHARD_STEP_TIMING=1``) and wraps each executed step in an NVTX range when
CUDA is available, so a profiler timeline shows plan steps by name.
"""

import os

from .cost import PlanCandidate
from .state import PlanStep

__all__ = [
    "ExecutionPlan",
    "set_last_plan",
    "last_plan",
    "last_candidates",
    "last_alternatives",
    "last_step_timings",
]

_TIMING = os.environ.get("EINSHARD_STEP_TIMING", "0") not in ("", "0")


def _nvtx_range(name):
    try:
        import torch
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            return torch.cuda.nvtx.range(name)
    except Exception:  # noqa: BLE001 - tracing must never break execution
        pass
    return None


class ExecutionPlan:
    def __init__(self):
        self.steps = []
        self.candidates = []
        self.alternatives = []
        self.timings = []

    def add(self, name, *args):
        self.steps.append(PlanStep(name, tuple(args)))

    def execute(self, name, fn, *fn_args, step_args=(), **fn_kwargs):
        self.add(name, *step_args)
        rng = _nvtx_range(f"einshard:{name}")
        if rng is None and not _TIMING:
            return fn(*fn_args, **fn_kwargs)
        timer = _StepTimer(name) if _TIMING else None
        if rng is not None:
            rng.__enter__()
        try:
            result = fn(*fn_args, **fn_kwargs)
        finally:
            if rng is not None:
                rng.__exit__(None, None, None)
        if timer is not None:
            self.timings.append(timer.stop())
        return result

    def consider(self, candidate, *args, status="considered", reason="", fallback_steps=()):
        if isinstance(candidate, PlanCandidate):
            self.candidates.append(candidate.with_result(status, reason))
        else:
            self.candidates.append(PlanCandidate(candidate, tuple(args), tuple(fallback_steps), status, reason))

    def rank(self, alternatives, selected=None, reason=""):
        self.alternatives = [
            alt.with_result("selected", reason) if alt.name == selected else alt
            for alt in alternatives
        ]

    def names(self):
        return [step.name for step in self.steps]

    def snapshot(self):
        return tuple(self.steps)


class _StepTimer:
    """Wall/device time of one step (device time when the step ran on CUDA)."""

    def __init__(self, name):
        import time
        import torch
        self.name = name
        self._cuda = torch.cuda.is_available() and torch.cuda.is_initialized()
        if self._cuda:
            self._start = torch.cuda.Event(enable_timing=True)
            self._end = torch.cuda.Event(enable_timing=True)
            self._start.record()
        self._t0 = time.perf_counter()

    def stop(self):
        import time
        if self._cuda:
            self._end.record()
            self._end.synchronize()
            return (self.name, self._start.elapsed_time(self._end))
        return (self.name, (time.perf_counter() - self._t0) * 1e3)


_last = {"steps": (), "candidates": (), "alternatives": (), "timings": ()}


def set_last_plan(plan):
    if isinstance(plan, ExecutionPlan):
        _last["steps"] = tuple(plan.steps)
        _last["candidates"] = tuple(plan.candidates)
        _last["alternatives"] = tuple(plan.alternatives)
        _last["timings"] = tuple(plan.timings)
    else:
        _last["steps"] = tuple(plan)
        _last["candidates"] = ()
        _last["alternatives"] = ()
        _last["timings"] = ()


def last_plan():
    return _last["steps"]


def last_candidates():
    return _last["candidates"]


def last_alternatives():
    return _last["alternatives"]


def last_step_timings():
    """``(step_name, milliseconds)`` pairs of the last plan (timing enabled only)."""
    return _last["timings"]
