"""Optimization policies that weight the plan cost model.

Precedence when a call site resolves its policy: ``policy=`` argument, then
``optimize=`` argument, then the innermost ``with optimize(...)`` scope, then
``set_default_policy``, then ``training``.  Mode weights and the integer
scoring formula are those of ``src/torch_einshard/symbolic.py:191-293`` so that
plans rank identically.
"""

from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass

__all__ = [
    "PlanPolicy",
    "resolve_plan_policy",
    "optimize",
    "set_default_policy",
    "get_default_policy",
    "get_optimization_policy",
    "coerce_policy",
]


@dataclass(frozen=True)
class PlanPolicy:
    mode: str = "training"
    forward_byte_weight: int = 1
    backward_byte_weight: int = 1
    peak_element_weight: int = 1
    materialized_element_weight: int = 1
    collective_weight: int = 100
    materialization_weight: int = 200
    base_step_weight: int = 1

    @staticmethod
    def from_mode(mode):
        if isinstance(mode, PlanPolicy):
            return mode
        if mode is None:
            return PlanPolicy()
        try:
            overrides = _MODES[mode]
        except (KeyError, TypeError):
            raise ValueError(f"Unknown optimization policy {mode!r}") from None
        return PlanPolicy(mode=mode, **overrides)

    def score(self, cost) -> int:
        byte_term = cost.forward_bytes * self.forward_byte_weight + cost.backward_bytes * self.backward_byte_weight
        return (
            cost.score * self.base_step_weight
            + cost.collectives * self.collective_weight
            + cost.materializations * self.materialization_weight
            + byte_term // 1024
            + (cost.peak_elements * self.peak_element_weight) // 1024
            + (cost.materialized_elements * self.materialized_element_weight) // 1024
        )


_MODES = {
    "training": {},
    "inference": dict(backward_byte_weight=0),
    "memory": dict(
        peak_element_weight=64,
        materialized_element_weight=64,
        collective_weight=50,
        materialization_weight=400,
    ),
    "communication": dict(
        forward_byte_weight=8,
        backward_byte_weight=8,
        collective_weight=50,
        materialization_weight=100,
    ),
    "latency": dict(collective_weight=1000, materialization_weight=100),
}

_scoped_policy = ContextVar("torch_einshard_b200_plan_policy", default=None)
_process_default = None


def coerce_policy(value) -> PlanPolicy:
    return value if isinstance(value, PlanPolicy) else PlanPolicy.from_mode(value)


def resolve_plan_policy(optimize=None, policy=None) -> PlanPolicy:
    if optimize is not None and policy is not None:
        raise ValueError("Pass either optimize or policy, not both")
    if policy is not None:
        return coerce_policy(policy)
    if optimize is not None:
        return coerce_policy(optimize)
    scoped = _scoped_policy.get()
    if scoped is not None:
        return scoped
    if _process_default is not None:
        return _process_default
    return PlanPolicy.from_mode("training")


@contextmanager
def optimize(policy):
    token = _scoped_policy.set(coerce_policy(policy))
    try:
        yield
    finally:
        _scoped_policy.reset(token)


def set_default_policy(policy) -> None:
    global _process_default
    _process_default = None if policy is None else coerce_policy(policy)


def get_default_policy() -> PlanPolicy:
    return _process_default if _process_default is not None else PlanPolicy.from_mode("training")


def get_optimization_policy() -> PlanPolicy:
    return resolve_plan_policy()
