"""Static + runtime cost model used to rank plan alternatives.

Each primitive has a fixed static score; with runtime information (local
shape, dtype size, mesh sizes, split shapes) every step also contributes the
bytes it moves forward and backward, its peak element count and the elements
it materialises.  A :class:`~.policy.PlanPolicy` folds the record into one
integer score.  Step scores, the byte accounting and the deterministic ranking
key follow ``src/torch_einshard/symbolic.py:159-188,296-324,622-877`` so that
the same alternative wins in this framework as in the reference.
"""

from dataclasses import dataclass, replace

from ..notation.spec import Axis
from .policy import coerce_policy, resolve_plan_policy

__all__ = [
    "PlanCost",
    "TensorRuntimeInfo",
    "PlanAlternative",
    "PlanCandidate",
    "step_cost",
    "estimate_plan_cost",
    "estimate_alternative_cost",
    "rank_alternatives",
    "sort_alternatives",
]


@dataclass(frozen=True)
class PlanCost:
    score: int
    collectives: int = 0
    materializations: int = 0
    peak_factor: int = 1
    forward_bytes: int = 0
    backward_bytes: int = 0
    peak_elements: int = 0
    materialized_elements: int = 0
    requires_shapes: bool = False
    invalid_reason: str = ""

    @property
    def total_bytes(self) -> int:
        return self.forward_bytes + self.backward_bytes

    def with_score(self, score) -> "PlanCost":
        return replace(self, score=score)


@dataclass(frozen=True)
class TensorRuntimeInfo:
    axes: tuple
    shape: tuple
    dtype_size: int

    def dim(self, axis_name):
        for index, axis in enumerate(self.axes):
            if axis.name == axis_name:
                return index
        return None

    def num_elements(self) -> int:
        count = 1
        for size in self.shape:
            count *= size
        return count

    def with_axis_size(self, axis_name, size) -> "TensorRuntimeInfo":
        dim = self.dim(axis_name)
        if dim is None:
            return self
        shape = list(self.shape)
        shape[dim] = size
        return TensorRuntimeInfo(self.axes, tuple(shape), self.dtype_size)

    def with_axis(self, axis_name, replacement) -> "TensorRuntimeInfo":
        axes = tuple(replacement if axis.name == axis_name else axis for axis in self.axes)
        return TensorRuntimeInfo(axes, self.shape, self.dtype_size)


@dataclass(frozen=True)
class PlanCandidate:
    name: str
    args: tuple = ()
    fallback_steps: tuple = ()
    status: str = "considered"
    reason: str = ""

    def with_result(self, status, reason="") -> "PlanCandidate":
        return replace(self, status=status, reason=reason)


@dataclass(frozen=True)
class PlanAlternative:
    name: str
    input0_steps: tuple = ()
    input1_steps: tuple = ()
    output_steps: tuple = ()
    candidates: tuple = ()
    cost: PlanCost = PlanCost(0)
    status: str = "ranked"
    reason: str = ""

    def steps(self) -> tuple:
        return (*self.input0_steps, *self.input1_steps, *self.output_steps)

    def with_result(self, status, reason="") -> "PlanAlternative":
        return replace(self, status=status, reason=reason)

    def with_cost(self, cost) -> "PlanAlternative":
        return replace(self, cost=cost)


# static (score, collectives, materializations, peak_factor) per primitive
_STATIC = {
    "rank_local_einsum": (0, 0, 0, 1),
    "reducescatter_forward_allgather_backward": (5, 1, 0, 1),
    "alltoall_repartition": (4, 1, 0, 1),
    "owner_swap": (6, 1, 0, 1),
    "broadcast_forward_allreduce_backward": (7, 1, 0, 1),
    "split_forward_allgather_backward": (3, 1, 0, 1),
    "allreduce_forward_identity_backward": (8, 1, 0, 1),
    "identity_forward_allreduce_backward": (8, 1, 0, 1),
    "allgather_forward_split_backward": (10, 1, 1, 2),
    "allgather_forward_reducescatter_backward": (10, 1, 1, 2),
}
_UNKNOWN_STEP = (20, 1, 0, 1)


def step_cost(step) -> PlanCost:
    score, collectives, materializations, peak = _STATIC.get(step.name, _UNKNOWN_STEP)
    return PlanCost(score, collectives=collectives, materializations=materializations, peak_factor=peak)


def _axis_extent(info, axis_name, shard_dim, mesh_sizes, split_shapes, direction):
    """Axis length after a split (largest shard) or a gather (global size)."""
    known = None if split_shapes is None else split_shapes.get((shard_dim, axis_name))
    if known is not None:
        return max(known) if direction == "split" else sum(known)
    dim = info.dim(axis_name)
    ways = 1 if mesh_sizes is None else mesh_sizes.get(shard_dim, 1)
    if direction == "gather":
        return info.shape[dim] * ways
    if direction == "split":
        ways = max(ways, 1)
        return max(1, -(-info.shape[dim] // ways))
    return info.shape[dim]


def _resize(info, axis_name, shard_dim, mesh_sizes, split_shapes, direction):
    if info.dim(axis_name) is None:
        return info
    return info.with_axis_size(
        axis_name, _axis_extent(info, axis_name, shard_dim, mesh_sizes, split_shapes, direction)
    )


_SPLITTING = ("split_forward_allgather_backward", "reducescatter_forward_allgather_backward")
_GATHERING = ("allgather_forward_split_backward", "allgather_forward_reducescatter_backward")
_REDUCING = (
    "allreduce_forward_identity_backward",
    "identity_forward_allreduce_backward",
    "broadcast_forward_allreduce_backward",
)


def _runtime_step_cost(step, info, mesh_sizes, split_shapes):
    static = step_cost(step)
    if info is None:
        return static, info
    before = info.num_elements()
    after = info
    fwd = bwd = peak = before
    materialized = 0
    needs_shapes = False
    if step.name == "rank_local_einsum":
        return PlanCost(0, peak_elements=before), info
    if step.name in _SPLITTING:
        axis_name, shard_dim = step.args
        after = _resize(info, axis_name, shard_dim, mesh_sizes, split_shapes, "split")
        bwd = peak = max(before, after.num_elements())
        known = None if split_shapes is None else split_shapes.get((shard_dim, axis_name))
        uneven_rs = step.name == "reducescatter_forward_allgather_backward" and known is not None and len(set(known)) != 1
        if uneven_rs:
            # uneven reduce-scatter runs as all-reduce + local split: the full tensor is materialised
            full = _resize(info, axis_name, shard_dim, mesh_sizes, split_shapes, "gather").num_elements()
            fwd = materialized = full
            peak = max(peak, full)
        after = after.with_axis(axis_name, Axis(axis_name, shard_dim))
    elif step.name in _GATHERING:
        axis_name, shard_dim = step.args
        after = _resize(info, axis_name, shard_dim, mesh_sizes, split_shapes, "gather")
        fwd = bwd = materialized = after.num_elements()
        peak = max(before, fwd)
        after = after.with_axis(axis_name, Axis(axis_name))
    elif step.name in _REDUCING:
        pass
    elif step.name == "alltoall_repartition":
        source_axis, dest_axis, shard_dim = step.args
        needs_shapes = True
        after = _resize(info, source_axis, shard_dim, mesh_sizes, split_shapes, "gather")
        after = _resize(after, dest_axis, shard_dim, mesh_sizes, split_shapes, "split")
        bwd = peak = max(before, after.num_elements())
        after = after.with_axis(source_axis, Axis(source_axis)).with_axis(dest_axis, Axis(dest_axis, shard_dim))
    elif step.name == "owner_swap":
        needs_shapes = True
    cost = PlanCost(
        static.score,
        static.collectives,
        static.materializations,
        static.peak_factor,
        fwd * info.dtype_size,
        bwd * info.dtype_size,
        peak,
        materialized,
        needs_shapes,
    )
    return cost, after


def _sum_costs(costs) -> PlanCost:
    total = PlanCost(0)
    for cost in costs:
        total = PlanCost(
            total.score + cost.score,
            total.collectives + cost.collectives,
            total.materializations + cost.materializations,
            max(total.peak_factor, cost.peak_factor),
            total.forward_bytes + cost.forward_bytes,
            total.backward_bytes + cost.backward_bytes,
            max(total.peak_elements, cost.peak_elements),
            total.materialized_elements + cost.materialized_elements,
            total.requires_shapes or cost.requires_shapes,
            total.invalid_reason or cost.invalid_reason,
        )
    return total


def _weighted(cost, policy):
    if policy is False or policy is None:
        return cost
    return cost.with_score(coerce_policy(policy).score(cost))


def estimate_plan_cost(steps, runtime_info=None, mesh_sizes=None, split_shapes=None, policy=None):
    """Cost of running ``steps`` on a tensor described by ``runtime_info``.

    Without runtime info only static scores are summed and no policy is
    applied; ``policy=False`` always returns the unweighted record.
    """
    costs = []
    info = runtime_info
    for step in steps:
        cost, info = _runtime_step_cost(step, info, mesh_sizes, split_shapes)
        costs.append(cost)
    if policy is None:
        policy = resolve_plan_policy() if runtime_info is not None else False
    return _weighted(_sum_costs(costs), policy)


def estimate_alternative_cost(alternative, input0_info, input1_info, output_info,
                              mesh_sizes=None, split_shapes=None, policy=None):
    parts = [
        estimate_plan_cost(alternative.input0_steps, input0_info, mesh_sizes, split_shapes, policy=False),
        estimate_plan_cost(alternative.input1_steps, input1_info, mesh_sizes, split_shapes, policy=False),
        estimate_plan_cost(alternative.output_steps, output_info, mesh_sizes, split_shapes, policy=False),
    ]
    if policy is None:
        policy = resolve_plan_policy()
    return _weighted(_sum_costs(parts), policy)


def sort_alternatives(alternatives) -> tuple:
    """Deterministic order: valid first, then score, peak, bytes, counts, name."""
    return tuple(sorted(alternatives, key=lambda alt: (
        bool(alt.cost.invalid_reason),
        alt.cost.score,
        alt.cost.peak_elements,
        alt.cost.total_bytes,
        alt.cost.materializations,
        alt.cost.collectives,
        alt.name,
    )))


def rank_alternatives(alternatives, input0_info=None, input1_info=None, output_info=None,
                      mesh_sizes=None, split_shapes=None, policy=None, output_infos=None):
    """Re-cost ``alternatives`` with runtime info and sort them.

    ``output_infos`` maps alternative names to output runtime infos for
    alternatives whose local output differs (e.g. before a post repartition).
    When only some alternatives can be costed, they are costed but the
    original order is kept.
    """
    have_inputs = input0_info is not None and input1_info is not None
    if have_inputs and output_info is not None:
        policy = resolve_plan_policy(policy=policy)
        recosted = tuple(
            alt.with_cost(estimate_alternative_cost(
                alt, input0_info, input1_info,
                output_infos.get(alt.name, output_info) if output_infos is not None else output_info,
                mesh_sizes, split_shapes, policy,
            ))
            for alt in alternatives
        )
        return sort_alternatives(recosted)
    if have_inputs and output_infos is not None:
        policy = resolve_plan_policy(policy=policy)
        recosted = tuple(
            alt.with_cost(estimate_alternative_cost(
                alt, input0_info, input1_info, output_infos[alt.name], mesh_sizes, split_shapes, policy,
            )) if alt.name in output_infos else alt
            for alt in alternatives
        )
        if all(alt.name in output_infos for alt in alternatives):
            return sort_alternatives(recosted)
        return recosted
    return sort_alternatives(alternatives)
