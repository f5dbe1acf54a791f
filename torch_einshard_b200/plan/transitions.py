"""Transition planning: which collectives turn one placement into another.

Unary plans (``x -> z``) and binary plans (``x, y -> z``) are sequences of the
autograd-paired primitives named in :mod:`..parallel.mappings`.  The plans are
pure functions of the (ellipsis-free) specs and are memoised per spec key.

The step choice is a public contract (``last_plan()`` reports it and user code
asserts on it), so the decision rules are the reference's:
``src/torch_einshard/symbolic.py:448-568`` (unary) and ``:571-1147`` (binary).
The code below is organised differently: a small ``_BinaryPlanner`` object
carries the per-expression lookups instead of closures.
"""

from dataclasses import dataclass

from .cost import PlanAlternative, PlanCandidate, estimate_plan_cost, sort_alternatives
from .state import PlanStep, TensorState, partials_of, require_expanded_axes

__all__ = [
    "UnaryAxisDelta",
    "UnaryClassification",
    "BinaryClassification",
    "UnaryTransitionPlan",
    "BinaryTransitionPlan",
    "BinaryPostRepartition",
    "classify_unary",
    "classify_binary",
    "build_unary_transition_plan",
    "build_binary_transition_plan",
    "clear_plan_cache",
    "contracted_target_axis",
]

_CACHE = {}


def clear_plan_cache():
    _CACHE.clear()


def _spec_key(spec):
    return tuple((axis.name, axis.shard_dim) for axis in require_expanded_axes(spec)), partials_of(spec)


@dataclass(frozen=True)
class UnaryAxisDelta:
    name: str
    source: object
    target: object


@dataclass(frozen=True)
class UnaryClassification:
    input_state: TensorState
    output_state: TensorState
    placement_deltas: tuple
    removed_partials: tuple
    added_partials: tuple


@dataclass(frozen=True)
class BinaryClassification:
    input0_state: TensorState
    input1_state: TensorState
    output_state: TensorState
    free_axes: tuple
    shared_output_axes: tuple
    contracted_axes: tuple
    output_only_axes: tuple


@dataclass(frozen=True)
class UnaryTransitionPlan:
    classification: UnaryClassification
    steps: tuple

    def names(self):
        return [step.name for step in self.steps]


@dataclass(frozen=True)
class BinaryPostRepartition:
    shard_dim: str
    source_axis: str
    dest_axis: str


@dataclass(frozen=True)
class BinaryTransitionPlan:
    classification: BinaryClassification
    input0_steps: tuple
    input1_steps: tuple
    output_steps: tuple
    reduction_dims: tuple
    scatter_output_by_dim: tuple
    candidates: tuple = ()
    alternatives: tuple = ()
    top_ranked_alternative: str = ""
    post_repartition: BinaryPostRepartition = None

    def names(self):
        return [step.name for step in self.steps()]

    def steps(self):
        return (*self.input0_steps, *self.input1_steps, *self.output_steps)


# --------------------------------------------------------------------------- unary

def classify_unary(input_spec, output_spec) -> UnaryClassification:
    src = TensorState.from_spec(input_spec)
    dst = TensorState.from_spec(output_spec)
    if set(src.names()) != set(dst.names()):
        raise ValueError("Input and output axes must match")
    deltas = tuple(
        UnaryAxisDelta(axis.name, src.placement(axis.name), dst.placement(axis.name))
        for axis in dst.axes
        if src.placement(axis.name) != dst.placement(axis.name)
    )
    return UnaryClassification(
        input_state=src,
        output_state=dst,
        placement_deltas=deltas,
        removed_partials=tuple(p for p in src.partials if p not in dst.partials),
        added_partials=tuple(p for p in dst.partials if p not in src.partials),
    )


def _unary_owner_swap(src: TensorState, dst: TensorState) -> tuple:
    """Axis pairs that one atomic owner swap can move, or ``()``.

    A swap applies when every moved axis is sharded on both sides, the mesh
    dims involved form a permutation (or a single move), and no other axis
    touches the involved mesh dims.
    """
    if dst.partials or src.names() != dst.names():
        return ()
    moved = [
        (src.axis(axis.name), axis)
        for axis in dst.axes
        if src.axis(axis.name).shard_dim and axis.shard_dim and src.axis(axis.name).shard_dim != axis.shard_dim
    ]
    if not moved:
        return ()
    sources = [a.shard_dim for a, _ in moved]
    targets = [b.shard_dim for _, b in moved]
    if len(set(sources)) != len(sources) or len(set(targets)) != len(targets):
        return ()
    if len(moved) > 1 and set(sources) != set(targets):
        return ()
    involved = set(sources) | set(targets)
    moved_names = {a.name for a, _ in moved}
    for a, b in zip(src.axes, dst.axes):
        if a.name not in moved_names and (a.shard_dim in involved or b.shard_dim in involved):
            return ()
    return tuple(moved)


def build_unary_transition_plan(input_spec, output_spec) -> UnaryTransitionPlan:
    key = ("unary", _spec_key(input_spec), _spec_key(output_spec))
    if key in _CACHE:
        return _CACHE[key]

    cls = classify_unary(input_spec, output_spec)
    src, dst = cls.input_state, cls.output_state
    placement = src.placement_dict()
    partials = list(src.partials)
    steps = []

    # 1. resolve partial sums first: reduce-scatter onto a newly sharded axis if possible
    for partial in cls.removed_partials:
        scatter = next(
            (axis for axis in dst.axes
             if src.placement(axis.name) is None and dst.placement(axis.name) == partial),
            None,
        )
        if scatter is None:
            steps.append(PlanStep("allreduce_forward_identity_backward", (partial,)))
        else:
            steps.append(PlanStep("reducescatter_forward_allgather_backward", (scatter.name, partial)))
            placement[scatter.name] = partial
        partials.remove(partial)

    # 2. one atomic owner swap for mesh-dim permutations
    swapped = _unary_owner_swap(src, dst)
    if swapped:
        steps.append(PlanStep("owner_swap", (
            tuple(a.shard_dim for a, _ in swapped),
            tuple(b.shard_dim for _, b in swapped),
        )))
        for a, b in swapped:
            placement[a.name] = b.shard_dim
    swapped_names = {a.name for a, _ in swapped}

    # 3. per-axis gather / split
    for axis in dst.axes:
        if axis.name in swapped_names:
            continue
        have, want = placement[axis.name], dst.placement(axis.name)
        if have == want:
            continue
        if have is None:
            steps.append(PlanStep("split_forward_allgather_backward", (axis.name, want)))
        elif want is None:
            if have in dst.partials:
                steps.append(PlanStep("allgather_forward_reducescatter_backward", (axis.name, have)))
                partials.append(have)
            else:
                steps.append(PlanStep("allgather_forward_split_backward", (axis.name, have)))
        else:
            steps.append(PlanStep("allgather_forward_split_backward", (axis.name, have)))
            steps.append(PlanStep("split_forward_allgather_backward", (axis.name, want)))
        placement[axis.name] = want

    # 4. new partial obligations (identity forward, all-reduce backward)
    for partial in cls.added_partials:
        if partial not in partials:
            steps.append(PlanStep("identity_forward_allreduce_backward", (partial,)))
            partials.append(partial)

    # 5. axis order
    if src.names() != dst.names():
        steps.append(PlanStep("permute", (dst.names(),)))

    plan = UnaryTransitionPlan(cls, tuple(steps))
    _CACHE[key] = plan
    return plan


# -------------------------------------------------------------------------- binary

def classify_binary(input0_spec, input1_spec, output_spec) -> BinaryClassification:
    s0 = TensorState.from_spec(input0_spec)
    s1 = TensorState.from_spec(input1_spec)
    so = TensorState.from_spec(output_spec)
    n0, n1, no = set(s0.names()), set(s1.names()), set(so.names())
    both = n0 & n1
    return BinaryClassification(
        input0_state=s0,
        input1_state=s1,
        output_state=so,
        free_axes=tuple(n for n in so.names() if n in (n0 | n1) and n not in both),
        shared_output_axes=tuple(n for n in so.names() if n in both),
        contracted_axes=tuple(n for n in s0.names() if n in n1 and n not in no),
        output_only_axes=tuple(n for n in so.names() if n not in (n0 | n1)),
    )


def contracted_target_axis(axis0, axis1):
    """Placement both operands agree on for a contracted axis."""
    if axis0 == axis1:
        return axis0
    if axis0.local() and not axis1.local():
        return axis1
    if axis1.local() and not axis0.local():
        return axis0
    if axis0.shard_dim and axis1.shard_dim:
        return axis0
    raise NotImplementedError("Unsupported contracted-axis sharding mismatch")


def _move_axis_steps(axis, target, active_output_dims) -> tuple:
    """Steps that move one input axis to the target placement."""
    if axis.local():
        return (PlanStep("split_forward_allgather_backward", (axis.name, target.shard_dim)),)
    gather = (
        "allgather_forward_reducescatter_backward"
        if axis.shard_dim in active_output_dims
        else "allgather_forward_split_backward"
    )
    steps = [PlanStep(gather, (axis.name, axis.shard_dim))]
    if not target.local():
        steps.append(PlanStep("split_forward_allgather_backward", (axis.name, target.shard_dim)))
    return tuple(steps)


class _BinaryPlanner:
    def __init__(self, cls: BinaryClassification):
        self.cls = cls
        self.by_name0 = {a.name: a for a in cls.input0_state.axes}
        self.by_name1 = {a.name: a for a in cls.input1_state.axes}
        self.out_by_name = {a.name: a for a in cls.output_state.axes}
        self.out_partials = set(cls.output_state.partials)
        self.targets = {
            name: contracted_target_axis(self.by_name0[name], self.by_name1[name])
            for name in cls.contracted_axes
        }
        self.reduction_dims = []
        for name in cls.contracted_axes:
            target = self.targets[name]
            if not target.local() and target.shard_dim not in self.reduction_dims:
                self.reduction_dims.append(target.shard_dim)
        self.scatter_by_dim = {}
        for axis in cls.output_state.axes:
            sources = self._sources(axis.name)
            if axis.shard_dim in self.reduction_dims and any(s.local() or s == axis for s in sources):
                self.scatter_by_dim[axis.shard_dim] = axis.name
        self.active_output_dims = self.out_partials | {
            a.shard_dim for a in cls.output_state.axes if a.shard_dim
        }
        self.candidates = []

    def _sources(self, name):
        return [a for a in (self.by_name0.get(name), self.by_name1.get(name)) if a is not None]

    def post_repartition(self):
        gathers, splits = [], []
        for out_axis in self.cls.output_state.axes:
            sources = self._sources(out_axis.name)
            if len(sources) != 1 or sources[0] == out_axis:
                continue
            src = sources[0]
            if src.shard_dim and out_axis.local():
                gathers.append((src, out_axis))
            elif src.local() and out_axis.shard_dim:
                splits.append((src, out_axis))
        if len(gathers) != 1 or len(splits) != 1:
            return None
        src_axis, dst_axis = gathers[0][0], splits[0][1]
        dim = src_axis.shard_dim
        if dim != dst_axis.shard_dim or dim in self.reduction_dims or dim in self.out_partials:
            return None
        self.candidates.append(PlanCandidate(
            "alltoall_repartition",
            (src_axis.name, dst_axis.name, dim),
            (
                PlanStep("allgather_forward_reducescatter_backward", (src_axis.name, dim)),
                PlanStep("split_forward_allgather_backward", (dst_axis.name, dim)),
            ),
        ))
        return BinaryPostRepartition(shard_dim=dim, source_axis=src_axis.name, dest_axis=dst_axis.name)

    def input_steps(self, state: TensorState) -> tuple:
        steps = []
        # contracted axes sharded on both sides but on different mesh dims
        moves = [
            (axis, self.targets[axis.name])
            for axis in state.axes
            if axis.name in self.targets
            and axis != self.targets[axis.name]
            and not axis.local()
            and not self.targets[axis.name].local()
        ]
        swapped = set()
        if len(moves) >= 2:
            sources = tuple(a.shard_dim for a, _ in moves)
            targets = tuple(t.shard_dim for _, t in moves)
            involved = set(sources) | set(targets)
            names = {a.name for a, _ in moves}
            ok = (
                len(set(sources)) == len(sources)
                and len(set(targets)) == len(targets)
                and set(sources) == set(targets)
                and all(a.name in names or a.shard_dim not in involved for a in state.axes)
            )
            if not ok:
                raise NotImplementedError(
                    "Multiple contracted-axis shard-dimension changes require an owner-swap-compatible permutation"
                )
            swap = PlanStep("owner_swap", (sources, targets))
            steps.append(swap)
            self.candidates.append(PlanCandidate("owner_swap", swap.args))
            swapped = names

        # free axes that will be reduce-scattered onto: gather them first
        gathered_for_scatter = set()
        for axis in state.axes:
            if axis.name in self.targets or axis.name not in self.out_by_name:
                continue
            out_axis = self.out_by_name[axis.name]
            if self.scatter_by_dim.get(out_axis.shard_dim) == out_axis.name and axis == out_axis:
                steps.append(PlanStep("allgather_forward_split_backward", (axis.name, axis.shard_dim)))
                gathered_for_scatter.add(axis.name)

        for axis in state.axes:
            if axis.name in gathered_for_scatter:
                continue
            if axis.name in self.targets:
                if axis.name not in swapped and axis != self.targets[axis.name]:
                    steps.extend(_move_axis_steps(axis, self.targets[axis.name], self.active_output_dims))
                continue
            if axis.name not in self.out_by_name:
                continue
            out_axis = self.out_by_name[axis.name]
            if axis == out_axis or (axis.local() and out_axis.shard_dim in self.reduction_dims):
                continue
            steps.extend(_move_axis_steps(axis, out_axis, self.active_output_dims))

        # output axes sharded on a mesh dim this operand is replicated over:
        # its gradient must be all-reduced over that dim
        names = set(state.names())
        own_dims = {a.shard_dim for a in state.axes if a.shard_dim}
        reduced_backward = {
            step.args[-1] for step in steps
            if step.name in ("allgather_forward_reducescatter_backward", "identity_forward_allreduce_backward")
        }
        for out_axis in self.cls.output_state.axes:
            dim = out_axis.shard_dim
            if not dim or out_axis.name in names:
                continue
            if dim in self.reduction_dims or dim in own_dims or dim in reduced_backward:
                continue
            steps.append(PlanStep("identity_forward_allreduce_backward", (dim,)))
            reduced_backward.add(dim)
        return tuple(steps)

    def output_steps(self) -> tuple:
        steps = [PlanStep("rank_local_einsum")]
        for dim in self.reduction_dims:
            scatter = self.scatter_by_dim.get(dim)
            if dim in self.out_partials:
                if scatter is not None:
                    steps.append(PlanStep("split_forward_allgather_backward", (scatter, dim)))
                continue
            if scatter is None:
                steps.append(PlanStep("allreduce_forward_identity_backward", (dim,)))
            else:
                steps.append(PlanStep("reducescatter_forward_allgather_backward", (scatter, dim)))
        return tuple(steps)


def _without_axis_steps(steps, post):
    """Input steps of the post-repartition alternative."""
    out = []
    for step in steps:
        if step.args and step.args[0] == post.source_axis:
            continue
        if step.args and step.args[0] == post.dest_axis:
            out.append(PlanStep("identity_forward_allreduce_backward", (post.shard_dim,)))
        else:
            out.append(step)
    return tuple(out)


def build_binary_transition_plan(input0_spec, input1_spec, output_spec) -> BinaryTransitionPlan:
    key = ("binary", _spec_key(input0_spec), _spec_key(input1_spec), _spec_key(output_spec))
    if key in _CACHE:
        return _CACHE[key]

    cls = classify_binary(input0_spec, input1_spec, output_spec)
    planner = _BinaryPlanner(cls)
    post = planner.post_repartition()
    in0 = planner.input_steps(cls.input0_state)
    in1 = planner.input_steps(cls.input1_state)
    out = planner.output_steps()
    candidates = tuple(planner.candidates)

    alternatives = [PlanAlternative(
        "default", in0, in1, out, candidates, estimate_plan_cost((*in0, *in1, *out)),
    )]
    if any(step.name == "reducescatter_forward_allgather_backward" for step in out):
        expanded = []
        for step in out:
            if step.name == "reducescatter_forward_allgather_backward":
                axis_name, dim = step.args
                expanded.append(PlanStep("allreduce_forward_identity_backward", (dim,)))
                expanded.append(PlanStep("split_forward_allgather_backward", (axis_name, dim)))
            else:
                expanded.append(step)
        expanded = tuple(expanded)
        alternatives.append(PlanAlternative(
            "allreduce_then_split", in0, in1, expanded, candidates,
            estimate_plan_cost((*in0, *in1, *expanded)),
        ))
    if post is not None:
        a0, a1 = _without_axis_steps(in0, post), _without_axis_steps(in1, post)
        a_out = (*out, PlanStep("alltoall_repartition", (post.source_axis, post.dest_axis, post.shard_dim)))
        alternatives.append(PlanAlternative(
            "alltoall_repartition", a0, a1, a_out, candidates,
            estimate_plan_cost((*a0, *a1, *a_out)),
            reason="requires runtime split-shape validation",
        ))
    alternatives = sort_alternatives(alternatives)

    plan = BinaryTransitionPlan(
        classification=cls,
        input0_steps=in0,
        input1_steps=in1,
        output_steps=out,
        reduction_dims=tuple(planner.reduction_dims),
        scatter_output_by_dim=tuple(planner.scatter_by_dim.items()),
        candidates=candidates,
        alternatives=alternatives,
        top_ranked_alternative=alternatives[0].name,
        post_repartition=post,
    )
    _CACHE[key] = plan
    return plan
