"""Symbolic planner: placement states, transition plans, cost model, policies, tracing."""

from .state import (
    PlanStep,
    StateAxis,
    TensorState,
    axes_of,
    flat_axes_of,
    local_axis,
    mesh_dim_components,
    mesh_dims_components,
    partials_of,
    require_expanded_axes,
    sharded_axis,
    tensor_spec,
)
from .policy import (
    PlanPolicy,
    get_default_policy,
    get_optimization_policy,
    optimize,
    resolve_plan_policy,
    set_default_policy,
)
from .cost import (
    PlanAlternative,
    PlanCandidate,
    PlanCost,
    TensorRuntimeInfo,
    estimate_alternative_cost,
    estimate_plan_cost,
    rank_alternatives,
)
from .trace import ExecutionPlan, last_alternatives, last_candidates, last_plan, last_step_timings, set_last_plan
from .transitions import (
    BinaryClassification,
    BinaryPostRepartition,
    BinaryTransitionPlan,
    UnaryAxisDelta,
    UnaryClassification,
    UnaryTransitionPlan,
    build_binary_transition_plan,
    build_unary_transition_plan,
    classify_binary,
    classify_unary,
    clear_plan_cache,
)
