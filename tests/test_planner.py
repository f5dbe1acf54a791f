"""Symbolic planner: placement states, unary/binary transition plans, cost
model, policies and execution tracing."""

import pytest

from torch_einshard_b200.notation.parser import parse_sharding
from torch_einshard_b200.plan import (
    ExecutionPlan,
    PlanPolicy,
    PlanStep,
    TensorRuntimeInfo,
    TensorState,
    build_binary_transition_plan,
    build_unary_transition_plan,
    classify_binary,
    classify_unary,
    clear_plan_cache,
    estimate_alternative_cost,
    estimate_plan_cost,
    get_default_policy,
    get_optimization_policy,
    last_alternatives,
    last_candidates,
    last_plan,
    local_axis,
    optimize,
    rank_alternatives,
    resolve_plan_policy,
    set_default_policy,
    set_last_plan,
    sharded_axis,
    tensor_spec,
)


def _steps(plan_steps):
    return [(s.name, s.args) for s in plan_steps]


def test_tensor_state_placements_partials_and_replication():
    x, _, _ = parse_sharding("a/dp b c/tp // sp -> a b c")
    st = TensorState.from_spec(x)
    assert st.placement_dict() == {"a": "dp", "b": None, "c": "tp"} and st.partials == ("sp",)
    x, _, _ = parse_sharding("a/dp b // tp -> a b")
    assert TensorState.from_spec(x, mesh_dim_names=("dp", "sp", "tp")).replicated_dims == ("sp",)
    x, _, _ = parse_sharding("a/dp-sp b // tp-sp -> a b")
    assert TensorState.from_spec(x, mesh_dim_names=("dp", "sp", "tp", "pp")).replicated_dims == ("pp",)
    x, _, _ = parse_sharding("a/sp1 b -> a b")
    assert TensorState.from_spec(x, mesh_dim_names=("sp1-sp2", "tp")).replicated_dims == ("tp",)
    x, _, _ = parse_sharding("a (b/tp c) -> a b/tp c")
    assert TensorState.from_spec(x).placement_dict() == {"a": None, "b": "tp", "c": None}
    with pytest.raises(ValueError, match="unique axis names"):
        TensorState.from_spec(parse_sharding("a a -> a")[0])
    with pytest.raises(ValueError, match="ellipsis expansion"):
        TensorState.from_spec(parse_sharding("... c -> ... c")[0])


def test_unary_classification_and_plans():
    x, _, z = parse_sharding("a/dp b // tp -> a b/sp // dp")
    cls = classify_unary(x, z)
    assert [(d.name, d.source, d.target) for d in cls.placement_deltas] == [("a", "dp", None), ("b", None, "sp")]
    assert cls.removed_partials == ("tp",) and cls.added_partials == ("dp",)
    with pytest.raises(ValueError, match="axes must match"):
        classify_unary(*parse_sharding("a b -> a c")[::2])
    cases = {
        "a b -> a/dp b": [("split_forward_allgather_backward", ("a", "dp"))],
        "a/dp b -> a b": [("allgather_forward_split_backward", ("a", "dp"))],
        "a/dp b/sp -> a/sp b/dp": [("owner_swap", (("dp", "sp"), ("sp", "dp")))],
        "a/dp b/sp -> a/sp b/sp": [("allgather_forward_split_backward", ("a", "dp")),
                                   ("split_forward_allgather_backward", ("a", "sp"))],
        "a b // tp -> a/tp b": [("reducescatter_forward_allgather_backward", ("a", "tp"))],
        "a/tp b -> a b // tp": [("allgather_forward_reducescatter_backward", ("a", "tp"))],
        "b a -> a b // dp": [("identity_forward_allreduce_backward", ("dp",)), ("permute", (("a", "b"),))],
    }
    for expr, expected in cases.items():
        x, _, z = parse_sharding(expr)
        assert _steps(build_unary_transition_plan(x, z).steps) == expected, expr
    x, _, z = parse_sharding("a/dp b/dp c/sp d/tp -> a/sp b/tp c/dp d/dp")
    assert "owner_swap" not in build_unary_transition_plan(x, z).names()


def test_binary_plans():
    clear_plan_cache()
    x, y, z = parse_sharding("a b/tp, b c -> a/tp c")
    first = build_binary_transition_plan(x, y, z)
    assert build_binary_transition_plan(x, y, z) is first
    clear_plan_cache()
    assert build_binary_transition_plan(x, y, z) is not first
    assert _steps(first.output_steps) == [("rank_local_einsum", ()),
                                          ("reducescatter_forward_allgather_backward", ("a", "tp"))]
    assert first.scatter_output_by_dim == (("tp", "a"),)
    assert [(a.name, a.cost.score) for a in first.alternatives] == [("default", 8), ("allreduce_then_split", 14)]

    x, y, z = parse_sharding("a b/tp, b c -> a c")
    plan = build_binary_transition_plan(x, y, z)
    assert _steps(plan.input1_steps) == [("split_forward_allgather_backward", ("b", "tp"))]
    assert _steps(plan.output_steps) == [("rank_local_einsum", ()), ("allreduce_forward_identity_backward", ("tp",))]
    assert plan.reduction_dims == ("tp",)
    assert _steps(build_binary_transition_plan(*parse_sharding("a b/tp, b c -> a c // tp")).output_steps) == [
        ("rank_local_einsum", ())]

    plan = build_binary_transition_plan(*parse_sharding("a/tp b, c d -> a c/tp"))
    assert _steps(plan.input0_steps) == [("allgather_forward_reducescatter_backward", ("a", "tp"))]
    assert _steps(plan.input1_steps) == [("split_forward_allgather_backward", ("c", "tp"))]
    assert plan.post_repartition.shard_dim == "tp"
    assert [(c.name, c.args) for c in plan.candidates] == [("alltoall_repartition", ("a", "c", "tp"))]
    assert [a.name for a in plan.alternatives] == ["alltoall_repartition", "default"]
    assert plan.alternatives[0].reason == "requires runtime split-shape validation"

    plan = build_binary_transition_plan(*parse_sharding("a/dp k, k/sp b -> a/dp b/sp"))
    assert _steps(plan.input1_steps) == [("identity_forward_allreduce_backward", ("dp",))]
    plan = build_binary_transition_plan(*parse_sharding("a k/dp m/sp, k/sp m/dp b -> a/sp b/dp"))
    assert _steps(plan.input1_steps) == [("owner_swap", (("sp", "dp"), ("dp", "sp")))]
    with pytest.raises(NotImplementedError, match="owner-swap-compatible"):
        build_binary_transition_plan(*parse_sharding("a k/dp m/sp n/dp, k/sp m/dp n/tp b -> a b"))

    cls = classify_binary(*parse_sharding("b/dp a c/sp, b/dp c/sp d -> b/dp a d"))
    assert (cls.free_axes, cls.shared_output_axes, cls.contracted_axes) == (("a", "d"), ("b",), ("c",))
    assert classify_binary(*parse_sharding("a b, b c -> a c d")).output_only_axes == ("d",)


def test_tp_mlp_and_sequence_parallel_plans():
    for expr, names in {
        "b n c, h/tp c -> b n h/tp": ["identity_forward_allreduce_backward", "rank_local_einsum"],
        "b n h/tp, c h/tp -> b n c // tp": ["rank_local_einsum"],
        "l/tp e, e f/tp -> l f/tp": ["allgather_forward_reducescatter_backward", "rank_local_einsum"],
        "l f/tp, f/tp e -> l/tp e": ["rank_local_einsum", "reducescatter_forward_allgather_backward"],
    }.items():
        assert build_binary_transition_plan(*parse_sharding(expr)).names() == names


def test_runtime_costs():
    x, y, z = parse_sharding("a b/tp, b c -> a/tp c")
    plan = build_binary_transition_plan(x, y, z)
    default = next(a for a in plan.alternatives if a.name == "default")
    expanded = next(a for a in plan.alternatives if a.name == "allreduce_then_split")
    infos = (TensorRuntimeInfo(tuple(x.axes), (8, 4), 4), TensorRuntimeInfo(tuple(y.axes), (4, 6), 4),
             TensorRuntimeInfo(tuple(z.axes), (8, 6), 4))
    training = PlanPolicy.from_mode("training")
    d = estimate_alternative_cost(default, *infos, {"tp": 2}, policy=training)
    e = estimate_alternative_cost(expanded, *infos, {"tp": 2}, policy=training)
    assert d.total_bytes == d.forward_bytes + d.backward_bytes
    assert d.total_bytes < e.total_bytes and d.score < e.score
    mem = estimate_alternative_cost(default, *infos, mesh_sizes={"tp": 2}, policy="memory")
    comm = estimate_alternative_cost(default, *infos, mesh_sizes={"tp": 2}, policy="communication")
    assert mem.score != comm.score
    assert estimate_plan_cost(default.output_steps, infos[2], mesh_sizes={"tp": 2}, policy="memory").score > \
        default.cost.score
    uneven_infos = (TensorRuntimeInfo(tuple(x.axes), (5, 8), 4), TensorRuntimeInfo(tuple(y.axes), (8, 6), 4),
                    TensorRuntimeInfo(tuple(z.axes), (3, 6), 4))
    even = estimate_alternative_cost(default, *uneven_infos, mesh_sizes={"tp": 2},
                                     split_shapes={("tp", "a"): (3, 3)}, policy=False)
    uneven = estimate_alternative_cost(default, *uneven_infos, mesh_sizes={"tp": 2},
                                       split_shapes={("tp", "a"): (3, 2)}, policy=False)
    assert uneven.materialized_elements > even.materialized_elements and uneven.forward_bytes > even.forward_bytes
    ranked = rank_alternatives(plan.alternatives, TensorRuntimeInfo(tuple(x.axes), (16, 8), 4),
                               TensorRuntimeInfo(tuple(y.axes), (8, 12), 4),
                               TensorRuntimeInfo(tuple(z.axes), (16, 12), 4), mesh_sizes={"tp": 4})
    assert [a.name for a in ranked] == ["default", "allreduce_then_split"]
    cost = estimate_plan_cost([PlanStep("broadcast_forward_allreduce_backward", ("dp", 0))],
                              TensorRuntimeInfo(tuple(x.axes), (8, 4), 4), policy=False)
    assert cost.collectives == 1 and cost.forward_bytes == 8 * 4 * 4

    x, y, z = parse_sharding("a/tp b, c d -> a c/tp")
    alt = next(a for a in build_binary_transition_plan(x, y, z).alternatives if a.name == "alltoall_repartition")
    small = estimate_alternative_cost(alt, TensorRuntimeInfo(tuple(x.axes), (4, 5), 2),
                                      TensorRuntimeInfo(tuple(y.axes), (6, 7), 2),
                                      TensorRuntimeInfo(tuple(z.axes), (8, 6), 2), mesh_sizes={"tp": 2}, policy=False)
    large = estimate_alternative_cost(alt, TensorRuntimeInfo(tuple(x.axes), (4, 5), 8),
                                      TensorRuntimeInfo(tuple(y.axes), (6, 7), 8),
                                      TensorRuntimeInfo(tuple(z.axes), (8, 6), 8), mesh_sizes={"tp": 2}, policy=False)
    assert large.total_bytes == small.total_bytes * 4 and alt.cost.score == large.score


def test_policies():
    assert resolve_plan_policy(optimize="memory").mode == "memory"
    with pytest.raises(ValueError, match="Unknown optimization policy"):
        resolve_plan_policy(optimize="unknown")
    p = PlanPolicy.from_mode("latency")
    assert resolve_plan_policy(policy=p) is p
    with pytest.raises(ValueError, match="either optimize or policy"):
        resolve_plan_policy(optimize="memory", policy=p)
    set_default_policy(None)
    assert get_default_policy().mode == "training"
    set_default_policy("communication")
    try:
        assert get_optimization_policy().mode == "communication"
        with optimize("memory"):
            assert resolve_plan_policy().mode == "memory"
            with optimize("training"):
                assert get_optimization_policy().mode == "training"
            assert get_optimization_policy().mode == "memory"
        assert get_optimization_policy().mode == "communication"
    finally:
        set_default_policy(None)
    assert PlanPolicy.from_mode("inference").backward_byte_weight == 0


def test_execution_trace():
    plan = ExecutionPlan()
    plan.add("split_forward_allgather_backward", "a", "dp")
    plan.add("rank_local_einsum")
    plan.consider("alltoall_repartition", "a", "b", "dp", status="rejected", reason="missing shapes")
    set_last_plan(plan)
    assert [s.name for s in last_plan()] == plan.names()
    (cand,) = last_candidates()
    assert (cand.name, cand.args, cand.status, cand.reason) == ("alltoall_repartition", ("a", "b", "dp"),
                                                               "rejected", "missing shapes")
    tp = build_binary_transition_plan(*parse_sharding("a b/tp, b c -> a/tp c"))
    plan.rank(tp.alternatives, selected="default", reason="validated")
    set_last_plan(plan)
    assert [(a.name, a.status) for a in last_alternatives()] == [("default", "selected"),
                                                                ("allreduce_then_split", "ranked")]
    result = ExecutionPlan()
    assert result.execute("double", lambda v: v * 2, 3, step_args=("x",)) == 6
    assert [(s.name, s.args) for s in result.snapshot()] == [("double", ("x",))]
    spec = tensor_spec([local_axis("a"), sharded_axis("b", "tp")], partials=("dp",))
    assert spec.axes[1].shard_dim == "tp" and spec.partials == ("dp",)
