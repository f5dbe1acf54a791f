"""Parameter metadata: states, validation, merging, registration helpers,
shard metadata, init sync, gradient reduction hooks and the DDP comm hook."""

import pytest
import torch
import torch.distributed as dist
from torch import nn
from torch.nn.parallel import DistributedDataParallel

import torch_einshard_b200 as es
from conftest import assert_close
from dist_harness import run_ranks
from torch_einshard_b200.params import PARAM_STATE_ATTR, parameter_operand_state, register_parameter_state


def _weight(expr):
    return es.parse_sharding(expr)[1]


def test_state_from_annotated_operand():
    st = es.ParameterState.from_spec(_weight("b c, out/tp c [param, grad=async] -> b out/tp"),
                                     mesh_dim_names=("tp", "sp1", "sp2"), source="formula")
    assert (st.source, st.layout_shard_dims, st.init_sync.mode, st.shared) == ("formula", ("tp",), "inferred",
                                                                              ("sp1", "sp2"))
    assert st.grad_comm.pending_inference and st.grad_comm.schedule == "async"
    assert st.tensor_state.replicated_dims == ("sp1", "sp2")
    st = es.ParameterState.from_spec(_weight("b c, out c [param, grad=dp:external, init_sync=none] -> b out"),
                                     mesh_dim_names=("dp", "tp"))
    assert st.init_sync.mode == "none" and st.grad_comm.backend == "external" and st.reduce == ()
    st = es.ParameterState.from_spec(_weight("b c, out c [param, grad=none] -> b out"))
    assert st.grad_comm.mode == "none" and not st.grad_comm.pending_inference


@pytest.mark.parametrize("expr,match", [
    ("b c, out/tp c/tp [param] -> b out", "same mesh dimension"),
    ("b c, out/dp-sp c/sp-dp [param] -> b out", "same mesh dimension"),
    ("b c, out/tp c [param, init_sync=tp] -> b out", "overlaps"),
    ("b c, out/tp c [param, grad=tp] -> b out", "overlaps"),
    ("b c, out/tp c [param, grad=tp:ddp] -> b out", "overlaps"),
])
def test_state_validation_errors(expr, match):
    with pytest.raises(ValueError, match=match):
        es.ParameterState.from_spec(_weight(expr))


def test_external_grad_may_overlap_and_object_validation():
    st = es.ParameterState.from_spec(_weight("b c, out/tp c [param, grad=tp:external] -> b out"))
    assert st.reduce == ()
    p = nn.Parameter(torch.zeros(2, 3))
    with pytest.raises(TypeError, match="ParameterGradComm"):
        register_parameter_state(p, es.ParameterState(spec=None, grad_comm="bad"))
    with pytest.raises(ValueError, match="explicit mode requires mesh_dims"):
        register_parameter_state(p, es.ParameterState(spec=None, init_sync=es.ParameterInitSync(mode="explicit")))
    assert getattr(p, PARAM_STATE_ATTR, None) is None


def test_einshard_registers_operands_atomically():
    weight = nn.Parameter(torch.ones(4, 3))
    z = es.einshard("b c, out c [param] -> b out", torch.ones(2, 3), weight)
    assert z.shape == (2, 4)
    st = es.get_parameter_state(weight)
    assert st.source == "formula" and st.grad_comm.mode == "none"
    with pytest.raises(ValueError, match="different layout"):
        es.einshard("b c, out/tp c [param] -> b out/tp", torch.ones(2, 3), weight, mesh=None)
    assert es.get_parameter_state(weight) is st
    with pytest.raises(TypeError, match="torch.nn.Parameter"):
        es.einshard("b c, out c [param] -> b out", torch.ones(2, 3), torch.ones(4, 3))
    fresh = nn.Parameter(torch.ones(4, 3))
    assert es.einshard_like("b c, out c [param, grad=dp] -> b out", None, fresh) is None
    assert es.get_parameter_state(fresh).grad_comm.mesh_dims == ("dp",)


def test_merge_rules():
    p = nn.Parameter(torch.zeros(3, 4))
    es.register_parameter_layout(p, "o c", grad="async")
    es.register_parameter_layout(p, "o c", grad="dp")
    st = es.get_parameter_state(p)
    assert st.grad_comm.mesh_dims == ("dp",) and st.grad_comm.schedule == "async"
    with pytest.raises(ValueError, match="incompatible metadata"):
        es.register_parameter_layout(p, "o c", grad="sp")
    q = nn.Parameter(torch.zeros(3, 4))
    es.register_parameter_layout(q, "o c", init_sync="none")
    with pytest.raises(ValueError, match="incompatible metadata"):
        es.register_parameter_layout(q, "o c", init_sync="dp")
    with pytest.raises(ValueError, match="rank"):
        es.register_parameter_layout(nn.Parameter(torch.zeros(3)), "o c")
    r = nn.Parameter(torch.zeros(3, 4))
    es.init_param_(r, None, sharded=("tp",))
    with pytest.raises(ValueError, match="different sharded mesh footprint"):
        es.register_parameter_layout(r, "o/sp c")
    es.register_parameter_layout(r, "o/tp c")
    assert es.get_parameter_state(r).spec is not None


def test_module_helpers_and_finalize():
    lin = nn.Linear(3, 4)
    es.register_linear_parameters_(lin, weight_layout="out/tp in", mesh_dim_names=("dp", "tp"))
    assert es.get_parameter_state(lin.bias).layout_shard_dims == ("tp",)
    assert es.get_parameter_state(lin.weight).shared == ("dp",)
    with pytest.raises(ValueError, match="bias layout must match"):
        es.register_linear_parameters_(nn.Linear(3, 4), weight_layout="out in", bias_layout="in")
    conv = nn.Conv2d(2, 3, 3)
    es.register_conv_parameters_(conv, grad="dp")
    assert [a.name for a in es.get_parameter_state(conv.weight).axes] == ["out", "in", "kh", "kw"]
    norm = nn.LayerNorm(5)
    es.register_norm_parameters_(norm, grad="dp")
    assert es.get_parameter_state(norm.bias).grad_comm.mesh_dims == ("dp",)
    mod = nn.Linear(2, 2, bias=False)
    es.register_module_parameter_layouts_(mod, {"weight": "o c"}, grad={"weight": "async"})
    with pytest.raises(ValueError, match="unknown parameter names"):
        es.register_module_parameter_layouts_(mod, {"weight": "o c"}, grad={"nope": "dp"})
    es.finalize_parameter_grad_comm_(mod.weight, "dp")
    assert es.get_parameter_state(mod.weight).grad_comm.mode == "explicit"
    with pytest.raises(ValueError, match="not pending inference"):
        es.finalize_parameter_grad_comm_(mod.weight, "dp")
    with pytest.raises(ValueError, match="pending inference"):
        es.validate_module_parameter_states_(nn.Sequential(nn.Linear(2, 2)).apply(
            lambda m: es.register_module_parameter_layouts_(m, {"weight": "o c"}, grad={"weight": "async"})
            if isinstance(m, nn.Linear) else None))
    st = parameter_operand_state(nn.Parameter(torch.zeros(4, 3)), es.parse_sharding("b/dp c, o c [param] -> b/dp o")[:2],
                                 es.parse_sharding("b/dp c, o c [param] -> b/dp o")[2], 1)
    assert st.grad_comm.mesh_dims == ("dp",)


def _dist_params(ctx):
    mesh2d = ctx.mesh((2, ctx.world_size // 2), ("dp", "sp"))
    wrapped = es.wrap_mesh(mesh2d)
    dp, sp = mesh2d["dp"].get_group(), mesh2d["sp"].get_group()
    # shard metadata
    p = nn.Parameter(torch.zeros(3, 4))
    es.register_parameter_layout(p, "o/sp c", mesh=mesh2d)
    meta = es.param_shard_metadata(p, (10, 4), mesh2d)
    sizes = es.compute_split_shapes(10, dist.get_world_size(sp))
    start = sum(sizes[:dist.get_rank(sp)])
    assert meta.local_slices == (slice(start, start + sizes[dist.get_rank(sp)]), slice(None))
    assert meta.local_shape == (sizes[dist.get_rank(sp)], 4) and meta.shard_dims == ("sp",)
    q = nn.Parameter(torch.zeros(3, 4))
    es.register_parameter_layout(q, "o/dp-sp c", mesh=wrapped)
    size = dist.get_world_size(wrapped["dp-sp"].get_group())
    rank = dist.get_rank(wrapped["dp-sp"].get_group())
    chunks = es.compute_split_shapes(16, size)
    assert es.param_local_slices(q, (16, 4), wrapped)[0] == slice(sum(chunks[:rank]), sum(chunks[:rank + 1]))

    # init sync broadcasts from group rank 0 of every replicated mesh dim
    w = nn.Parameter(torch.full((2, 2), float(dist.get_rank())))
    es.init_param_(w, mesh2d)
    world_rank0 = dist.get_global_rank(dp, 0)
    assert es.get_parameter_state(w).shared == ("dp", "sp")

    # native hooks and explicit reduction
    lin = nn.Linear(1, 1, bias=False)
    lin.weight.data.fill_(1.0)
    es.set_parameter_state(lin.weight, es.ParameterState.from_spec(es.parse_sharding("o c [param, grad=sp] -> o c")[0]))
    handle = es.register_native_grad_reduction_hooks_(lin, mesh2d)
    lin(torch.tensor([[float(dist.get_rank(sp) + 1)]])).sum().backward()
    P = dist.get_world_size(sp)
    assert_close(lin.weight.grad, torch.full_like(lin.weight.grad, float(P * (P + 1) // 2)))
    handle.remove()
    lin.weight.grad = None
    lin(torch.tensor([[1.0]])).sum().backward()
    es.reduce_module_grads_(lin, mesh2d)
    assert_close(lin.weight.grad, torch.full_like(lin.weight.grad, float(P)))

    # DDP comm hook: average over dp, then sum over the parameter's sp group
    for combined in (False, True):
        model = nn.Linear(1, 1, bias=False)
        model.weight.data.fill_(1.0)
        es.set_parameter_state(model.weight, es.ParameterState.from_spec(
            es.parse_sharding("o c [param, grad=sp] -> o c")[0]))
        ddp = DistributedDataParallel(model, process_group=dp)
        if combined:
            es.register_grad_reduction_hook_(ddp, wrapped, ddp_group="dp", combined_reduce_group="dp-sp",
                                             combined_reduce="sp")
        else:
            es.register_grad_reduction_hook_(ddp, mesh2d, ddp_group="dp")
        ddp(torch.tensor([[float(dist.get_rank() + 1)]])).sum().backward()
        D = dist.get_world_size(dp)
        expected = sum(1.0 + r + P * (D - 1) / 2 for r in range(P))
        assert_close(model.weight.grad, torch.full_like(model.weight.grad, expected))
    with pytest.raises(ValueError, match="pending inference"):
        m2 = nn.Linear(1, 1, bias=False)
        es.set_parameter_state(m2.weight, es.ParameterState.from_layout("o c", grad="ddp"))
        es.register_grad_reduction_hook_(DistributedDataParallel(m2, process_group=dp), mesh2d, ddp_group="dp")

    # sharded checkpoint round trip
    import tempfile
    path = tempfile.gettempdir() + "/es_ckpt_test"
    ck = nn.Linear(4, 6, bias=False)
    es.register_parameter_layout(ck.weight, "o/sp c", mesh=mesh2d)
    full = torch.arange(2 * 6 * 4, dtype=torch.float32).reshape(12, 4)[:10]
    sl = es.param_local_slices(ck.weight, (10, 4), mesh2d)
    ck.weight.data = full[sl].clone()
    es.save_sharded(ck, path, mesh2d)
    ck.weight.data.zero_()
    es.load_sharded(ck, path, mesh2d)
    assert_close(ck.weight.data, full[sl])


def test_distributed_params_hooks_ddp_and_checkpoint():
    run_ranks(_dist_params)
