"""Runs transition plans on real tensors: the distributed unary/binary executor.

``distributed_1d`` dispatches a parsed expression to :class:`UnaryExecutor`
(``x -> z``: split / gather / repartition / partial handling) or
:class:`BinaryExecutor` (``x, y -> z``: normalise both operands, contract
locally, then reduce / scatter / repartition the result).  The executors add
the runtime decisions the symbolic plan cannot make alone - owner swaps and
all-to-all repartitions need split metadata that matches the local shapes -
and record what actually ran in an :class:`ExecutionPlan` (``last_plan()``).

Behavioural contract (step names, fallback warnings, error types/texts,
recorded candidates and alternatives): ``src/torch_einshard/distributed.py``
(binary ``:84-620``, unary ``:622-996``).

Fused execution: when the binary plan is ``[identity_forward_allreduce_backward]``
on an operand followed by the local contraction, or the contraction followed
by ``allreduce_forward_identity_backward``, and the operands are CUDA bf16/fp16
tensors on a group with a native communicator, the contraction and its
all-reduce run as one sm_100a kernel (:mod:`..ops.fused`).  The recorded plan
steps are unchanged.
"""

import weakref
import warnings

import torch
import torch.distributed as dist

from ..notation.spec import Axes, Axis, EllipsisAxis, TensorSpec
from ..ops.einsum import einsum
from ..plan.cost import TensorRuntimeInfo, rank_alternatives
from ..plan.policy import resolve_plan_policy
from ..plan.state import PlanStep
from ..plan.trace import ExecutionPlan, set_last_plan
from ..plan.transitions import build_binary_transition_plan, build_unary_transition_plan
from . import mappings as M
from .collectives import resolve_split_shapes

__all__ = ["distributed_1d", "distributed_1d_1", "distributed_1d_2", "expand_unary_ellipsis"]

_FALLBACK_WARNING = (
    "Using gather/split fallback for distributed repartition; this may materialize a larger tensor. "
    "The optimized path currently requires same-mesh axis-to-axis repartition with explicit split metadata."
)


def _axes(spec):
    return spec.axes if hasattr(spec, "axes") else spec


def _partials(spec):
    return getattr(spec, "partials", ())


def _no_ellipsis(axes):
    return Axes(axis for axis in axes if not isinstance(axis, EllipsisAxis))


def expand_unary_ellipsis(input_axes, output_axes, x):
    """Replace ``...`` in a unary expression by ``__ellipsis<i>`` local axes."""
    has_in = any(isinstance(a, EllipsisAxis) for a in input_axes)
    has_out = any(isinstance(a, EllipsisAxis) for a in output_axes)
    if not has_in and not has_out:
        return input_axes, output_axes
    if has_in != has_out:
        raise NotImplementedError("Distributed unary ellipsis requires ellipsis in both input and output")
    width_in = x.dim() - (len(input_axes) - 1)
    width_out = x.dim() - (len(output_axes) - 1)
    if width_in < 0 or width_out < 0 or width_in != width_out:
        raise ValueError("Input tensor rank is incompatible with ellipsis notation")
    filler = [Axis(f"__ellipsis{i}") for i in range(width_in)]

    def expand(axes):
        out = Axes()
        for axis in axes:
            if isinstance(axis, EllipsisAxis):
                out.extend(filler)
            else:
                out.append(axis)
        return out

    return expand(input_axes), expand(output_axes)


def _replace_axis(axes, name, replacement):
    return Axes(
        replacement if not isinstance(axis, EllipsisAxis) and axis.name == name else axis
        for axis in axes
    )


def _dim_of(axes, name, tensor):
    """Tensor dimension of axis ``name`` in ``axes`` (accounts for an ellipsis)."""
    fixed = sum(1 for axis in axes if not isinstance(axis, EllipsisAxis))
    span = tensor.dim() - fixed
    dim = 0
    for axis in axes:
        if isinstance(axis, EllipsisAxis):
            dim += span
        elif axis.name == name:
            return dim
        else:
            dim += 1
    raise ValueError(f"Axis {name!r} is not present in input")


def distributed_1d(shard, *xs, mesh, shapes, policy=None):
    if shard[1] is None:
        return distributed_1d_1(shard, *xs, mesh, shapes, policy=policy)
    return distributed_1d_2(shard, *xs, mesh=mesh, shapes=shapes, policy=policy)


# ============================================================================ binary

_MESH_SIZES = {}  # id(mesh) -> (weakref to the mesh, {dim name: size})



def _binary_fusion(executor):
    """A fused compute + collective kernel for this binary plan (see
    ``ops/fused_native.py:provider``), or None: only while the native
    communicators are active (``setup_native_comm``)."""
    from . import symmetric
    if not symmetric.enabled():
        return None
    from ..ops import fused_native
    return fused_native.provider(executor)

class BinaryExecutor:
    def __init__(self, shard, x, y, mesh, shapes, policy):
        self.plan = ExecutionPlan()
        self.policy = resolve_plan_policy(policy=policy)
        self.mesh, self.shapes = mesh, shapes
        self.x0, self.y0 = x, y
        self.spec0, self.spec1, self.spec_out = shard
        self.axes0 = _no_ellipsis(_axes(self.spec0))
        self.axes1 = _no_ellipsis(_axes(self.spec1))
        self.out_axes = _no_ellipsis(_axes(self.spec_out))
        self.tp = build_binary_transition_plan(
            TensorSpec(self.axes0, _partials(self.spec0)),
            TensorSpec(self.axes1, _partials(self.spec1)),
            TensorSpec(self.out_axes, _partials(self.spec_out)),
        )
        self.by0 = {a.name: a for a in self.axes0}
        self.by1 = {a.name: a for a in self.axes1}
        out_by_name = {a.name: a for a in self.out_axes}
        self.reduction_dims = list(self.tp.reduction_dims)
        # mesh dim -> output Axis object that receives the reduce-scatter
        self.scatter_by_dim = {dim: out_by_name[name] for dim, name in self.tp.scatter_output_by_dim}
        self.post = self._runtime_post_repartition()

    # -- helpers ---------------------------------------------------------
    def group(self, dim):
        return self.mesh[dim].get_group()

    def split_shapes(self, dim, axis_name):
        return resolve_split_shapes(self.shapes, dim, axis_name, self.group(dim))

    def runtime_info(self, axes, tensor):
        return TensorRuntimeInfo(tuple(_no_ellipsis(axes)), tuple(tensor.shape), tensor.element_size())

    def mesh_sizes(self):
        # DeviceMesh.mesh rebuilds a tensor on every access: cache the sizes per mesh object
        mesh = self.mesh
        hit = _MESH_SIZES.get(id(mesh))
        if hit is None or hit[0]() is not mesh:
            sizes = {name: int(mesh.mesh.shape[i]) for i, name in enumerate(mesh.mesh_dim_names)}
            try:
                hit = (weakref.ref(mesh), sizes)
            except TypeError:
                return sizes
            _MESH_SIZES[id(mesh)] = hit
        return dict(hit[1])

    def cost_split_shapes(self):
        known = {}
        for axes in (self.axes0, self.axes1, self.out_axes):
            for axis in axes:
                if isinstance(axis, EllipsisAxis) or not axis.shard_dim:
                    continue
                try:
                    found = resolve_split_shapes(self.shapes, axis.shard_dim, axis.name, self.group(axis.shard_dim))
                except ValueError:
                    continue
                if found is not None:
                    known[(axis.shard_dim, axis.name)] = tuple(found)
        return known

    def _runtime_post_repartition(self):
        gathers, splits = [], []
        for out_axis in self.out_axes:
            sources = [a for a in (self.by0.get(out_axis.name), self.by1.get(out_axis.name)) if a is not None]
            if len(sources) != 1 or sources[0] == out_axis:
                continue
            src = sources[0]
            if src.shard_dim and out_axis.local():
                gathers.append((src, out_axis))
            elif src.local() and out_axis.shard_dim:
                splits.append((src, out_axis))
        if len(gathers) != 1 or len(splits) != 1:
            return None
        (src_in, src_out), (dst_in, dst_out) = gathers[0], splits[0]
        dim = src_in.shard_dim
        if dim != dst_out.shard_dim or dim in self.reduction_dims or dim in _partials(self.spec_out):
            return None
        src_shapes = self.split_shapes(dim, src_in.name)
        dst_shapes = self.split_shapes(dim, dst_out.name)
        if src_shapes is None or dst_shapes is None:
            return None
        return dict(shard_dim=dim, source_input_axis=src_in, source_output_axis=src_out,
                    dest_input_axis=dst_in, dest_output_axis=dst_out,
                    source_shapes=src_shapes, dest_shapes=dst_shapes)

    def runtime_input_steps(self, steps):
        if self.post is None:
            return steps
        src, dst, dim = self.post["source_input_axis"].name, self.post["dest_input_axis"].name, self.post["shard_dim"]
        out = []
        for step in steps:
            if step.args and step.args[0] == src:
                continue
            if step.args and step.args[0] == dst:
                out.append(PlanStep("identity_forward_allreduce_backward", (dim,)))
                continue
            out.append(step)
        return tuple(out)

    # -- operand normalisation -------------------------------------------
    def _owner_swap(self, tensor, axes, step):
        source_dims, dest_dims = step.args
        targets = {}
        for name in self.tp.classification.contracted_axes:
            from ..plan.transitions import contracted_target_axis
            targets[name] = contracted_target_axis(self.by0[name], self.by1[name])
        changes = [
            (axis, targets[axis.name]) for axis in _no_ellipsis(axes)
            if axis.name in targets and axis != targets[axis.name]
            and not axis.local() and not targets[axis.name].local()
        ]
        ok = len(set(source_dims)) == len(source_dims) and len(set(dest_dims)) == len(dest_dims)
        out_shape = list(tensor.shape)
        names = self.mesh.mesh_dim_names
        for axis, target in changes:
            if not ok:
                break
            if self.mesh.mesh.shape[names.index(axis.shard_dim)] != self.mesh.mesh.shape[names.index(target.shard_dim)]:
                ok = False
                break
            src_group, dst_group = self.group(axis.shard_dim), self.group(target.shard_dim)
            src_shapes = resolve_split_shapes(self.shapes, axis.shard_dim, axis.name, src_group)
            dst_shapes = resolve_split_shapes(self.shapes, target.shard_dim, axis.name, dst_group)
            if src_shapes is None or dst_shapes is None or src_shapes != dst_shapes:
                ok = False
                break
            dim = _dim_of(axes, axis.name, tensor)
            if tensor.shape[dim] != src_shapes[dist.get_rank(src_group)]:
                ok = False
                break
            out_shape[dim] = dst_shapes[dist.get_rank(dst_group)]
        if not ok:
            self.plan.consider(step.name, *step.args, status="rejected", reason="runtime owner-swap validation failed")
            set_last_plan(self.plan)
            raise NotImplementedError(
                "Multiple contracted-axis shard-dimension changes require an owner-swap-compatible permutation"
            )
        self.plan.consider(step.name, *step.args, status="accepted")
        tensor = self.plan.execute(step.name, M.owner_swap_forward_backward, tensor, self.mesh,
                                   source_dims, dest_dims, tuple(out_shape), step_args=step.args)
        for axis, target in changes:
            axes = _replace_axis(axes, axis.name, target)
        return tensor, axes

    def normalize(self, tensor, spec, steps, defer_allreduce=None):
        """Apply ``steps`` to one operand; returns ``(tensor, normalised spec)``.

        ``defer_allreduce``: list that receives the group of a trailing
        ``identity_forward_allreduce_backward`` instead of applying it, so the
        caller can fuse that backward all-reduce into the contraction.
        """
        axes = _axes(spec)
        steps = self.runtime_input_steps(steps)
        reduced_backward = {
            s.args[-1] for s in steps
            if s.name in ("allgather_forward_reducescatter_backward", "identity_forward_allreduce_backward")
        }
        for index, step in enumerate(steps):
            if step.name == "owner_swap":
                tensor, axes = self._owner_swap(tensor, axes, step)
                continue
            if step.name == "identity_forward_allreduce_backward":
                (dim,) = step.args
                if defer_allreduce is not None and index == len(steps) - 1:
                    self.plan.add(step.name, *step.args)
                    defer_allreduce.append(self.group(dim))
                    continue
                tensor = self.plan.execute(step.name, M.identity_forward_allreduce_backward, tensor,
                                           self.group(dim), step_args=step.args)
                continue
            if step.name == "broadcast_forward_allreduce_backward":
                dim = step.args[0]
                src = step.args[1] if len(step.args) > 1 else 0
                tensor = self.plan.execute(step.name, M.broadcast_forward_allreduce_backward, tensor,
                                           self.group(dim), src, step_args=step.args)
                continue
            name, dim = step.args
            tdim = _dim_of(axes, name, tensor)
            group = self.group(dim)
            shapes = resolve_split_shapes(self.shapes, dim, name, group)
            if step.name == "split_forward_allgather_backward":
                tensor = self.plan.execute(step.name, M.split_forward_allgather_backward, tensor, group, tdim,
                                           shapes, step_args=step.args)
                axes = _replace_axis(axes, name, Axis(name, dim))
            elif step.name == "allgather_forward_split_backward":
                tensor = self.plan.execute(step.name, M.allgather_forward_split_backward, tensor, group, tdim,
                                           shapes, step_args=step.args)
                axes = _replace_axis(axes, name, Axis(name))
            elif step.name == "allgather_forward_reducescatter_backward":
                tensor = self.plan.execute(step.name, M.allgather_forward_reducescatter_backward, tensor, group,
                                           tdim, shapes, step_args=step.args)
                axes = _replace_axis(axes, name, Axis(name))
            else:
                raise NotImplementedError(f"Unsupported binary input plan step {step.name!r}")

        names = {a.name for a in _no_ellipsis(axes)}
        own_dims = {a.shard_dim for a in _no_ellipsis(axes) if a.shard_dim}
        extra = []
        for out_axis in self.out_axes:
            dim = out_axis.shard_dim
            if not dim or out_axis.name in names:
                continue
            if dim in self.reduction_dims or dim in own_dims or dim in reduced_backward:
                continue
            if dim not in extra:
                extra.append(dim)
        for dim in extra:
            tensor = self.plan.execute("identity_forward_allreduce_backward", M.identity_forward_allreduce_backward,
                                       tensor, self.group(dim), step_args=(dim,))
        return tensor, TensorSpec(axes, _partials(spec))

    def _localize(self, axis):
        if self.scatter_by_dim.get(axis.shard_dim) == axis:
            axis = Axis(axis.name)
        if self.post is not None:
            if axis == self.post["source_output_axis"]:
                return self.post["source_input_axis"]
            if axis == self.post["dest_output_axis"]:
                return self.post["dest_input_axis"]
        return axis

    # -- main ------------------------------------------------------------
    def run(self):
        plan, tp = self.plan, self.tp
        plan.rank(tp.alternatives, selected=None if self.post is not None else "default", reason="fallback selected")
        if self.post is None:
            for candidate in tp.candidates:
                if candidate.name == "alltoall_repartition":
                    plan.consider(candidate, status="rejected", reason="runtime split-shape validation failed")

        fuse = _binary_fusion(self)
        deferred0 = [] if fuse is not None and fuse.kind == "dgrad_allreduce" and fuse.operand == 0 else None
        deferred1 = [] if fuse is not None and fuse.kind == "dgrad_allreduce" and fuse.operand == 1 else None
        if fuse is not None and fuse.kind == "allgather_gemm":
            z = self._run_allgather_gemm(fuse)
            if z is not None:
                return z
        x, spec0 = self.normalize(self.x0, self.spec0, tp.input0_steps, deferred0)
        y, spec1 = self.normalize(self.y0, self.spec1, tp.input1_steps, deferred1)
        local_out_axes = Axes(
            self._localize(a) if not isinstance(a, EllipsisAxis) else a for a in _axes(self.spec_out)
        )
        local_out = TensorSpec(local_out_axes, _partials(self.spec_out))
        by0 = {a.name: a for a in _no_ellipsis(_axes(spec0))}
        by1 = {a.name: a for a in _no_ellipsis(_axes(spec1))}
        local_by_name = {a.name: a for a in _no_ellipsis(local_out_axes)}
        out_names = {a.name for a in self.out_axes}
        for name in [a.name for a in _no_ellipsis(_axes(spec0)) if a.name in by1 and a.name in out_names]:
            assert by0[name] == by1[name], "Shared axes must use matching sharding"
            assert by0[name] == local_by_name[name], "Output shared axes must preserve input sharding"

        plan.add("rank_local_einsum")
        output_steps = [s for s in tp.output_steps if s.name not in ("rank_local_einsum", "alltoall_repartition")]
        fused_out = False
        fused_rs = None
        if fuse is not None and fuse.kind == "gemm_reducescatter" and len(output_steps) == 1 and \
                output_steps[0].name == "reducescatter_forward_allgather_backward" and self._even_split(output_steps[0]):
            name, dim = output_steps[0].args
            fused_rs = fuse.run_gemm_reducescatter((spec0, spec1, local_out), x, y, self.group(dim), name)
        if fused_rs is not None:
            z = fused_rs
        elif fuse is not None and fuse.kind == "gemm_allreduce" and output_steps and \
                output_steps[0].name == "allreduce_forward_identity_backward":
            z = fuse.run_gemm_allreduce((spec0, spec1, local_out), x, y, self.group(output_steps[0].args[0]))
            fused_out = True
        elif fuse is not None and fuse.kind == "dgrad_allreduce" and (deferred0 or deferred1):
            group = (deferred0 or deferred1)[0]
            z = fuse.run_dgrad_allreduce((spec0, spec1, local_out), x, y, group)
        else:
            if deferred0:
                x = M.identity_forward_allreduce_backward(x, deferred0[0])
            if deferred1:
                y = M.identity_forward_allreduce_backward(y, deferred1[0])
            z = einsum((spec0, spec1, local_out), x, y)

        current = local_out_axes
        if self.post is None:
            ranked = rank_alternatives(
                tp.alternatives,
                self.runtime_info(self.axes0, self.x0), self.runtime_info(self.axes1, self.y0),
                self.runtime_info(local_out_axes, z), self.mesh_sizes(), self.cost_split_shapes(), self.policy,
            )
            plan.rank(ranked, selected="default", reason="fallback selected")
        else:
            ranked = rank_alternatives(
                tp.alternatives,
                self.runtime_info(self.axes0, self.x0), self.runtime_info(self.axes1, self.y0),
                mesh_sizes=self.mesh_sizes(), split_shapes=self.cost_split_shapes(), policy=self.policy,
                output_infos={"alltoall_repartition": self.runtime_info(local_out_axes, z)},
            )
            plan.rank(ranked)

        for index, step in enumerate(output_steps):
            if fused_rs is not None and index == 0:
                # already reduce-scattered by the fused kernel
                plan.add(step.name, *step.args)
                current = _replace_axis(current, step.args[0], self.scatter_by_dim[step.args[1]])
                continue
            if step.name == "allreduce_forward_identity_backward":
                if fused_out and index == 0:
                    plan.add(step.name, *step.args)
                    continue
                (dim,) = step.args
                z = plan.execute(step.name, M.allreduce_forward_identity_backward, z, comm=self.group(dim),
                                 step_args=step.args)
                continue
            name, dim = step.args
            target_axis = self.scatter_by_dim[dim]
            tdim = _dim_of(current, name, z)
            group = self.group(dim)
            shapes = resolve_split_shapes(self.shapes, dim, name, group)
            if step.name == "split_forward_allgather_backward":
                z = plan.execute(step.name, M.split_forward_allgather_backward, z, group, tdim, shapes,
                                 step_args=step.args)
            elif step.name == "reducescatter_forward_allgather_backward":
                z = plan.execute(step.name, M.reducescatter_forward_allgather_backward, z, group, tdim, shapes,
                                 step_args=step.args)
            else:
                raise NotImplementedError(f"Unsupported binary output plan step {step.name!r}")
            current = _replace_axis(current, name, target_axis)

        if self.post is not None:
            z = self._post_repartition(z, current, ranked)
        set_last_plan(plan)
        return z

    def _even_split(self, step):
        name, dim = step.args
        group = self.group(dim)
        shapes = resolve_split_shapes(self.shapes, dim, name, group)
        return shapes is None or len(set(shapes)) == 1

    def _run_allgather_gemm(self, fuse):
        """AG of operand 0 along a GEMM row axis + the contraction, as one fused op
        (its backward is the fused GEMM + reduce-scatter).  None: run unfused."""
        tp, plan = self.tp, self.plan
        step = tp.input0_steps[0]
        name, dim = step.args
        if not self._even_split(step) or any(isinstance(a, EllipsisAxis) for a in _axes(self.spec0)) or \
                any(isinstance(a, EllipsisAxis) for a in _axes(self.spec1)) or \
                any(isinstance(a, EllipsisAxis) for a in _axes(self.spec_out)):
            return None
        axes0 = list(_axes(self.spec0))
        tdim = [a.name for a in axes0].index(name)
        spec0 = TensorSpec(Axes(Axis(a.name) if a.name == name else a for a in axes0), _partials(self.spec0))
        local_out_axes = Axes(self._localize(a) for a in _axes(self.spec_out))
        local_out = TensorSpec(local_out_axes, _partials(self.spec_out))
        z = fuse.run_allgather_gemm((spec0, self.spec1, local_out), self.x0, self.y0, self.group(dim), name, tdim)
        if z is None:
            return None
        plan.add(step.name, *step.args)
        plan.add("rank_local_einsum")
        ranked = rank_alternatives(
            tp.alternatives,
            self.runtime_info(self.axes0, self.x0), self.runtime_info(self.axes1, self.y0),
            self.runtime_info(local_out_axes, z), self.mesh_sizes(), self.cost_split_shapes(), self.policy,
        )
        plan.rank(ranked, selected="default", reason="fallback selected")
        set_last_plan(plan)
        return z

    def _post_repartition(self, z, current, ranked):
        post, plan = self.post, self.plan
        group = self.group(post["shard_dim"])
        rank = dist.get_rank(group)
        src_name, dst_name = post["source_input_axis"].name, post["dest_input_axis"].name
        src_dim, dst_dim = _dim_of(current, src_name, z), _dim_of(current, dst_name, z)
        local_ok = z.shape[src_dim] == post["source_shapes"][rank] and z.shape[dst_dim] == sum(post["dest_shapes"])
        flag = torch.tensor(int(local_ok), device=z.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        args = (src_name, dst_name, post["shard_dim"])
        if not bool(flag.item()):
            plan.rank(ranked)
            plan.consider("alltoall_repartition", *args, status="rejected",
                          reason="runtime tensor shape does not match split metadata")
            set_last_plan(plan)
            raise ValueError("Runtime tensor shape does not match alltoall_repartition split metadata")
        result = M.alltoall_repartition(z, group, src_dim, dst_dim, post["source_shapes"], post["dest_shapes"])
        if result is None:
            plan.rank(ranked)
            plan.consider("alltoall_repartition", *args, status="rejected", reason="alltoall_repartition returned None")
            set_last_plan(plan)
            raise ValueError("Runtime tensor shape does not match alltoall_repartition split metadata")
        plan.rank(ranked, selected="alltoall_repartition", reason="runtime split-shape validation passed")
        plan.consider("alltoall_repartition", *args, status="accepted")
        plan.add("alltoall_repartition", *args)
        return result


def distributed_1d_2(shard, x, y, mesh, shapes=None, policy=None):
    return BinaryExecutor(shard, x, y, mesh, shapes, policy).run()


# ============================================================================= unary

class UnaryExecutor:
    def __init__(self, shard, x, mesh, shapes, policy):
        self.plan = ExecutionPlan()
        resolve_plan_policy(policy=policy)
        self.shard, self.mesh, self.shapes = shard, mesh, shapes
        in_axes, out_axes = expand_unary_ellipsis(_axes(shard[0]), _axes(shard[2]), x)
        self.in_axes, self.out_axes = in_axes, out_axes
        self.in_partials = list(_partials(shard[0]))
        self.out_partials = list(_partials(shard[2]))
        assert len(in_axes) == len(out_axes), "Input and output dimensions must match in the equation"
        if not (x.dim() == 0 and len(in_axes) == 1 and in_axes[0].name == out_axes[0].name):
            assert len(in_axes) == x.dim(), "Input dimensions must match those in the equation"
        self.in_by = {a.name: a for a in in_axes}
        self.out_by = {a.name: a for a in out_axes}
        assert self.in_by.keys() == self.out_by.keys(), "Input and output axes must match"
        self.tp = build_unary_transition_plan(
            TensorSpec(in_axes, tuple(self.in_partials)), TensorSpec(out_axes, tuple(self.out_partials))
        )
        self.z = x
        self.current = list(in_axes)
        self.partials = list(self.in_partials)
        self.changed = [
            a.name for a in out_axes
            if self.in_by[a.name].shard_dim and a.shard_dim and self.in_by[a.name].shard_dim != a.shard_dim
        ]

    def group(self, dim):
        return self.mesh[dim].get_group()

    def dim_of(self, name):
        return next(i for i, a in enumerate(self.current) if a.name == name)

    def split_shapes(self, dim, name):
        return resolve_split_shapes(self.shapes, dim, name, self.group(dim))

    def _swap_validation(self, pairs, source_dims, dest_dims):
        """Output shape of an owner swap, or None when metadata does not allow it."""
        if len(set(source_dims)) != len(source_dims) or len(set(dest_dims)) != len(dest_dims):
            return None
        names = self.mesh.mesh_dim_names
        shape = list(self.z.shape)
        for a, b in pairs:
            if self.mesh.mesh.shape[names.index(a.shard_dim)] != self.mesh.mesh.shape[names.index(b.shard_dim)]:
                return None
            src_group, dst_group = self.group(a.shard_dim), self.group(b.shard_dim)
            src = resolve_split_shapes(self.shapes, a.shard_dim, a.name, src_group)
            dst = resolve_split_shapes(self.shapes, b.shard_dim, b.name, dst_group)
            if src is None or dst is None or src != dst:
                return None
            if self.z.shape[self.dim_of(a.name)] != src[dist.get_rank(src_group)]:
                return None
            shape[self.dim_of(b.name)] = dst[dist.get_rank(dst_group)]
        return shape

    def step(self, step):
        plan, name = self.plan, step.name
        if name == "allreduce_forward_identity_backward":
            (partial,) = step.args
            self.z = plan.execute(name, M.allreduce_forward_identity_backward, self.z, self.group(partial),
                                  step_args=step.args)
            self.partials.remove(partial)
        elif name in ("reducescatter_forward_allgather_backward", "split_forward_allgather_backward",
                      "allgather_forward_split_backward", "allgather_forward_reducescatter_backward"):
            axis_name, dim = step.args
            tdim = self.dim_of(axis_name)
            fn = {
                "reducescatter_forward_allgather_backward": M.reducescatter_forward_allgather_backward,
                "split_forward_allgather_backward": M.split_forward_allgather_backward,
                "allgather_forward_split_backward": M.allgather_forward_split_backward,
                "allgather_forward_reducescatter_backward": M.allgather_forward_reducescatter_backward,
            }[name]
            self.z = plan.execute(name, fn, self.z, self.group(dim), tdim, self.split_shapes(dim, axis_name),
                                  step_args=step.args)
            if name in ("reducescatter_forward_allgather_backward", "split_forward_allgather_backward"):
                self.current[tdim] = self.out_by[axis_name]
            else:
                self.current[tdim] = Axis(axis_name)
            if name == "reducescatter_forward_allgather_backward":
                self.partials.remove(dim)
            elif name == "allgather_forward_reducescatter_backward":
                self.partials.append(dim)
        elif name == "identity_forward_allreduce_backward":
            (partial,) = step.args
            self.z = plan.execute(name, M.identity_forward_allreduce_backward, self.z, self.group(partial),
                                  step_args=step.args)
            self.partials.append(partial)
        elif name == "broadcast_forward_allreduce_backward":
            dim = step.args[0]
            src = step.args[1] if len(step.args) > 1 else 0
            self.z = plan.execute(name, M.broadcast_forward_allreduce_backward, self.z, self.group(dim), src,
                                  step_args=step.args)
        elif name == "owner_swap":
            self._planned_owner_swap(step)
        elif name == "permute":
            plan.add(name, *step.args)
            self.z = einsum(self.shard, self.z, name_only=True)
            self.current = list(self.out_axes)
        else:
            raise NotImplementedError(f"Unsupported unary plan step {name!r}")

    def _planned_owner_swap(self, step):
        source_dims, dest_dims = step.args
        pairs = [
            (self.in_by[n], self.out_by[n]) for n in self.changed
            if self.in_by[n].shard_dim in source_dims and self.out_by[n].shard_dim in dest_dims
        ]
        shape = self._swap_validation(pairs, source_dims, dest_dims)
        if shape is None:
            warnings.warn(_FALLBACK_WARNING, RuntimeWarning, stacklevel=4)
            for a, _ in pairs:
                tdim = self.dim_of(a.name)
                self.z = self.plan.execute("allgather_forward_split_backward", M.allgather_forward_split_backward,
                                           self.z, self.group(a.shard_dim), tdim,
                                           self.split_shapes(a.shard_dim, a.name), step_args=(a.name, a.shard_dim))
                self.current[tdim] = Axis(a.name)
            for _, b in pairs:
                tdim = self.dim_of(b.name)
                self.z = self.plan.execute("split_forward_allgather_backward", M.split_forward_allgather_backward,
                                           self.z, self.group(b.shard_dim), tdim,
                                           self.split_shapes(b.shard_dim, b.name), step_args=(b.name, b.shard_dim))
                self.current[tdim] = b
            return
        self.z = self.plan.execute("owner_swap", M.owner_swap_forward_backward, self.z, self.mesh, source_dims,
                                   dest_dims, tuple(shape), step_args=step.args)
        for a, b in pairs:
            self.current[self.dim_of(a.name)] = b

    def _has_repartition_change(self):
        gathered = split = 0
        across = False
        for b in self.out_axes:
            a = self.in_by[b.name]
            if a.shard_dim == b.shard_dim:
                continue
            if a.shard_dim and b.shard_dim:
                across = True
            elif a.shard_dim:
                gathered += 1
            elif b.shard_dim:
                split += 1
        return across or (gathered > 0 and split > 0)

    def _same_order(self):
        return [a.name for a in self.in_axes] == [a.name for a in self.out_axes]

    def _try_repartition(self):
        if self.out_partials or not self._same_order():
            return None
        gathers, splits = [], []
        for b in self.out_axes:
            a = self.in_by[b.name]
            if a.shard_dim == b.shard_dim:
                continue
            if a.shard_dim and b.local():
                gathers.append(a)
            elif a.local() and b.shard_dim:
                splits.append(b)
        if len(gathers) != 1 or len(splits) != 1 or gathers[0].shard_dim != splits[0].shard_dim:
            return None
        src, dst = gathers[0], splits[0]
        group = self.group(src.shard_dim)
        result = M.alltoall_repartition(self.z, group, self.dim_of(src.name), self.dim_of(dst.name),
                                        self.split_shapes(src.shard_dim, src.name),
                                        self.split_shapes(dst.shard_dim, dst.name))
        if result is not None:
            self.plan.add("alltoall_repartition", src.name, dst.name, src.shard_dim)
        return result

    def _try_owner_swap(self):
        if self.out_partials or not self._same_order() or not self.changed:
            return None
        pairs = [(self.in_by[n], self.out_by[n]) for n in self.changed]
        source_dims = tuple(a.shard_dim for a, _ in pairs)
        dest_dims = tuple(b.shard_dim for _, b in pairs)
        if len(set(source_dims)) != len(source_dims) or len(set(dest_dims)) != len(dest_dims):
            return None
        if len(pairs) > 1 and set(source_dims) != set(dest_dims):
            return None
        involved = set(source_dims) | set(dest_dims)
        for a, b in zip(self.in_axes, self.out_axes):
            if a.name not in self.changed and (a.shard_dim in involved or b.shard_dim in involved):
                return None
        shape = self._swap_validation(pairs, source_dims, dest_dims)
        if shape is None:
            return None
        return self.plan.execute("owner_swap", M.owner_swap_forward_backward, self.z, self.mesh, source_dims,
                                 dest_dims, tuple(shape), step_args=(source_dims, dest_dims))

    def run(self):
        remaining = list(self.tp.steps)
        while remaining and remaining[0].name in ("allreduce_forward_identity_backward",
                                                  "reducescatter_forward_allgather_backward"):
            self.step(remaining.pop(0))
        planned_swap = any(s.name == "owner_swap" for s in remaining)
        swapped = None if planned_swap else self._try_owner_swap()
        swap_applied = False
        if swapped is not None:
            self.z = swapped
            for name in self.changed:
                self.current[self.dim_of(name)] = self.out_by[name]
            remaining = [s for s in remaining if not s.args or s.args[0] not in self.changed]
            swap_applied = True
        repartitioned = self._try_repartition()
        if repartitioned is not None:
            self.z = repartitioned
            self.current = list(self.out_axes)
            set_last_plan(self.plan)
            return self.z
        if self._has_repartition_change() and not swap_applied and not planned_swap:
            warnings.warn(_FALLBACK_WARNING, RuntimeWarning, stacklevel=4)
        for step in remaining:
            self.step(step)
        if [a.name for a in self.current] == [a.name for a in self.out_axes]:
            set_last_plan(self.plan)
            return self.z
        raise AssertionError("Unary symbolic plan did not produce the requested output axes")


def distributed_1d_1(shard, x, mesh, shapes=None, policy=None):
    return UnaryExecutor(shard, x, mesh, shapes, policy).run()
