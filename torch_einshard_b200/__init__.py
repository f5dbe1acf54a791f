"""torch_einshard_b200: einsum-style notation for local and distributed tensor ops,
built for B200 (sm_100a) with native tcgen05 kernels and NVLink collectives.

Public API parity with the reference ``torch_einshard`` package
(``src/torch_einshard/__init__.py:1-372``): ``einshard``, ``einshard_like``,
``einfft``, ``einhalo``, ``einwindow``, ``einconv``, ``einroll``, mesh
wrapping, planner/policy/trace helpers and parameter metadata utilities.
"""

from . import params as _params
from .notation.families import cached_expand_axis_families
from .notation.parser import parse_sharding
from .notation.spec import Axes, AxisGroup, EllipsisAxis, TensorSpec
from .ops.conv import einconv
from .ops.einsum import einsum
from .ops.fft import einfft
from .ops.halo import einhalo, einwindow
from .ops.roll import einroll
from .parallel.executor import distributed_1d
from .parallel.mesh import CompoundDeviceMesh, wrap_mesh
from .parallel.collectives import compute_split_shapes, compute_split_shapes_for_factors, init_process_group, resolve_split_shapes
from .parallel.symmetric import setup_native_comm, teardown_native_comm
from .params import (
    NativeGradReductionHandle,
    ParameterGradComm,
    ParameterInitSync,
    ParameterState,
    ParamShardMetadata,
    finalize_module_parameter_grad_comm_,
    finalize_parameter_grad_comm_,
    get_parameter_state,
    init_param_,
    init_params_,
    iter_parameter_states,
    load_sharded,
    param_local_shape,
    param_local_slices,
    param_shard_dims,
    param_shard_metadata,
    parameter_operand_state,
    reduce_grad_,
    reduce_module_grads_,
    register_conv_parameters_,
    register_grad_reduction_hook_,
    register_linear_parameters_,
    register_module_parameter_layouts_,
    register_native_grad_reduction_hooks_,
    register_norm_parameters_,
    register_parameter_layout,
    register_parameter_operand,
    register_parameter_state,
    save_sharded,
    set_parameter_state,
    sync_module_params_,
    sync_param_,
    validate_module_parameter_states_,
)
from .plan.policy import (
    PlanPolicy,
    get_default_policy,
    get_optimization_policy,
    optimize,
    resolve_plan_policy,
    set_default_policy,
)
from .plan.state import TensorState
from .plan.trace import ExecutionPlan, last_alternatives, last_candidates, last_plan, set_last_plan
from .plan.transitions import build_binary_transition_plan, build_unary_transition_plan
from .api import einshard, einshard_like, local_operation

__version__ = "0.1.0"

