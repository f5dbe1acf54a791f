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
from .parallel.setup import setup_native_comm
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
from . import helpers, mappings, grammar, sharding, symbolic, families  # noqa: F401  (module aliases)

__version__ = "0.1.0"

# Module paths of the reference package (``torch_einshard.fft``, ``.einsum``, ...)
# name the implementation modules here, so code and tests that patch
# ``<package>.fft._distributed_fft_1d_no_autograd`` and the like keep working.
import sys as _sys

from .ops import conv as _conv_mod, einsum as _einsum_mod, fft as _fft_mod, halo as _halo_mod, roll as _roll_mod
from .parallel import executor as _executor_mod, mesh as _mesh_mod

for _alias, _module in (("fft", _fft_mod), ("halo", _halo_mod), ("conv", _conv_mod), ("roll", _roll_mod),
                        ("einsum", _einsum_mod), ("distributed", _executor_mod), ("mesh", _mesh_mod)):
    _sys.modules.setdefault(f"{__name__}.{_alias}", _module)
del _alias, _module
