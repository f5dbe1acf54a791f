"""Parameter metadata, init sync, gradient communication and shard metadata."""

from .state import (
    PARAM_STATE_ATTR,
    NativeGradReductionHandle,
    ParameterGradComm,
    ParameterInitSync,
    ParameterState,
    ParamShardMetadata,
)
from .state import check_known_groups as _validate_known_mesh_groups
from .state import check_state_rank as _validate_parameter_state_rank
from .state import mesh_dim_names_from as _mesh_dim_names_from
from .registry import (
    finalize_module_parameter_grad_comm_,
    finalize_parameter_grad_comm_,
    get_parameter_state,
    iter_parameter_states,
    parameter_operand_state,
    register_conv_parameters_,
    register_linear_parameters_,
    register_module_parameter_layouts_,
    register_norm_parameters_,
    register_parameter_layout,
    register_parameter_operand,
    register_parameter_state,
    set_parameter_state,
    validate_module_parameter_states_,
)
from .registry import attached_state as _parameter_state_from_attached_metadata
from .registry import merge_parameter_state as _merge_parameter_state
from .comm import (
    init_param_,
    init_params_,
    reduce_grad_,
    reduce_module_grads_,
    register_grad_reduction_hook_,
    register_native_grad_reduction_hooks_,
    sync_module_params_,
    sync_param_,
)
from .shard_meta import param_local_shape, param_local_slices, param_shard_dims, param_shard_metadata
from .ckpt import load_sharded, save_sharded
