"""Fused contraction + collective paths selected by the binary executor.

``binary_fusion(executor)`` inspects a binary plan and returns a fusion
descriptor when one of the patterns below applies and the operands can run on
the native NVLink path (CUDA bf16/fp16 tensors, a native communicator for the
group); otherwise ``None`` and the executor runs the unfused steps.

* ``gemm_allreduce``  - ``rank_local_einsum`` then ``allreduce_forward_identity_backward``
  (row-parallel ``b n h/tp, c h/tp -> b n c``): one kernel computes the GEMM
  tiles and all-reduces them over peer memory as they finish.
* ``dgrad_allreduce`` - ``identity_forward_allreduce_backward`` on an operand
  then ``rank_local_einsum`` (column-parallel ``b n c, h/tp c -> b n h/tp``):
  forward is the plain GEMM, and backward's input-gradient GEMM is fused with
  the all-reduce of that gradient.

Fuses the planner steps ``rank_local_einsum`` +
``allreduce_forward_identity_backward`` /
``reducescatter_forward_allgather_backward`` and
``allgather_forward_reducescatter_backward`` + ``rank_local_einsum``
(``src/torch_einshard/mappings.py:169-187``,
``src/torch_einshard/distributed.py:84-620``).
"""

__all__ = ["binary_fusion", "register_fusion_provider"]

_provider = {"fn": None}


def register_fusion_provider(fn):
    """Install the function that builds fusion descriptors (native module)."""
    _provider["fn"] = fn


def binary_fusion(executor):
    fn = _provider["fn"]
    if fn is None:
        return None
    return fn(executor)
