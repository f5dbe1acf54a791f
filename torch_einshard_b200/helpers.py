"""Collective helpers (module path kept for users of ``es.helpers``).

Reference counterpart: ``src/torch_einshard/helpers.py:5-354`` (process-group
bootstrap, collective helpers, split shapes).
"""

import torch  # noqa: F401  (exposed for callers that patch torch.cuda through this module)
import torch.distributed as dist  # noqa: F401

from .parallel.collectives import (  # noqa: F401
    all_gather,
    all_reduce,
    all_to_all_repartition,
    broadcast,
    compute_split_shapes,
    compute_split_shapes_for_factors,
    init_process_group,
    owner_swap,
    reduce_scatter,
    resolve_split_shapes,
    roll_sharded,
    roll_shards,
    split,
)
