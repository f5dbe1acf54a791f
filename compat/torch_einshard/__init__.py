"""Drop-in import name for code written against the reference package.

With ``compat`` on ``PYTHONPATH``, ``import torch_einshard as es`` gives this
framework's API under the reference's package name, and its module paths
(``torch_einshard.symbolic``, ``.params``, ``.fft``, ``.halo``, ``.helpers``,
...) name the corresponding modules here, so existing code, monkeypatches in
tests and pickled references keep working unchanged.
"""

import importlib
import sys

import torch_einshard_b200 as _pkg

for _key in dir(_pkg):
    if not _key.startswith("__"):
        globals()[_key] = getattr(_pkg, _key)

# reference module path -> the module here that implements it
_PATHS = {
    "helpers": "parallel.collectives",
    "mappings": "parallel.mappings",
    "grammar": "notation.parser",
    "sharding": "notation.spec",
    "families": "notation.families",
    "symbolic": "plan",
    "params": "params",
    "einsum": "ops.einsum",
    "fft": "ops.fft",
    "halo": "ops.halo",
    "conv": "ops.conv",
    "roll": "ops.roll",
    "mesh": "parallel.mesh",
    "distributed": "parallel.executor",
}
for _name, _path in _PATHS.items():
    _module = importlib.import_module(f"torch_einshard_b200.{_path}")
    sys.modules[f"{__name__}.{_name}"] = _module
    globals()[_name] = _module

del _path
del _key, _name, _module
