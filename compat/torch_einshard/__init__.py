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

for _name in ("helpers", "mappings", "grammar", "sharding", "symbolic", "families", "params", "einsum", "fft",
              "halo", "conv", "roll", "mesh", "distributed"):
    _module = sys.modules.get(f"torch_einshard_b200.{_name}") or importlib.import_module(f"torch_einshard_b200.{_name}")
    sys.modules[f"{__name__}.{_name}"] = _module

del _key, _name, _module
