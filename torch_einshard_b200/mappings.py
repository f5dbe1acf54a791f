"""Autograd-paired collectives (module path kept for users of ``es.mappings``).

Reference counterpart: ``src/torch_einshard/mappings.py:4-199``.
"""

from .parallel.mappings import *  # noqa: F401,F403
from .parallel.mappings import __all__  # noqa: F401
