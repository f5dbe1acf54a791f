"""Notation data model (module path kept for users of ``es.sharding``).

Reference counterpart: ``src/torch_einshard/sharding.py``.
"""

from .notation.spec import *  # noqa: F401,F403
from .notation.spec import __all__  # noqa: F401
