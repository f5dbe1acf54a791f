"""Notation data model (module path kept for users of ``es.sharding``)."""

from .notation.spec import *  # noqa: F401,F403
from .notation.spec import __all__  # noqa: F401
