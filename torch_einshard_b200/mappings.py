"""Autograd-paired collectives (module path kept for users of ``es.mappings``)."""

from .parallel.mappings import *  # noqa: F401,F403
from .parallel.mappings import __all__  # noqa: F401
