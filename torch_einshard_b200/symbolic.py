"""Flat namespace of the symbolic planner (same module path role as the reference's
``torch_einshard.symbolic``)."""

from .plan import *  # noqa: F401,F403
from .plan import __dict__ as _plan_namespace

__all__ = [name for name in _plan_namespace if not name.startswith("_")]
